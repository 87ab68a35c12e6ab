// INT4 group-wise dequant-matmul for decode-sized M, the storage dequantizer and the
// quantizer.
//
// Replaces the reference's memory-mode projection path (model.py:15-21 default
// memory_efficient=True; kernels/matmul.py:14-132 `_fused_int4_matmul`), its
// storage dequant (kernels/matmul.py:309-326 `_dequant_storage`, loader.py:157-190
// `dequantize_int4`) and its quantizer (loader.py:9-41 `quantize_int4_groupwise`).
//
// Weight format (loader.py:9-41): packed int8 [N, K/2], byte j of row n holds
// w[n, 2j] in its low nibble and w[n, 2j+1] in its high nibble, two's complement in
// [-8, 7]; scales fp16 [N, K/groupsize]. A weight is fp16(q * scale) (one rounding),
// exactly as the reference computes it; products and sums are fp32, output fp16.
//
// fi_int4_gemm (M <= 64) streams the 4-bit weights once from HBM:
// * Persistent CTAs of one or two groups of (one producer warp + 8 consumer warps)
//   sharing x staged in shared memory. Each group's producer streams
//   R-row x 512-byte weight tiles (1024 k; R = 16, or 8 where that balances the SMs)
//   with TMA into a shared-memory ring (one 3-D box of 4 x 128-byte chunks per tile,
//   128B-swizzled so the consumers' 16-byte reads are conflict-free); each consumer
//   warp takes 128 k of every tile.
// * Nibbles become fp16 without a conversion instruction: lop3 drops a nibble (sign
//   bit flipped) into the mantissa of 1024.0 (0x6400) in each half of a register, an
//   exact f16x2 subtract / fma removes the offset, and an f16x2 multiply by the group
//   scale gives fp16(q * scale) with the reference's single rounding.
// * mma.sync m16n8k16 computes C^T = W x^T: the 16 weight rows are the MMA's M, the
//   tokens its N (tiles of 8), so a decode batch of up to 8 tokens costs two MMAs per
//   32-bit weight word and no padding. The 8 warps' partial sums are added in warp
//   order through shared memory (deterministic); no scratch memory is used.
#include <cuda_fp16.h>

#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kI4Consumers = 8;                         // math warps of a group
constexpr int kI4Threads = (kI4Consumers + 1) * 32;     // + one TMA producer warp
constexpr int kI4Rows = 16;        // weight rows (output columns) per work item, at most
constexpr int kI4KIter = 128;      // k per consumer warp per round: 4 threads x 32 nibbles
constexpr int kI4RoundK = kI4Consumers * kI4KIter;      // 1024 k per round
constexpr int kI4BoxBytes = 128;   // one 128B-swizzled TMA box: R rows x 128 packed bytes
constexpr int kI4Boxes = kI4RoundK / 2 / kI4BoxBytes;   // 4 boxes per stage
#ifndef FI_I4_STAGES
#define FI_I4_STAGES 6
#endif
constexpr int kI4Stages = FI_I4_STAGES;
constexpr int kI4XBatch = 8;      // x chunks each thread loads at once when staging
constexpr int kI4MaxM = 64;        // up to eight 8-token tiles
constexpr int kI4ConsumerBar = 1;  // named barrier of the 256 consumer threads
constexpr int kI4XRItems = 2;      // most items per slot when x is staged round by round

struct I4Args {
  const __half* x;
  const __half* s;
  __half* c;
  int* err;
  int M, N, K, gs, gs_shift;  // gs_shift = log2(gs) for a power of two, else -1
  int rounds, xstride;        // k rounds of 1024; staged x row stride (halves)
  int tma3d;                  // 1: one 3-D box per stage (K % 256 == 0), 0: four 2-D boxes
  int tma_scales;             // 1: each round's 16 x 8 scales arrive by TMA with its weights
  int64_t xs0, ss0, ss1, cs0, cs1;
};

// A work item is R = 16 weight rows (the whole M of the m16n8k16 A operand) or R = 8
// (rows 8-15 of the A operand zero; batches of up to 8 tokens): where 16-row items
// leave some SMs one item more than others, 8-row items halve that overhang. An R-row
// stage is R x 512 bytes, and the 8-row ring has twice the stages, so the bytes in
// flight stay the same.
template <int R>
__host__ __device__ constexpr int i4_stage_bytes() { return R * kI4RoundK / 2; }
template <int R>
__host__ __device__ constexpr int i4_scale_bytes() { return R * (kI4RoundK / 128) * 2; }
template <int R>
__host__ __device__ constexpr int i4_stages() {
  return R == kI4Rows ? kI4Stages : 2 * kI4Stages;
}

// Item epilogue buffer in shared memory: consumer warps x 8*NT tokens x (R + 1) floats
// (R rows + 1 of padding).
template <int NT, int R>
__host__ __device__ constexpr size_t i4_red_bytes() {
  return (size_t)kI4Consumers * NT * 8 * (R + 1) * 4;
}

// One group's shared memory: weight ring, scale ring, barriers, epilogue buffer,
// rounded up to 1024 bytes so every group's ring keeps the swizzle alignment.
template <int NT, int R>
__host__ __device__ constexpr size_t i4_group_bytes() {
  return ((size_t)i4_stages<R>() * (i4_stage_bytes<R>() + i4_scale_bytes<R>()) + 256 +
          i4_red_bytes<NT, R>() + 1023) /
         1024 * 1024;
}

struct I4Bars {  // sized for the deeper (8-row) ring: 192 of the 256 bytes reserved
  uint64_t full[2 * kI4Stages], empty[2 * kI4Stages];
};

// (a & b) ^ c
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// f16x2 arithmetic on raw 32-bit registers, round-to-nearest-even, no contraction.
__device__ __forceinline__ uint32_t hfma2_rn(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One packed word (nibbles k0..k7, k0 lowest) -> fp16(q * scale) as the half2 pairs
// (k0,k1) (k2,k3) (k4,k5) (k6,k7); s2 = the fp16 scale in both halves. Byte b is
// copied to all four byte positions; the low half keeps bits 0-3 (value 1024 + u'),
// the high half bits 4-7 of its byte (1024 + 16 u'), u' = u ^ 8;
// h * (1, 1/16) - (1032, 72) = q exactly, then one rounding in the multiply by s2.
__device__ __forceinline__ void dequant_word(uint32_t q, uint32_t s2, uint32_t* p) {
  constexpr uint32_t kMul = 0x2C003C00u;  // (1.0, 0.0625)
  constexpr uint32_t kOff = 0xD480E408u;  // (-1032.0, -72.0)
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t r = __byte_perm(q, 0u, 0x1111u * b);
    p[b] = hmul2_rn(hfma2_rn(lop3_and_xor(r, 0x00F0000Fu, 0x64806408u), kMul, kOff), s2);
  }
}

// Same values in the pair order (k0,k4) (k1,k5) (k2,k6) (k3,k7), three operations fewer:
// each 16-bit half takes its nibble straight from the word (bits 0-3 -> 1024 + u',
// bits 4-7 -> 1024 + 16 u'), the odd nibbles of each byte after one shift by 8.
__device__ __forceinline__ void dequant_word_perm(uint32_t q, uint32_t s2, uint32_t* p) {
  constexpr uint32_t kOffLo = 0x64086408u;  // (1032.0, 1032.0)
  constexpr uint32_t kSixteenth = 0x2C002C00u;  // (0.0625, 0.0625)
  constexpr uint32_t kOffHi = 0xD480D480u;  // (-72.0, -72.0)
  const uint32_t q2 = q >> 8;
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(lop3_and_xor(q, 0x000F000Fu, 0x64086408u)), "r"(kOffLo));
  p[0] = hmul2_rn(d, s2);
  p[1] = hmul2_rn(hfma2_rn(lop3_and_xor(q, 0x00F000F0u, 0x64806480u), kSixteenth, kOffHi), s2);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(lop3_and_xor(q2, 0x000F000Fu, 0x64086408u)), "r"(kOffLo));
  p[2] = hmul2_rn(d, s2);
  p[3] = hmul2_rn(hfma2_rn(lop3_and_xor(q2, 0x00F000F0u, 0x64806480u), kSixteenth, kOffHi), s2);
}

// fp16 bits in both halves of a 32-bit register
__device__ __forceinline__ uint32_t splat16(uint16_t h) { return __byte_perm(h, 0u, 0x1010u); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

#ifndef FI_I4_EVICT_FIRST
#define FI_I4_EVICT_FIRST 0
#endif
// Weight and scale tiles are read once per call; FI_I4_EVICT_FIRST=1 gives their copies
// an L2 evict-first policy (measured neutral here: 31.5-31.9 vs 31.3-31.7 us per
// Llama-3.2-3B layer at batch 1, so off by default).
__device__ __forceinline__ void i4_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                           int c1) {
#if FI_I4_EVICT_FIRST
  tma_load_2d_hint(dst, m, bar, c0, c1, l2_policy_evict_first());
#else
  tma_load_2d(dst, m, bar, c0, c1);
#endif
}
__device__ __forceinline__ void i4_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                           int c1, int c2) {
#if FI_I4_EVICT_FIRST
  tma_load_3d_hint(dst, m, bar, c0, c1, c2, l2_policy_evict_first());
#else
  tma_load_3d(dst, m, bar, c0, c1, c2);
#endif
}

// Persistent: CTA b takes work items b, b + grid, ... ; an item = R weight rows x all
// of K, processed in rounds of 1024 k. The producer warp streams each round's
// R x 512-byte weight tile into a ring as [4 chunks][R rows][128 bytes], 128B-swizzled;
// consumer warp w multiplies k = round*1024 + w*128 + 32t .. +32 of both 8-row halves
// (rows g and g+8 of the tile; g+8 only when R = 16) against x, computing C^T = W x^T
// with the weight rows
// as the MMA's M dimension and the tokens as N (tiles of 8). At the end of an item the
// 8 warps add their partial sums in warp order through shared memory.
// kSmemX: x is staged once into shared memory (rows < M, each 8-group in the order
// 0,4,1,5,2,6,3,7 that dequant_word_perm produces, zeros past K); otherwise x
// fragments come from global memory in natural order and dequant_word is used.
// G > 1: G groups (8 math warps + 1 producer warp each, own ring and item slots)
// share one staged x, so 9-16 tokens get 16 math warps per SM where a second CTA's
// copy of x would not fit.
// Every mbarrier wait is bounded: after a timeout (FI_DEVERR_TIMEOUT) the waits are
// skipped, the loops still run to the end and the producer lets its copies land.
// Up to 8 tokens the kernel fits 56 registers, so up to 4 CTAs share an SM (the ring
// and staged x then decide); larger token tiles run one CTA per SM.
// Launched with programmatic dependent launch: the producer pulls its first ring of
// weight tiles into L2 while the previous kernel finishes; every read of x, of the
// scales and of the ring waits for it (grid_dep_wait).
// kXR (x too large for shared memory, 9-16 tokens): x is staged one 1024-k round at a
// time into two shared-memory slices that the groups share, and each slot's items (at
// most kI4XRItems) advance round by round, so x is read from L2 once per round instead
// of once per weight word.
template <int NT, bool kSmemX, int G, int R, bool kXR = false>
__global__ void __launch_bounds__(G * kI4Threads, NT == 1 ? 32 / kI4Consumers : 1)
    int4_gemm_kernel(const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_s, const I4Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  // G groups of (8 consumer warps + 1 producer warp), each with its own ring, share
  // one staged copy of x: group grp owns warps [grp*9, grp*9 + 9).
  const int warp_all = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp_all / (kI4Consumers + 1);
  const int warp = warp_all - grp * (kI4Consumers + 1);  // warp within the group
  const int tid = warp * 32 + lane;                       // thread within the group
  constexpr int kSB = i4_stage_bytes<R>(), kScB = i4_scale_bytes<R>(), kSt = i4_stages<R>();
  uint8_t* stages = smem + grp * i4_group_bytes<NT, R>();
  uint8_t* sstages = stages + kSt * kSB;  // kSt scale tiles of R rows x 8 groups
  I4Bars* bars = reinterpret_cast<I4Bars*>(sstages + kSt * kScB);
  // partial sums of the item epilogue: [warp][token][row], rows padded to R + 1
  auto red = reinterpret_cast<float(*)[NT * 8][R + 1]>(reinterpret_cast<uint8_t*>(bars) + 256);
  __half* xs = reinterpret_cast<__half*>(smem + G * i4_group_bytes<NT, R>());
  const int group_bar = kI4ConsumerBar + grp;  // named barrier of this group's consumers

  // Item slots, group-major (slot grp * grid + b for group grp of CTA b), so items past
  // one per slot go to different CTAs; a slot takes items slot, slot + grid*G, ...
  const int items = (a.N + R - 1) / R;
  const int slot = grp * gridDim.x + blockIdx.x, nslots = gridDim.x * G;
  const int my_items = slot < items ? (items - slot + nslots - 1) / nslots : 0;
  const int total = my_items * a.rounds;
  // Stage q of this slot: item-major, or round-major when x is staged by round.
  auto q_item = [&](int q) {
    return slot + (kXR ? q % my_items : q / a.rounds) * nslots;
  };
  auto q_round = [&](int q) { return kXR ? q / my_items : q % a.rounds; };

  if (tid == 0) {
    for (int i = 0; i < kSt; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], kI4Consumers * 32);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // The next projection may start launching now: it only reads weights into L2
  // until this grid has completed.
  grid_dep_launch();

  if (warp == kI4Consumers) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      if (a.tma_scales) prefetch_tmap(&tm_s);
      // Before the previous kernel on the stream is known to be done (it may have
      // written these weights), the first ring's worth of weight tiles only goes to
      // L2; the shared-memory copies start after grid_dep_wait().
      for (int q = 0; q < total && q < kSt; ++q) {
        const int item = q_item(q), r = q_round(q);
        if (a.tma3d) {
          tma_prefetch_l2_3d(&tm_w, 0, item * R, r * kI4Boxes);
        } else {
#pragma unroll
          for (int b = 0; b < kI4Boxes; ++b)
            tma_prefetch_l2_2d(&tm_w, r * (kI4RoundK / 2) + b * kI4BoxBytes, item * R);
        }
      }
      grid_dep_wait();
      bool dead = false;
      for (int q = 0; q < total; ++q) {
        const int st = q % kSt;
        if (q >= kSt && !dead) dead = !mbar_wait(&bars->empty[st], ((q / kSt) - 1) & 1, a.err);
        const int item = q_item(q), r = q_round(q);
        mbar_arrive_expect_tx(&bars->full[st], kSB + (a.tma_scales ? kScB : 0));
        if (a.tma_scales)  // scales [N, K/128] fp16: 8 groups x R rows
          i4_load_2d(sstages + st * kScB, &tm_s, &bars->full[st], r * (kI4RoundK / 128),
                     item * R);
        if (a.tma3d) {
          // (byte, row, 128-byte chunk): one box = 4 chunks x R rows x 128 bytes
          i4_load_3d(stages + st * kSB, &tm_w, &bars->full[st], 0, item * R, r * kI4Boxes);
        } else {
#pragma unroll
          for (int b = 0; b < kI4Boxes; ++b)
            i4_load_2d(stages + st * kSB + b * (R * kI4BoxBytes), &tm_w, &bars->full[st],
                       r * (kI4RoundK / 2) + b * kI4BoxBytes, item * R);
        }
      }
      // Let the last copy of every stage land before the CTA can exit.
      for (int q = total > kSt ? total - kSt : 0; q < total; ++q)
        mbar_wait(&bars->full[q % kSt], (q / kSt) & 1, a.err);
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  grid_dep_wait();  // x and the scales may be the previous kernel's output
  const int g = lane >> 2, t = lane & 3;
  if constexpr (kSmemX) {
    // Each thread owns chunk columns c (8 k each) and walks the token rows kXB at a
    // time, with kXB independent 16-byte loads in flight: staging costs a few memory
    // latencies, not one per chunk, and no index division (one token keeps a batch
    // of one in the 56-register one-tile instance).
    constexpr int kXB = NT == 1 ? 1 : kI4XBatch;
    constexpr int kStride = G * kI4Consumers * 32;
    const int chunks = a.rounds * (kI4RoundK / 8);
    const int kchunks = a.K / 8;
    for (int c = grp * kI4Consumers * 32 + tid; c < chunks; c += kStride) {
      const __half* xc = a.x + c * 8;
      __half* sc = xs + c * 8;
      for (int m0 = 0; m0 < a.M; m0 += kXB) {
        uint4 u[kXB];
#pragma unroll
        for (int j = 0; j < kXB; ++j) {
          u[j] = make_uint4(0u, 0u, 0u, 0u);
          if (m0 + j < a.M && c < kchunks)
            u[j] = *reinterpret_cast<const uint4*>(xc + (int64_t)(m0 + j) * a.xs0);
        }
#pragma unroll
        for (int j = 0; j < kXB; ++j) {
          if (m0 + j >= a.M) break;
          *reinterpret_cast<uint4*>(sc + (m0 + j) * a.xstride) = make_uint4(
              __byte_perm(u[j].x, u[j].z, 0x5410), __byte_perm(u[j].x, u[j].z, 0x7632),
              __byte_perm(u[j].y, u[j].w, 0x5410), __byte_perm(u[j].y, u[j].w, 0x7632));
        }
      }
    }
    named_bar_sync(kI4ConsumerBar + G, G * kI4Consumers * 32);  // every group's consumers
  }
  // Element offset of this lane's x row (token nt*8 + g) in xs or x. Tokens past M
  // (padding of the last 8-token tile) read row M-1: their MMA columns are computed
  // and never stored, so the loads need no predicate and no zero fill.
  int64_t xo[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = min(nt * 8 + g, a.M - 1);
    xo[nt] = kXR ? (int64_t)tok * (kI4RoundK + 8)
                 : kSmemX ? (int64_t)tok * a.xstride : (int64_t)tok * a.xs0;
  }

  if constexpr (kXR) {
    // Requires scales by TMA (the host checks) and at most kI4XRItems items per slot.
    constexpr int kXS = kI4RoundK + 8;   // slice row stride (halves)
    constexpr int kC8 = kI4RoundK / 8;   // 16-byte chunks per slice row
    constexpr int kAll = G * kI4Consumers * 32;
    const int xtid = grp * kI4Consumers * 32 + tid;
    // slice r of x into dst, pair order as for the whole staged x, 4 loads in flight
    auto stage_x = [&](int r, __half* dst) {
      const int n = a.M * kC8;
      for (int c0 = xtid; c0 < n; c0 += 4 * kAll) {
        uint4 u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = c0 + j * kAll, m = c / kC8, k0 = r * kI4RoundK + (c - m * kC8) * 8;
          u[j] = make_uint4(0u, 0u, 0u, 0u);
          if (c < n && k0 < a.K)
            u[j] = *reinterpret_cast<const uint4*>(a.x + (int64_t)m * a.xs0 + k0);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = c0 + j * kAll, m = c / kC8;
          if (c < n)
            *reinterpret_cast<uint4*>(dst + m * kXS + (c - m * kC8) * 8) = make_uint4(
                __byte_perm(u[j].x, u[j].z, 0x5410), __byte_perm(u[j].x, u[j].z, 0x7632),
                __byte_perm(u[j].y, u[j].w, 0x5410), __byte_perm(u[j].y, u[j].w, 0x7632));
        }
      }
    };
    stage_x(0, xs);
    named_bar_sync(kI4ConsumerBar + G, kAll);
    float ac[kI4XRItems][NT][4];
#pragma unroll
    for (int j = 0; j < kI4XRItems; ++j)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) ac[j][nt][e] = 0.f;
    bool dead = false;
    const int box = warp >> 1, chunk = ((warp & 1) << 2) + t, swz = (chunk ^ g) << 4;
    const int kloc = warp * kI4KIter + 32 * t;  // this lane's x column within the round
    int q = 0;
    for (int r = 0; r < a.rounds; ++r) {
      // slice r + 1 goes to the buffer every group finished reading in round r - 1
      if (r + 1 < a.rounds) stage_x(r + 1, xs + ((r + 1) & 1) * a.M * kXS);
      const __half* xr = xs + (r & 1) * a.M * kXS;
#pragma unroll
      for (int j = 0; j < kI4XRItems; ++j) {
        if (j >= my_items) break;
        const int st = q % kSt;
        if (!dead)
          dead = !__all_sync(0xffffffffu, mbar_wait(&bars->full[st], (q / kSt) & 1, a.err));
        const uint8_t* sbase = stages + st * kSB + box * (R * kI4BoxBytes);
        const uint4 qa4 = *reinterpret_cast<const uint4*>(sbase + g * kI4BoxBytes + swz);
        uint4 qb4 = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (R == kI4Rows)
          qb4 = *reinterpret_cast<const uint4*>(sbase + (g + 8) * kI4BoxBytes + swz);
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(sstages + st * kScB);
        const uint32_t s2a = splat16(sc[g * (kI4RoundK / 128) + warp]);
        uint32_t s2b = 0u;
        if constexpr (R == kI4Rows) s2b = splat16(sc[(g + 8) * (kI4RoundK / 128) + warp]);
        fence_proxy_async_smem();  // generic reads before the next TMA write of the stage
        mbar_arrive(&bars->empty[st]);
        const uint32_t wa4[4] = {qa4.x, qa4.y, qa4.z, qa4.w};
        const uint32_t wb4[4] = {qb4.x, qb4.y, qb4.z, qb4.w};
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
          uint32_t ba[4], bb[4] = {0u, 0u, 0u, 0u};
          dequant_word_perm(wa4[wd], s2a, ba);
          if constexpr (R == kI4Rows) dequant_word_perm(wb4[wd], s2b, bb);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint4 u = *reinterpret_cast<const uint4*>(xr + xo[nt] + kloc + 8 * wd);
            mma_16816(ac[j][nt], ba[0], bb[0], ba[1], bb[1], u.x, u.y);
            mma_16816(ac[j][nt], ba[2], bb[2], ba[3], bb[3], u.z, u.w);
          }
        }
        ++q;
      }
      named_bar_sync(kI4ConsumerBar + G, kAll);
    }
    // items done: add the 8 warps' partial sums in warp order, store fp16
#pragma unroll
    for (int j = 0; j < kI4XRItems; ++j) {
      if (j >= my_items) break;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (R == kI4Rows || e < 2)
            red[warp][nt * 8 + 2 * t + (e & 1)][g + (e >> 1) * 8] = ac[j][nt][e];
      named_bar_sync(group_bar, kI4Consumers * 32);
      const int nbase = (slot + j * nslots) * R;
      for (int i = tid; i < a.M * R; i += kI4Consumers * 32) {
        const int m = i / R, rr = i - m * R, n = nbase + rr;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kI4Consumers; ++w) sum += red[w][m][rr];
        if (n < a.N) a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(sum);
      }
      named_bar_sync(group_bar, kI4Consumers * 32);
    }
    return;
  }

  // scale of (row, k) for this lane; fetched one round ahead
  auto scale_of = [&](int item, int r, int h) -> uint16_t {
    const int n = item * R + g + 8 * h;
    const int kk = r * kI4RoundK + warp * kI4KIter + 32 * t;
    if (n >= a.N || kk >= a.K) return 0;
    const int grp = a.gs_shift >= 0 ? kk >> a.gs_shift : kk / a.gs;
    return reinterpret_cast<const uint16_t*>(a.s)[n * a.ss0 + grp * a.ss1];
  };
  uint16_t sa_n = 0, sb_n = 0;
  if (total > 0 && !a.tma_scales) {
    sa_n = scale_of(slot, 0, 0);
    if constexpr (R == kI4Rows) sb_n = scale_of(slot, 0, 1);
  }

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  bool dead = false;
  const int box = warp >> 1;                 // which 128-byte box of the stage
  const int chunk = ((warp & 1) << 2) + t;   // 16-byte chunk inside the box row
  const int swz = (chunk ^ g) << 4;          // 128B swizzle: chunk ^ (row % 8), row = g or g+8
  // 8-row items: rows 8-15 of the A operand are zero (their outputs are not stored)
  int q = 0;
  for (int j = 0; j < my_items; ++j) {
    const int item = slot + j * nslots;
    for (int r = 0; r < a.rounds; ++r, ++q) {
      uint32_t s2a = splat16(sa_n), s2b = splat16(sb_n);
      if (!a.tma_scales) {  // prefetch the next round's scales
        const int r1 = r + 1 < a.rounds ? r + 1 : 0;
        const int it1 = r + 1 < a.rounds ? item : item + nslots;
        const bool more = q + 1 < total;
        sa_n = more ? scale_of(it1, r1, 0) : 0;
        if constexpr (R == kI4Rows) sb_n = more ? scale_of(it1, r1, 1) : 0;
      }
      const int st = q % kSt;
      if (!dead) dead = !__all_sync(0xffffffffu, mbar_wait(&bars->full[st], (q / kSt) & 1, a.err));
      const uint8_t* sbase = stages + st * kSB + box * (R * kI4BoxBytes);
      const uint4 qa4 = *reinterpret_cast<const uint4*>(sbase + g * kI4BoxBytes + swz);
      uint4 qb4 = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (R == kI4Rows)
        qb4 = *reinterpret_cast<const uint4*>(sbase + (g + 8) * kI4BoxBytes + swz);
      if (a.tma_scales) {  // [R rows][groups of the round]: this warp's group is `warp`
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(sstages + st * kScB);
        s2a = splat16(sc[g * (kI4RoundK / 128) + warp]);
        if constexpr (R == kI4Rows) s2b = splat16(sc[(g + 8) * (kI4RoundK / 128) + warp]);
      }
      // The stage is released before these values are used, and the next write to it
      // is a TMA (async proxy) write: order this thread's generic reads before it.
      fence_proxy_async_smem();
      mbar_arrive(&bars->empty[st]);
      const int kk = r * kI4RoundK + warp * kI4KIter + 32 * t;  // this lane's x column
      const bool kval = kk < a.K;
      const uint32_t wa4[4] = {qa4.x, qa4.y, qa4.z, qa4.w};
      const uint32_t wb4[4] = {qb4.x, qb4.y, qb4.z, qb4.w};
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        uint32_t ba[4], bb[4] = {0u, 0u, 0u, 0u};
        if constexpr (kSmemX) {
          dequant_word_perm(wa4[wd], s2a, ba);
          if constexpr (R == kI4Rows) dequant_word_perm(wb4[wd], s2b, bb);
        } else {
          dequant_word(wa4[wd], s2a, ba);
          if constexpr (R == kI4Rows) dequant_word(wb4[wd], s2b, bb);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // B = x^T: token nt*8 + g, this lane's 8 k (pair order matching ba/bb)
          uint4 u;
          if constexpr (kSmemX) {
            u = *reinterpret_cast<const uint4*>(xs + xo[nt] + kk + 8 * wd);
          } else {
            u = make_uint4(0u, 0u, 0u, 0u);
            if (kval) u = __ldg(reinterpret_cast<const uint4*>(a.x + xo[nt] + kk + 8 * wd));
          }
          // A = weights: rows g (ba) and g+8 (bb), two k pairs each
          mma_16816(acc[nt], ba[0], bb[0], ba[1], bb[1], u.x, u.y);
          mma_16816(acc[nt], ba[2], bb[2], ba[3], bb[3], u.z, u.w);
        }
      }
    }
    // ---- item done: add the 8 warps' partial sums in warp order, store fp16
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // C^T fragment: weight row g + 8*(e>>1), token nt*8 + 2t + (e&1)
        if (R == kI4Rows || e < 2)
          red[warp][nt * 8 + 2 * t + (e & 1)][g + (e >> 1) * 8] = acc[nt][e];
        acc[nt][e] = 0.f;
      }
    named_bar_sync(group_bar, kI4Consumers * 32);
    const int nbase = item * R;
    for (int i = tid; i < a.M * R; i += kI4Consumers * 32) {
      const int m = i / R, rr = i - m * R, n = nbase + rr;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kI4Consumers; ++w) sum += red[w][m][rr];
      if (n < a.N) a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(sum);
    }
    named_bar_sync(group_bar, kI4Consumers * 32);
  }
}

// Storage dequantizer: one thread per packed word (8 consecutive k of one row).
__global__ void __launch_bounds__(256) int4_dequant_kernel(const uint8_t* w, const __half* s,
                                                           __half* out, int N, int K, int gs,
                                                           int64_t ws0, int64_t ss0,
                                                           int64_t ss1, int64_t os0) {
  const int64_t words_per_row = K / 8;
  const int64_t total = (int64_t)N * words_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / words_per_row;
    const int k = (int)(i - n * words_per_row) * 8;
    const uint32_t q = *reinterpret_cast<const uint32_t*>(w + n * ws0 + k / 2);
    uint32_t p[4];
    dequant_word(q, splat16(__half_as_ushort(s[n * ss0 + (k / gs) * ss1])), p);
    *reinterpret_cast<uint4*>(out + n * os0 + k) = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

constexpr size_t kI4SmemOptin = 232448;  // per-block shared memory limit (227 KB)

// Dynamic shared memory without x: 1 KB of alignment slack and G groups.
template <int NT, int G, int R>
constexpr size_t i4_smem_base() {
  return 1024 + (size_t)G * i4_group_bytes<NT, R>();
}

// Largest staged x for an instance: the limit minus the groups, less 1 KB of margin.
#ifndef FI_I4_XMAX_KB
#define FI_I4_XMAX_KB 1024
#endif
template <int NT, int G, int R>
constexpr size_t i4_smem_x_max() {
  constexpr size_t used = i4_smem_base<NT, G, R>() + 1024;
  constexpr size_t fit = used < kI4SmemOptin ? kI4SmemOptin - used : 0;
  return fit < (size_t)FI_I4_XMAX_KB * 1024 ? fit : (size_t)FI_I4_XMAX_KB * 1024;
}

// Opts each instance in to its largest shared-memory layout (once per device), sizes
// the persistent grid with the occupancy calculator for this call's layout, launches.
// Two x slices of up to NT*8 rows for the round-by-round staging.
template <int NT>
constexpr size_t i4_xr_bytes() {
  return 2 * (size_t)NT * 8 * (kI4RoundK + 8) * 2;
}

template <int NT, bool kSmemX, int G, int R, bool kXR = false>
static int launch_int4_gemm(cudaStream_t st, const CUtensorMap& tm, const CUtensorMap& tms,
                            const I4Args& a) {
  static DeviceOnce attr_once;
  {
    const cudaError_t e = attr_once.run([] {
      const size_t x_max = kSmemX ? i4_smem_x_max<NT, G, R>() : kXR ? i4_xr_bytes<NT>() : 0;
      const int max_smem = (int)(i4_smem_base<NT, G, R>() + x_max);
      return cudaFuncSetAttribute(int4_gemm_kernel<NT, kSmemX, G, R, kXR>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    });
    if (e != cudaSuccess) return cuda_fail(e, "fi_int4_gemm: cudaFuncSetAttribute");
  }
  const size_t smem = i4_smem_base<NT, G, R>() +
                      (kSmemX ? (size_t)a.M * (size_t)a.xstride * 2
                              : kXR ? 2 * (size_t)a.M * (kI4RoundK + 8) * 2 : 0);
  const int threads = G * kI4Threads;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, int4_gemm_kernel<NT, kSmemX, G, R, kXR>,
                                                    threads, smem) != cudaSuccess || nb < 1)
    nb = 1;
  const int items = (a.N + R - 1) / R;
  // up to one CTA per item: with group-major slots, items beyond one per CTA go to the
  // second group of different CTAs, so every SM gets work before any gets two items
  int grid = nb * sm_count();
  if (grid > items) grid = items;
  if (kXR && items > kI4XRItems * G * grid)
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_gemm: too many items for round-major staging");
  cudaError_t e = launch_pdl(int4_gemm_kernel<NT, kSmemX, G, R, kXR>, dim3((unsigned)grid),
                             dim3(threads), smem, st, tm, tms, a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_int4_gemm launch");
  return FI_OK;
}

// x staged in shared memory when it fits; for two 8-token tiles (9-16 tokens) two
// groups share one staged x when both rings fit beside it (16 math warps per SM).
template <int NT, int R>
static int launch_int4_gemm_nt(cudaStream_t st, const CUtensorMap& tm, const CUtensorMap& tms,
                               const I4Args& a) {
  const size_t xbytes = (size_t)a.M * (size_t)a.xstride * 2;
  if constexpr (NT == 2) {
    if (xbytes <= i4_smem_x_max<NT, 2, R>())
      return launch_int4_gemm<NT, true, 2, R>(st, tm, tms, a);
  }
  if (xbytes <= i4_smem_x_max<NT, 1, R>()) return launch_int4_gemm<NT, true, 1, R>(st, tm, tms, a);
  if constexpr (NT == 2) {
    // x by round: scales must come by TMA, every slot must hold at most kI4XRItems
    // items (at least min(items, SMs) CTAs of two groups are launched), and there must
    // be more items than SMs. Per call, batch 16, K = 8192 (x from global memory / by
    // round): N = 3072 16.7 / 15.3 us, N = 5120 24.2 / 19.8; but N = 2368 (148 items)
    // 9.6 / 11.9, where staging x every round costs more than the loads it saves.
    const int64_t items = (a.N + R - 1) / R;
    if (a.tma_scales && items > sm_count() && items <= (int64_t)kI4XRItems * 2 * sm_count() &&
        i4_smem_base<NT, 2, R>() + i4_xr_bytes<NT>() + 1024 <= kI4SmemOptin)
      return launch_int4_gemm<NT, false, 2, R, true>(st, tm, tms, a);
  }
  return launch_int4_gemm<NT, false, 1, R>(st, tm, tms, a);
}

// Rows per work item for batches of up to 8 tokens: 8 when 16-row items number at most
// two per SM and 8-row items lower the most rows any SM streams, else 16. N = 3072 on
// 148 SMs: 192 items of 16 leave 44 SMs two (32 rows), 384 items of 8 give every SM at
// most three (24 rows). Measured per call (CUDA graphs, weights rotated past L2, batch
// 1, K = 3072 / 8192, 16-row / 8-row): N = 3072 4.73 / 4.18 and 9.17 / 8.61 us, N = 1184
// 3.04 / 2.79 and 5.96 / 5.17; above two items per SM 8-row items lose (N = 5120: 5.11
// / 6.58, 11.36 / 14.2), as they do at 9-16 tokens (N = 3072, K = 8192: 16.7 / 23.5).
#ifndef FI_I4_ROWS8
#define FI_I4_ROWS8 1
#endif
static int int4_rows_per_item(int64_t m, int64_t n) {
  if (!FI_I4_ROWS8 || m > 8) return kI4Rows;
  const int64_t sms = sm_count();
  const int64_t load16 = (n + 15) / 16, load8 = (n + 7) / 8;
  if (load16 > 2 * sms) return kI4Rows;
  const int64_t max16 = (load16 + sms - 1) / sms * 16, max8 = (load8 + sms - 1) / sms * 8;
  return max8 < max16 ? 8 : kI4Rows;
}

}  // namespace fi

extern "C" int fi_int4_gemm(const void* x, const void* packed, const void* scales, void* c,
                            int64_t m, int64_t n, int64_t k, int64_t groupsize,
                            const int64_t* x_strides, const int64_t* packed_strides,
                            const int64_t* scales_strides, const int64_t* c_strides,
                            int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (m < 0 || n < 0 || k <= 0 || groupsize <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_gemm: bad sizes");
  if (k % groupsize != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_gemm: K (%lld) must be a multiple of groupsize (%lld)",
                (long long)k, (long long)groupsize);
  if (groupsize % 32 != 0)
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_gemm: groupsize must be a multiple of 32");
  if (m > kI4MaxM)
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_gemm: M (%lld) > %d; dequantize and use a dense GEMM",
                (long long)m, kI4MaxM);
  if (m == 0 || n == 0) return FI_OK;
  if (n > (1 << 30) || k > (1 << 30))
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_gemm: sizes too large");
  if (!x || !packed || !scales || !c || !x_strides || !packed_strides || !scales_strides ||
      !c_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_gemm: null pointer argument");
  if (x_strides[1] != 1 || x_strides[0] % 8 != 0 || !aligned16(x))
    return fail(FI_ERR_ALIGNMENT,
                "fi_int4_gemm x: needs a 16-byte aligned base, unit K stride and a row stride "
                "that is a multiple of 8");
  if (packed_strides[1] != 1 || packed_strides[0] % 16 != 0 || !aligned16(packed))
    return fail(FI_ERR_ALIGNMENT,
                "fi_int4_gemm packed: needs a 16-byte aligned base, unit stride along K/2 and a "
                "row stride that is a multiple of 16 bytes");
  // packed [N, K/2] bytes through a tensor map with 128B swizzle. When K/2 is a whole
  // number of 128-byte chunks: 3-D (byte, row, chunk), one 4-chunk x R-row box per
  // stage; otherwise 2-D (byte, row) with four 128 x R boxes (the 3-D view would let
  // the last chunk of the last row run past the tensor).
  CUtensorMap tm;
  const int tma3d = (k / 2) % kI4BoxBytes == 0 ? 1 : 0;
  const int rows = int4_rows_per_item(m, n);  // weight rows per work item (TMA box height)
  int r;
  if (tma3d) {
    const uint64_t dims[3] = {(uint64_t)kI4BoxBytes, (uint64_t)n,
                              (uint64_t)(k / 2 / kI4BoxBytes)};
    const uint64_t sb[2] = {(uint64_t)packed_strides[0], (uint64_t)kI4BoxBytes};
    const uint32_t box[3] = {(uint32_t)kI4BoxBytes, (uint32_t)rows, (uint32_t)kI4Boxes};
    r = encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, packed, dims, sb, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, "fi_int4_gemm packed");
  } else {
    const uint64_t dims[2] = {(uint64_t)(k / 2), (uint64_t)n};
    const uint64_t sb[1] = {(uint64_t)packed_strides[0]};
    const uint32_t box[2] = {(uint32_t)kI4BoxBytes, (uint32_t)rows};
    r = encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, packed, dims, sb, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, "fi_int4_gemm packed");
  }
  if (r != FI_OK) return r;
  I4Args a;
  a.x = static_cast<const __half*>(x);
  a.s = static_cast<const __half*>(scales);
  a.c = static_cast<__half*>(c);
  a.err = error_flag;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.gs = (int)groupsize;
  a.gs_shift = (groupsize & (groupsize - 1)) == 0 ? __builtin_ctzll((unsigned long long)groupsize) : -1;
  a.rounds = (int)((k + kI4RoundK - 1) / kI4RoundK);
  a.xstride = a.rounds * kI4RoundK + 8;
  a.tma3d = tma3d;
  // Scales by TMA when one round's 8 groups are whole 16-byte rows of a dense,
  // 16-byte aligned [N, K/128] tensor (groupsize 128, K a multiple of 1024).
  CUtensorMap tms;
  memset(&tms, 0, sizeof(tms));
  a.tma_scales = groupsize == 128 && k % kI4RoundK == 0 && scales_strides[1] == 1 &&
                 (scales_strides[0] * 2) % 16 == 0 && aligned16(scales);
  if (a.tma_scales) {
    const uint64_t sdims[2] = {(uint64_t)(k / 128), (uint64_t)n};
    const uint64_t ssb[1] = {(uint64_t)scales_strides[0] * 2};
    const uint32_t sbox[2] = {(uint32_t)(kI4RoundK / 128), (uint32_t)rows};
    r = encode_tiled(&tms, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, scales, sdims, ssb, sbox,
                     CU_TENSOR_MAP_SWIZZLE_NONE, "fi_int4_gemm scales");
    if (r != FI_OK) return r;
  }
  a.xs0 = x_strides[0];
  a.ss0 = scales_strides[0];
  a.ss1 = scales_strides[1];
  a.cs0 = c_strides[0];
  a.cs1 = c_strides[1];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 8-token tiles: 1, 2, 4 or 8
  if (m <= 8)
    r = rows == 8 ? launch_int4_gemm_nt<1, 8>(st, tm, tms, a)
                  : launch_int4_gemm_nt<1, kI4Rows>(st, tm, tms, a);
  else if (m <= 16) r = launch_int4_gemm_nt<2, kI4Rows>(st, tm, tms, a);
  else if (m <= 32) r = launch_int4_gemm_nt<4, kI4Rows>(st, tm, tms, a);
  else r = launch_int4_gemm_nt<8, kI4Rows>(st, tm, tms, a);
  if (r != FI_OK) return r;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fi_int4_gemm launch");
  return FI_OK;
}

extern "C" int fi_int4_dequant(const void* packed, const void* scales, void* out, int64_t n,
                               int64_t k, int64_t groupsize, const int64_t* packed_strides,
                               const int64_t* scales_strides, const int64_t* out_strides,
                               void* stream) {
  using namespace fi;
  clear_error();
  if (n < 0 || k <= 0 || groupsize <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_dequant: bad sizes");
  if (k % groupsize != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_dequant: K must be a multiple of groupsize");
  if (groupsize % 8 != 0)
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_dequant: groupsize must be a multiple of 8");
  if (n == 0) return FI_OK;
  if (n > (1 << 30) || k > (1 << 30))
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_dequant: sizes too large");
  if (!packed || !scales || !out || !packed_strides || !scales_strides || !out_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_dequant: null pointer argument");
  if (packed_strides[1] != 1 || packed_strides[0] % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(packed) & 3u) != 0)
    return fail(FI_ERR_ALIGNMENT,
                "fi_int4_dequant packed: needs a 4-byte aligned base, unit stride along K/2 and "
                "a row stride that is a multiple of 4 bytes");
  if (out_strides[1] != 1 || out_strides[0] % 8 != 0 || !aligned16(out))
    return fail(FI_ERR_ALIGNMENT,
                "fi_int4_dequant out: needs a 16-byte aligned base, unit K stride and a row "
                "stride that is a multiple of 8");
  const int64_t total = n * (k / 8);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  int4_dequant_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(packed), static_cast<const __half*>(scales),
      static_cast<__half*>(out), (int)n, (int)k, (int)groupsize, packed_strides[0],
      scales_strides[0], scales_strides[1], out_strides[0]);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fi_int4_dequant launch");
  return FI_OK;
}

namespace fi {

// Group-wise symmetric quantizer, one thread per (row, group). Each step rounds to
// fp16 where the reference's fp16 tensor ops do (loader.py:19-39): max|w|, clamp to
// fp16(1e-6), scale = fp16(max / 7), q = round_half_even(fp16(w / scale)) in [-8, 7].
__global__ void __launch_bounds__(256) int4_quantize_kernel(const __half* w, uint8_t* packed,
                                                            __half* s, int N, int K, int gs,
                                                            int64_t ws0, int64_t ws1,
                                                            int64_t ps0, int64_t ss0,
                                                            int64_t ss1) {
  const int groups = K / gs;
  const int64_t total = (int64_t)N * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / groups;
    const int grp = (int)(i - n * groups);
    const __half* src = w + n * ws0 + (int64_t)grp * gs * ws1;
    float mx = 0.f;
    for (int j = 0; j < gs; ++j) mx = fmaxf(mx, fabsf(__half2float(src[j * ws1])));
    const float floor16 = __half2float(__float2half_rn(1e-6f));
    mx = fmaxf(mx, floor16);
    const __half sc = __float2half_rn(mx / 7.0f);
    s[n * ss0 + grp * ss1] = sc;
    const float scf = __half2float(sc);
    uint8_t* dst = packed + n * ps0 + (int64_t)grp * gs / 2;
    for (int j = 0; j < gs; j += 2) {
      int q[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float r = rintf(__half2float(__float2half_rn(__half2float(src[(j + e) * ws1]) / scf)));
        q[e] = (int)fminf(fmaxf(r, -8.f), 7.f);
      }
      dst[j / 2] = (uint8_t)((q[0] & 0xF) | ((q[1] & 0xF) << 4));
    }
  }
}

}  // namespace fi

extern "C" int fi_int4_quantize(const void* w, void* packed, void* scales, int64_t n, int64_t k,
                                int64_t groupsize, const int64_t* w_strides,
                                const int64_t* packed_strides, const int64_t* scales_strides,
                                void* stream) {
  using namespace fi;
  clear_error();
  if (n < 0 || k <= 0 || groupsize <= 0 || groupsize % 2 != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_quantize: bad sizes (groupsize must be even)");
  if (k % groupsize != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_quantize: K must be a multiple of groupsize");
  if (n == 0) return FI_OK;
  if (n > (1 << 30) || k > (1 << 30))
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_quantize: sizes too large");
  if (!w || !packed || !scales || !w_strides || !packed_strides || !scales_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_int4_quantize: null pointer argument");
  if (packed_strides[1] != 1)
    return fail(FI_ERR_ALIGNMENT, "fi_int4_quantize packed: stride along K/2 must be 1");
  const int64_t total = n * (k / groupsize);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  int4_quantize_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(w), static_cast<uint8_t*>(packed), static_cast<__half*>(scales),
      (int)n, (int)k, (int)groupsize, w_strides[0], w_strides[1], packed_strides[0],
      scales_strides[0], scales_strides[1]);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fi_int4_quantize launch");
  return FI_OK;
}
