// Paged decode attention for sm_100a: one query token per sequence, GQA, split-KV.
//
// Replaces the Triton kernel `_paged_attention_kernel` and its launcher
// (reference kernels/attention.py:116-233). Semantics per (sequence b, query head h):
//   kv = h / (Hq / Hkv)                           (attention.py:138-139)
//   for every logical page j < ceil(n / 64):      (attention.py:155)
//     phys = block_table[b, j]                    (attention.py:156)
//     s_t  = q . K[phys, t, kv, :] * scale, t < n (attention.py:163-169)
//   o = softmax(s) . V                            (online softmax, attention.py:172-186)
//
// B200 design (HBM-bound; every K/V byte crosses HBM once):
// * A CTA owns one (sequence, KV head, split) and serves all G = Hq/Hkv query heads
//   of that KV head from a single read of each page (the reference re-reads every
//   page once per query head).
// * A producer warp gathers pages through the block table with TMA: each page of
//   one KV head is 64 rows x 256 B, fetched as four 8 KB boxes (K/V x two 64-dim
//   halves) into a 128B-swizzled, 3-stage shared-memory ring (mbarrier full/empty).
// * Four consumer warps each own 16 of the 64 rows of every page. QK^T and PV run on
//   the tensor cores as m16n8k16 tiles (tokens x 8 head slots), P is transposed in
//   registers with movmatrix, softmax statistics use warp shuffles; the four
//   warps' partial (max, sum, acc) are merged through shared memory at the end.
// * Split-KV (flash-decoding): a sequence's pages are cut into splits of
//   `pages_per_split`; each split writes (max, sum, unnormalised acc) to the
//   workspace and a small combine kernel produces the output. With one split the
//   main kernel writes the output directly. The hardware block scheduler hands
//   (sequence, KV head, split) CTAs to SMs as earlier ones finish, which balances
//   ragged lengths better than a static partition of all pages over one wave of
//   CTAs (measured: that partition pays a ring drain at every unit boundary inside a
//   CTA and a per-CTA scan of the lengths, and was slower on every shape).
#include <math.h>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kD = 128;
constexpr int kPage = 64;
// K/V pages are read once per call: their TMA copies carry an L2 evict-first policy,
// so the stream does not push the block table, the queries and the partials (or a
// neighbouring kernel's data) out of L2.
#ifndef FI_DEC_EVICT_FIRST
#define FI_DEC_EVICT_FIRST 1
#endif
constexpr int kDecWarps = 4;  // consumer warps of a page group (16 rows each)
// Threads of a CTA whose kGrp groups of 4 consumer warps take alternate pages.
__host__ __device__ constexpr int dec_threads(int kgrp) { return (kDecWarps * kgrp + 1) * 32; }
// Ring slots per page group: 3 (two CTAs per SM), or 2 for grids of two to four CTAs
// per SM, where a third resident CTA per SM puts the working CTAs into one wave.
constexpr int kDecStages = 3;
constexpr int kRegionBytes = kPage * 64 * 2;    // 64 rows x 64 fp16
constexpr int kStageBytes = 4 * kRegionBytes;   // K lo, K hi, V lo, V hi
constexpr int kMaxPagesPerSplit = 32;
// Shared memory of a CTA with kgrp page groups, each with its own ring of kst slots.
__host__ __device__ constexpr int dec_smem_bytes(int kgrp, int kst = kDecStages) {
  return 1024 + kgrp * kst * kStageBytes + 2 * kgrp * kst * 8 + kMaxPagesPerSplit * 4;
}

struct DecodeParams {
  const __half* q;
  __half* o;
  const int32_t* bt;
  const int32_t* ctx_lens;
  float* ws_acc;   // [batch][hq][max_splits][128]
  float2* ws_ml;   // [batch][hq][max_splits] = (max (log2 domain), sum)
  int* err;
  int64_t qs[3], os[3], bts[2];
  int num_tokens;
  int batch, hq, hkv, group, num_blocks, max_blocks, pps, max_splits;
  float scale_log2;
};

__device__ __forceinline__ int seq_pages(const DecodeParams& p, int b, int& ctx, bool report) {
  ctx = p.ctx_lens ? p.ctx_lens[b] : p.num_tokens;
  if (ctx <= 0) {
    ctx = 0;
    return 0;
  }
  int np = (ctx + kPage - 1) / kPage;
  const int cap = min(p.max_blocks, p.max_splits * p.pps);
  if (np > cap) {
    if (report) set_error(p.err, FI_DEVERR_CONTEXT_LEN);
    np = cap;
    ctx = np * kPage;
  }
  return np;
}

__device__ __forceinline__ uint32_t swz(uint32_t region, int row, int chunk) {
  return region + row * 128 + ((chunk ^ (row & 7)) << 4);
}

// The query of (sequence b, KV head kvh) as m16n8k16 B fragments: head slot
// g = lane/4 holds query head kvh*G + g (zero for g >= G), dims 2*(lane&3) + {0, 1, 8,
// 9} of every 16-dim step.
__device__ __forceinline__ void load_q(const DecodeParams& p, int b, int kvh, int lane,
                                       uint32_t (&qf)[8][2]) {
  const int g = lane >> 2, tq = lane & 3;
  const bool hv = g < p.group;
  const __half* qrow = p.q + b * p.qs[0] + (int64_t)(kvh * p.group + (hv ? g : 0)) * p.qs[1];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d0 = kk * 16 + 2 * tq;
    float x0 = 0.f, x1 = 0.f, x8 = 0.f, x9 = 0.f;
    if (hv) {
      x0 = __half2float(qrow[d0 * p.qs[2]]);
      x1 = __half2float(qrow[(d0 + 1) * p.qs[2]]);
      x8 = __half2float(qrow[(d0 + 8) * p.qs[2]]);
      x9 = __half2float(qrow[(d0 + 9) * p.qs[2]]);
    }
    qf[kk][0] = pack_half2(x0, x1);
    qf[kk][1] = pack_half2(x8, x9);
  }
}

// One page of one (sequence, KV head) for a consumer warp: its 16 rows of the page
// (row_base..row_base+15, `valid` of them live) against the G <= 8 query heads held
// as m16n8k16 B fragments in qf, folded into the warp's online-softmax state
// (m0/m1, l0/l1: head slots 2*(lane&3) and +1; acc: [8 dim tiles][4]).
__device__ __forceinline__ void decode_page(uint32_t st, int row_base, int lane, int valid,
                                            const uint32_t (&qf)[8][2], float scale_log2,
                                            float& m0, float& m1, float& l0, float& l1,
                                            float (&acc)[8][4]) {
  const int g = lane >> 2;
  const uint32_t klo = st, khi = st + kRegionBytes;
  const uint32_t vlo = st + 2 * kRegionBytes, vhi = st + 3 * kRegionBytes;
  // S^T tile: 16 tokens x 8 head slots, K from shared memory, q^T in registers.
  float c[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int r = row_base + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(swz(kk < 4 ? klo : khi, r, (kk & 3) * 2 + (lane >> 4)), a0, a1, a2, a3);
      mma_16816(c, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
    }
  }
  float s0 = c[0] * scale_log2, s1 = c[1] * scale_log2;
  float s2 = c[2] * scale_log2, s3 = c[3] * scale_log2;
  if (g >= valid) s0 = s1 = -INFINITY;
  if (g + 8 >= valid) s2 = s3 = -INFINITY;
  float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
  const float al0 = fast_exp2(m0 - mn0), al1 = fast_exp2(m1 - mn1);
  const float p0 = fast_exp2(s0 - mn0), p1 = fast_exp2(s1 - mn1);
  const float p2 = fast_exp2(s2 - mn0), p3 = fast_exp2(s3 - mn1);
  l0 = l0 * al0 + p0 + p2;
  l1 = l1 * al1 + p1 + p3;
  m0 = mn0;
  m1 = mn1;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    acc[mt][0] *= al0;
    acc[mt][1] *= al1;
    acc[mt][2] *= al0;
    acc[mt][3] *= al1;
  }
  if (valid < 16) {
    // Rows past the context may hold anything (stale pages): zero this warp's
    // dead V rows so 0 * (inf/nan) cannot reach the accumulator.
    const int dead = 16 - valid;
    for (int idx = lane; idx < dead * 16; idx += 32) {
      const int row = row_base + valid + (idx >> 4);
      const int ch = idx & 15;
      const uint32_t addr = swz(ch < 8 ? vlo : vhi, row, ch & 7);
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
    }
    __syncwarp();
  }
  const uint32_t pb0 = movmatrix_t(pack_half2(p0, p1));
  const uint32_t pb1 = movmatrix_t(pack_half2(p2, p3));
  {
    const int tok = row_base + ((lane >> 4) << 3) + (lane & 7);
    const int chb = (lane >> 3) & 1;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(swz(mt < 4 ? vlo : vhi, tok, (mt & 3) * 2 + chb), a0, a1, a2, a3);
      mma_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
    }
  }
  // the zeroed rows were written by the generic proxy; the slot's next TMA write
  // (async proxy) must come after them
  if (valid < 16) fence_proxy_async_smem();
}

// kGrp = 2 (grids of at most one CTA per SM): two groups of four consumer warps take
// alternate pages of the split, so a CTA has two pages in flight through its
// per-page dependency chain (QK^T, softmax, PV) where one group would leave the SM
// waiting; the groups' states merge with the warps' at the end. Each group has its
// own ring (page i -> group i % kGrp, slot (i / kGrp) % kSt of that ring), so
// every waiter is at most one mbarrier phase ahead: with one shared ring a group
// could wait on a slot two phases ahead, and the parity test would report the
// previous phase as the one it wants.
// kSt = ring slots per group: 3 with two CTAs per SM, 2 with three (kGrp = 1 only).
// kCl > 1 (small grids): the kCl splits of a (sequence, KV head) form one thread-block
// cluster; each CTA leaves its merged (max, sum, acc) in its own shared memory and
// CTA 0 of the cluster reads the others' through distributed shared memory, merges
// and writes the output: no workspace and no combine launch. Every CTA of a cluster,
// with pages or not, reaches both cluster barriers.
template <int kGrp, int kSt, int kCl>
__global__ void __launch_bounds__(dec_threads(kGrp), kGrp == 1 ? (kSt == 2 ? 3 : 2) : 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const DecodeParams p) {
  constexpr int kDecStages = kSt;  // shadows the default for this instance
  constexpr int kCW = kDecWarps * kGrp;  // consumer warps
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  constexpr int kS = kGrp * kDecStages;  // ring slots of all groups
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kS * kStageBytes);
  uint64_t* empty = full + kS;
  int* s_phys = reinterpret_cast<int*>(empty + kS);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_dep_wait();  // lengths, block table, K/V and q may come from the previous kernel
  grid_dep_launch();
  int ctx;
  const int npages = seq_pages(p, b, ctx, split == 0 && threadIdx.x == 0 && kvh == 0);
  const int pg0 = split * p.pps;

  if constexpr (kCl == 1) {
    if (npages == 0) {  // empty sequence: output zeros (kernels/attention.py:205-206)
      if (split == 0 && threadIdx.x < p.group * (kD / 8)) {
        const int h = kvh * p.group + threadIdx.x / (kD / 8);
        const int d0 = (threadIdx.x % (kD / 8)) * 8;
        __half* orow = p.o + b * p.os[0] + h * p.os[1];
        for (int d = 0; d < 8; ++d) orow[(d0 + d) * p.os[2]] = __float2half(0.f);
      }
      return;
    }
    if (pg0 >= npages) return;
  }
  // pages of this CTA (cluster CTAs past the sequence's end have none; an empty
  // sequence merges to zeros)
  const int n = pg0 < npages ? min(npages - pg0, p.pps) : 0;
  const int nsplits = (npages + p.pps - 1) / p.pps;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecWarps);
    }
    fence_barrier_init();
  }
  if (warp == kCW) {
    for (int i = lane; i < n; i += 32) {
      int ph = p.bt[b * p.bts[0] + (int64_t)(pg0 + i) * p.bts[1]];
      if (ph < 0 || ph >= p.num_blocks) {
        set_error(p.err, FI_DEVERR_BAD_BLOCK);
        ph = -1;
      }
      s_phys[i] = ph;
    }
  }
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      for (int i = 0; i < n; ++i) {
        const int j = i / kGrp;  // page index within its group
        const int s = (i % kGrp) * kDecStages + j % kDecStages;
        if (j >= kDecStages && !mbar_wait(&empty[s], ((j / kDecStages) - 1) & 1, p.err)) break;
        const int ph = s_phys[i];
        if (ph < 0) {
          mbar_arrive(&full[s]);
          continue;
        }
        uint8_t* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
#if FI_DEC_EVICT_FIRST
        const uint64_t pol = l2_policy_evict_first();
        tma_load_4d_hint(st, &tm_k, &full[s], 0, kvh, 0, ph, pol);
        tma_load_4d_hint(st + kRegionBytes, &tm_k, &full[s], 64, kvh, 0, ph, pol);
        tma_load_4d_hint(st + 2 * kRegionBytes, &tm_v, &full[s], 0, kvh, 0, ph, pol);
        tma_load_4d_hint(st + 3 * kRegionBytes, &tm_v, &full[s], 64, kvh, 0, ph, pol);
#else
        tma_load_4d(st, &tm_k, &full[s], 0, kvh, 0, ph);
        tma_load_4d(st + kRegionBytes, &tm_k, &full[s], 64, kvh, 0, ph);
        tma_load_4d(st + 2 * kRegionBytes, &tm_v, &full[s], 0, kvh, 0, ph);
        tma_load_4d(st + 3 * kRegionBytes, &tm_v, &full[s], 64, kvh, 0, ph);
#endif
      }
    }
    __syncthreads();  // pairs with the consumers' barrier before the merge
    if constexpr (kCl > 1) {  // the cluster merge's two barriers
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int g = lane >> 2, tq = lane & 3;
  uint32_t qf[8][2];
  load_q(p, b, kvh, lane, qf);

  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
  const int row_base = (warp % kDecWarps) * 16;
  bool aborted = false;

  for (int i = warp / kDecWarps; i < n; i += kGrp) {
    const int j = i / kGrp;  // page index within this group
    const int s = (i % kGrp) * kDecStages + j % kDecStages;
    if (!mbar_wait(&full[s], (j / kDecStages) & 1, p.err)) {
      aborted = true;
      break;
    }
    const int valid = ctx - (pg0 + i) * kPage - row_base;  // live rows among this warp's 16
    if (s_phys[i] >= 0 && valid > 0) {
      decode_page(smem_u32(smem + s * kStageBytes), row_base, lane, valid, qf, p.scale_log2, m0,
                  m1, l0, l1, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }

  // ------------------------------------------------ merge the four warps' state
  __syncthreads();  // every page consumed, every TMA landed: the ring is free
  float* s_acc = reinterpret_cast<float*>(smem);            // [kCW warps][8 heads][128]
  float* s_m = s_acc + kCW * 8 * kD;                         // [kCW][8]
  float* s_l = s_m + kCW * 8;                                // [kCW][8]
  {
    float* wa = s_acc + warp * 8 * kD;
    const int h0 = 2 * tq, h1 = 2 * tq + 1;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = mt * 16 + g;
      wa[h0 * kD + d] = acc[mt][0];
      wa[h1 * kD + d] = acc[mt][1];
      wa[h0 * kD + d + 8] = acc[mt][2];
      wa[h1 * kD + d + 8] = acc[mt][3];
    }
    if (g == 0) {
      s_m[warp * 8 + h0] = m0;
      s_m[warp * 8 + h1] = m1;
      s_l[warp * 8 + h0] = l0;
      s_l[warp * 8 + h1] = l1;
    }
  }
  named_bar_sync(1, kCW * 32);
  // cluster merge buffers, past the warps' (the ring is free): [8 heads][128] + (M, L)
  float* s_cl = s_l + kCW * 8;
  float2* s_clml = reinterpret_cast<float2*>(s_cl + 8 * kD);
  if ((kCl == 1 && aborted) || threadIdx.x >= kDecWarps * 32) {
    if constexpr (kCl > 1) {
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }
  {
    const int t = threadIdx.x;            // 0..127
    const int h = t >> 4;                 // head slot 0..7
    const int d0 = (t & 15) * 8;
    if (h < p.group) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kCW; ++w) M = fmaxf(M, s_m[w * 8 + h]);
      float L = 0.f, o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kCW; ++w) {
          const float wt = fast_exp2(s_m[w * 8 + h] - M);
          L += s_l[w * 8 + h] * wt;
          const float* src = s_acc + (w * 8 + h) * kD + d0;
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] += src[e] * wt;
        }
      }
      const int hq = kvh * p.group + h;
      if (kCl > 1) {  // leave this split's state for the cluster's CTA 0
        float4* dst = reinterpret_cast<float4*>(s_cl + h * kD + d0);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        if ((t & 15) == 0) s_clml[h] = make_float2(M, L);
      } else if (nsplits == 1) {
        const float inv = (L > 0.f) ? 1.f / L : 0.f;
        __half* orow = p.o + b * p.os[0] + hq * p.os[1];
        if (p.os[2] == 1 && ((reinterpret_cast<uintptr_t>(orow + d0) & 15) == 0)) {
          uint4 pk;
          pk.x = pack_half2(o[0] * inv, o[1] * inv);
          pk.y = pack_half2(o[2] * inv, o[3] * inv);
          pk.z = pack_half2(o[4] * inv, o[5] * inv);
          pk.w = pack_half2(o[6] * inv, o[7] * inv);
          *reinterpret_cast<uint4*>(orow + d0) = pk;
        } else {
          for (int e = 0; e < 8; ++e) orow[(d0 + e) * p.os[2]] = __float2half(o[e] * inv);
        }
      } else {
        const size_t slot = ((size_t)b * p.hq + hq) * p.max_splits + split;
        float4* dst = reinterpret_cast<float4*>(p.ws_acc + slot * kD + d0);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
        if ((t & 15) == 0) p.ws_ml[slot] = make_float2(M, L);
      }
    }
  }
  if constexpr (kCl > 1) {
    cluster_sync_all();  // every split's state is in its CTA's shared memory
    const int t = threadIdx.x, h = t >> 4, d0 = (t & 15) * 8;
    if (split == 0 && h < p.group) {
      float Ms[kCl], Ls[kCl];
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kCl; ++r) {
        const float2 ml = ld_cluster_f2(cluster_map(smem_u32(s_clml + h), r));
        Ms[r] = ml.x;
        Ls[r] = ml.y;
        M = fmaxf(M, ml.x);
      }
      float L = 0.f, o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kCl; ++r) {
          const float wt = fast_exp2(Ms[r] - M);
          L += Ls[r] * wt;
          const uint32_t src = cluster_map(smem_u32(s_cl + h * kD + d0), r);
          const float4 a = ld_cluster_f4(src), c = ld_cluster_f4(src + 16);
          o[0] += a.x * wt;
          o[1] += a.y * wt;
          o[2] += a.z * wt;
          o[3] += a.w * wt;
          o[4] += c.x * wt;
          o[5] += c.y * wt;
          o[6] += c.z * wt;
          o[7] += c.w * wt;
        }
      }
      const float inv = (L > 0.f) ? 1.f / L : 0.f;
      __half* orow = p.o + b * p.os[0] + (kvh * p.group + h) * p.os[1];
      if (p.os[2] == 1 && ((reinterpret_cast<uintptr_t>(orow + d0) & 15) == 0)) {
        uint4 pk;
        pk.x = pack_half2(o[0] * inv, o[1] * inv);
        pk.y = pack_half2(o[2] * inv, o[3] * inv);
        pk.z = pack_half2(o[4] * inv, o[5] * inv);
        pk.w = pack_half2(o[6] * inv, o[7] * inv);
        *reinterpret_cast<uint4*>(orow + d0) = pk;
      } else {
        for (int e = 0; e < 8; ++e) orow[(d0 + e) * p.os[2]] = __float2half(o[e] * inv);
      }
    }
    cluster_sync_all();  // CTA 0 has read every CTA's shared memory
  }
}

// Merge split-KV partials: one warp per (sequence, query head), 4 dims per lane.
__global__ void __launch_bounds__(128) paged_decode_combine_kernel(const DecodeParams p) {
  grid_dep_wait();
  grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.x * 4 + warp, b = blockIdx.y;
  if (hq >= p.hq) return;
  int ctx;
  const int npages = seq_pages(p, b, ctx, false);
  const int nsplits = (npages + p.pps - 1) / p.pps;
  if (nsplits <= 1) return;
  const size_t base = ((size_t)b * p.hq + hq) * p.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < nsplits; ++s) M = fmaxf(M, p.ws_ml[base + s].x);
  float L = 0.f;
  float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
    for (int s = 0; s < nsplits; ++s) {
      const float2 ml = p.ws_ml[base + s];
      const float w = fast_exp2(ml.x - M);
      L += ml.y * w;
      const float4 a = reinterpret_cast<const float4*>(p.ws_acc + (base + s) * kD)[lane];
      O.x += a.x * w;
      O.y += a.y * w;
      O.z += a.z * w;
      O.w += a.w * w;
    }
  }
  const float inv = (L > 0.f) ? 1.f / L : 0.f;
  __half* orow = p.o + b * p.os[0] + hq * p.os[1];
  const int d0 = lane * 4;
  if (p.os[2] == 1 && ((reinterpret_cast<uintptr_t>(orow + d0) & 7) == 0)) {
    uint2 pk;
    pk.x = pack_half2(O.x * inv, O.y * inv);
    pk.y = pack_half2(O.z * inv, O.w * inv);
    *reinterpret_cast<uint2*>(orow + d0) = pk;
  } else {
    orow[(d0 + 0) * p.os[2]] = __float2half(O.x * inv);
    orow[(d0 + 1) * p.os[2]] = __float2half(O.y * inv);
    orow[(d0 + 2) * p.os[2]] = __float2half(O.z * inv);
    orow[(d0 + 3) * p.os[2]] = __float2half(O.w * inv);
  }
}

// Split size: aim for ~4 waves of 2 CTAs per SM over all (sequence, KV head) pairs.
static int choose_pps(int64_t batch, int64_t hkv, int64_t max_pages, int64_t requested) {
  if (requested > 0) return (int)(requested < kMaxPagesPerSplit ? requested : kMaxPagesPerSplit);
  const int64_t units = batch * hkv > 0 ? batch * hkv : 1;
  // Small grids run one CTA per SM with two page groups; measured on B200 the best
  // split gives about half the SMs such a CTA (B=1..16 x 1..8 KV heads, 1K-8K
  // tokens: within 7 % of the best of pages_per_split 4..32). Unsplit once one CTA
  // per (sequence, KV head) reaches that (32 pages per CTA at most).
  const int64_t splits = (int64_t)sm_count() / (2 * units);
  if (splits <= 1) return kMaxPagesPerSplit;
  int64_t pps = (max_pages + splits - 1) / splits;
  if (pps < 4) pps = 4;
  if (pps > kMaxPagesPerSplit) pps = kMaxPagesPerSplit;
  return (int)pps;
}

static int64_t max_pages_of(int64_t max_context_len) {
  return max_context_len <= 0 ? 1 : (max_context_len + kPage - 1) / kPage;
}

#ifndef FI_DEC_CLUSTER_MAX
#define FI_DEC_CLUSTER_MAX 8
#endif
#ifndef FI_DEC_CLUSTER_MIN_PAGES
#define FI_DEC_CLUSTER_MIN_PAGES 4
#endif
// Automatic split of a small grid: when one CTA per (sequence, KV head) would leave
// most SMs idle, the pages of each are split over a thread-block cluster of 2, 4 or 8
// CTAs (about one CTA per SM in all; at least FI_DEC_CLUSTER_MIN_PAGES pages per CTA)
// that merge in shared memory. Returns 1 when a cluster does not apply (explicit
// split, large grids, or more than kMaxPagesPerSplit pages per CTA).
static int choose_cluster(int64_t batch, int64_t hkv, int64_t max_pages, int64_t requested) {
  if (requested > 0) return 1;
  const int64_t units = batch * hkv > 0 ? batch * hkv : 1;
  int64_t cs = (int64_t)sm_count() / units;
  if (cs > FI_DEC_CLUSTER_MAX) cs = FI_DEC_CLUSTER_MAX;
  if (cs > max_pages / FI_DEC_CLUSTER_MIN_PAGES) cs = max_pages / FI_DEC_CLUSTER_MIN_PAGES;
  cs = cs >= 8 ? 8 : cs >= 4 ? 4 : cs >= 2 ? 2 : 1;
  if (cs > 1 && (max_pages + cs - 1) / cs > kMaxPagesPerSplit) return 1;
  return (int)cs;
}

}  // namespace fi

extern "C" size_t fi_paged_decode_workspace_size(int64_t batch, int64_t num_q_heads,
                                                 int64_t num_kv_heads, int64_t head_dim,
                                                 int64_t max_context_len, int64_t block_size,
                                                 int64_t pages_per_split) {
  using namespace fi;
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim != kD ||
      block_size != kPage)
    return 0;
  const int64_t mp = max_pages_of(max_context_len);
  if (choose_cluster(batch, num_kv_heads, mp, pages_per_split) > 1) return 0;
  const int pps = choose_pps(batch, num_kv_heads, mp, pages_per_split);
  const int64_t max_splits = (mp + pps - 1) / pps;
  if (max_splits <= 1) return 0;
  return (size_t)(batch * num_q_heads * max_splits) * (kD * sizeof(float) + sizeof(float2));
}

extern "C" int fi_paged_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
                               const int32_t* block_table, const int32_t* context_lens,
                               int64_t num_tokens, int64_t max_context_len, int64_t batch,
                               int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                               int64_t num_blocks, int64_t block_size, int64_t max_blocks_per_seq,
                               const int64_t* q_strides, const int64_t* kc_strides,
                               const int64_t* vc_strides, const int64_t* o_strides,
                               const int64_t* bt_strides, float sm_scale, int64_t pages_per_split,
                               void* workspace, size_t workspace_bytes, int32_t* error_flag,
                               void* stream) {
  using namespace fi;
  clear_error();
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_paged_decode: non-positive size");
  if (head_dim != kD) return fail(FI_ERR_UNSUPPORTED, "fi_paged_decode: head_dim %lld != 128", (long long)head_dim);
  if (block_size != kPage)
    return fail(FI_ERR_UNSUPPORTED, "fi_paged_decode: block_size %lld != 64", (long long)block_size);
  if (num_q_heads % num_kv_heads != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_paged_decode: num_q_heads %% num_kv_heads != 0");
  const int64_t group = num_q_heads / num_kv_heads;
  if (group > 8) return fail(FI_ERR_UNSUPPORTED, "fi_paged_decode: more than 8 query heads per KV head");
  if (batch == 0) return FI_OK;
  if (!q || !k_cache || !v_cache || !o || !block_table || !q_strides || !kc_strides ||
      !vc_strides || !o_strides || !bt_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_paged_decode: null pointer argument");
  if (kc_strides[3] != 1 || vc_strides[3] != 1)
    return fail(FI_ERR_ALIGNMENT, "fi_paged_decode: cache innermost stride must be 1");
  if (!context_lens) {
    if (num_tokens < 0) return fail(FI_ERR_INVALID_ARG, "fi_paged_decode: negative num_tokens");
    if ((num_tokens + kPage - 1) / kPage > max_blocks_per_seq)
      return fail(FI_ERR_INVALID_ARG, "fi_paged_decode: num_tokens %lld exceeds the block table",
                  (long long)num_tokens);
    max_context_len = num_tokens;
  } else if (max_context_len < 0) {
    return fail(FI_ERR_INVALID_ARG, "fi_paged_decode: negative max_context_len");
  }
  if (max_context_len > max_blocks_per_seq * kPage) max_context_len = max_blocks_per_seq * kPage;
  if (max_context_len > (int64_t)INT32_MAX / 2)
    return fail(FI_ERR_UNSUPPORTED, "fi_paged_decode: context too long");

  const int64_t mp = max_pages_of(max_context_len);
  const int cluster = choose_cluster(batch, num_kv_heads, mp, pages_per_split);
  const int pps = cluster > 1 ? (int)((mp + cluster - 1) / cluster)
                              : choose_pps(batch, num_kv_heads, mp, pages_per_split);
  const int64_t max_splits = cluster > 1 ? cluster : (mp + pps - 1) / pps;
  const size_t need = fi_paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                     max_context_len, block_size, pages_per_split);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(FI_ERR_WORKSPACE, "fi_paged_decode: workspace of %zu bytes needed, %zu given",
                need, workspace_bytes);
  if (max_splits > 65535 || num_kv_heads > 65535 || batch > 65535)
    return fail(FI_ERR_UNSUPPORTED, "fi_paged_decode: launch grid too large");

  CUtensorMap tmk, tmv;
  {
    const uint64_t dims[4] = {(uint64_t)kD, (uint64_t)num_kv_heads, (uint64_t)kPage,
                              (uint64_t)num_blocks};
    const uint32_t box[4] = {64, 1, kPage, 1};
    const uint64_t sk[3] = {(uint64_t)kc_strides[2] * 2, (uint64_t)kc_strides[1] * 2,
                            (uint64_t)kc_strides[0] * 2};
    const uint64_t sv[3] = {(uint64_t)vc_strides[2] * 2, (uint64_t)vc_strides[1] * 2,
                            (uint64_t)vc_strides[0] * 2};
    int r = encode_tiled(&tmk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, k_cache, dims, sk, box,
                         CU_TENSOR_MAP_SWIZZLE_128B, "fi_paged_decode k_cache");
    if (r != FI_OK) return r;
    r = encode_tiled(&tmv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, v_cache, dims, sv, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, "fi_paged_decode v_cache");
    if (r != FI_OK) return r;
  }

  DecodeParams p;
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(o);
  p.bt = block_table;
  p.ctx_lens = context_lens;
  p.ws_acc = static_cast<float*>(workspace);
  p.ws_ml = reinterpret_cast<float2*>(
      static_cast<uint8_t*>(workspace) +
      (need > 0 ? (size_t)(batch * num_q_heads * max_splits) * kD * sizeof(float) : 0));
  p.err = error_flag;
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = q_strides[i];
    p.os[i] = o_strides[i];
  }
  p.bts[0] = bt_strides[0];
  p.bts[1] = bt_strides[1];
  p.num_tokens = (int)(context_lens ? 0 : num_tokens);
  p.batch = (int)batch;
  p.hq = (int)num_q_heads;
  p.hkv = (int)num_kv_heads;
  p.group = (int)group;
  p.num_blocks = (int)num_blocks;
  p.max_blocks = (int)max_blocks_per_seq;
  p.pps = pps;
  p.max_splits = (int)max_splits;
  p.scale_log2 = (float)((double)sm_scale * 1.4426950408889634);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  static DeviceOnce attr_once;
  {
    const cudaError_t e = attr_once.run([] {
      cudaError_t r = cudaFuncSetAttribute(paged_decode_kernel<1, 3, 1>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           dec_smem_bytes(1, 3));
      if (r == cudaSuccess)
        r = cudaFuncSetAttribute(paged_decode_kernel<1, 2, 1>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, dec_smem_bytes(1, 2));
      if (r == cudaSuccess)
        r = cudaFuncSetAttribute(paged_decode_kernel<2, 3, 1>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, dec_smem_bytes(2, 3));
      if (r == cudaSuccess)
        r = cudaFuncSetAttribute(paged_decode_kernel<2, 3, 2>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, dec_smem_bytes(2, 3));
      if (r == cudaSuccess)
        r = cudaFuncSetAttribute(paged_decode_kernel<2, 3, 4>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, dec_smem_bytes(2, 3));
      if (r == cudaSuccess)
        r = cudaFuncSetAttribute(paged_decode_kernel<2, 3, 8>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, dec_smem_bytes(2, 3));
      return r;
    });
    if (e != cudaSuccess) return cuda_fail(e, "fi_paged_decode: cudaFuncSetAttribute");
  }
  dim3 grid((unsigned)max_splits, (unsigned)num_kv_heads, (unsigned)batch);
  // At most one CTA per SM: two page groups per CTA (see paged_decode_kernel). Two
  // to four CTAs per SM: a 2-slot ring and three resident CTAs per SM, so the CTAs
  // that have pages (splits past a sequence's end exit at once) fit one wave; measured
  // on config 5 with one KV head (256 sequences, 512 CTAs): 58.7 vs 63.2 us, and
  // within 1 % either way on the grids of config 3 and config 5 with 2-8 KV heads.
  const int64_t ctas = max_splits * num_kv_heads * batch, sms = sm_count();
  cudaError_t e;
  if (cluster > 1) {  // at most one CTA per SM, merged in shared memory: no combine launch
    const dim3 blk(dec_threads(2));
    const size_t sm = dec_smem_bytes(2, 3);
    e = cluster == 2   ? launch_pdl_cluster(paged_decode_kernel<2, 3, 2>, grid, blk, sm, s, 2, tmk, tmv, p)
        : cluster == 4 ? launch_pdl_cluster(paged_decode_kernel<2, 3, 4>, grid, blk, sm, s, 4, tmk, tmv, p)
                       : launch_pdl_cluster(paged_decode_kernel<2, 3, 8>, grid, blk, sm, s, 8, tmk, tmv, p);
    if (e != cudaSuccess) return cuda_fail(e, "fi_paged_decode: cluster launch");
    return FI_OK;
  }
  if (ctas <= sms)
    e = launch_pdl(paged_decode_kernel<2, 3, 1>, grid, dim3(dec_threads(2)), dec_smem_bytes(2, 3), s,
                   tmk, tmv, p);
  else if (ctas <= 4 * sms)
    e = launch_pdl(paged_decode_kernel<1, 2, 1>, grid, dim3(dec_threads(1)), dec_smem_bytes(1, 2), s,
                   tmk, tmv, p);
  else
    e = launch_pdl(paged_decode_kernel<1, 3, 1>, grid, dim3(dec_threads(1)), dec_smem_bytes(1, 3), s,
                   tmk, tmv, p);
  if (e != cudaSuccess) return cuda_fail(e, "fi_paged_decode: launch");
  if (max_splits > 1) {
    dim3 g2((unsigned)((num_q_heads + 3) / 4), (unsigned)batch);
    e = launch_pdl(paged_decode_combine_kernel, g2, dim3(128), 0, s, p);
    if (e != cudaSuccess) return cuda_fail(e, "fi_paged_decode: combine launch");
  }
  return FI_OK;
}
