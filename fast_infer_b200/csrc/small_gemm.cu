// Decode-sized fp16 GEMM with an optional RMSNorm prologue and residual epilogue:
//   c[m, :] = (residual[m, :] +) norm(x[m, :]) @ w^T,   m < M <= 16,
// w [N, K] fp16 (the reference's linear-weight layout, kernels/matmul.py:187-212
// `_fp16_matmul`), fp32 accumulation, fp16 out (one rounding, after the residual).
// norm(x) = the reference's RMSNorm (kernels/rms_norm.py:29-43) with the same fp32
// arithmetic and reduction order as fi_rms_norm, so the normalised rows are the
// ones fi_rms_norm would produce; without a norm weight x is used as is.
//
// Replaces, in the decode step of the attention stack (model.py:82-93,134-141 at
// batch <= 16), the RMSNorm launch plus the QKV library GEMM, and the O-projection
// GEMM plus the residual add. At these sizes the library GEMM streams the weights at
// about half the HBM rate; the weights are the whole cost (M x K of x is ~100 KB).
//
// B200 design (same skeleton as the INT4 kernel): persistent CTAs, one TMA producer
// warp streaming 16-row x 512-k weight tiles (one 3-D box of 8 x 128-byte chunks,
// 128B-swizzled) into a ring; 8 math warps each take one 64-k chunk of every tile:
// A fragments straight from the swizzled tile with ldmatrix, B = x^T fragments with
// ldmatrix from x staged once per CTA in shared memory, mma.sync m16n8k16 computing
// C^T = W x^T (weight rows = MMA M, tokens = N). The 8 warps' partial sums are added
// in warp order through shared memory (deterministic). Every mbarrier wait is
// bounded (FI_DEVERR_TIMEOUT). Launched with programmatic dependent launch: the
// first ring of weight tiles goes to L2 before the wait for the previous kernel.
#include <cuda_fp16.h>

#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace fi {

#ifndef FI_SG_EVICT_FIRST
#define FI_SG_EVICT_FIRST 1
#endif
// A weight tile: every weight byte is read once per call, so it may leave L2 first.
__device__ __forceinline__ void sg_load_w(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                          int c1, int c2) {
#if FI_SG_EVICT_FIRST
  tma_load_3d_hint(dst, m, bar, c0, c1, c2, l2_policy_evict_first());
#else
  tma_load_3d(dst, m, bar, c0, c1, c2);
#endif
}

constexpr int kSgWarps = 8;                        // math warps
constexpr int kSgThreads = (kSgWarps + 1) * 32;    // + one TMA producer warp
constexpr int kSgRows = 16;                        // weight rows (outputs) per work item
constexpr int kSgChunk = 64;                       // k per math warp per round (128 bytes)
constexpr int kSgRoundK = kSgWarps * kSgChunk;     // 512
constexpr int kSgChunkBytes = kSgRows * 128;       // 2 KB: 16 rows x 64 fp16
constexpr int kSgStageBytes = kSgWarps * kSgChunkBytes;  // 16 KB
constexpr int kSgStages = 4;
constexpr int kSgMaxM = 16;
constexpr int kSgBar = 1;                          // named barrier of the math warps

struct SgArgs {
  const __half* x;
  const __half* res;   // residual (nullable)
  const __half* normw; // RMSNorm weight [K] (nullable)
  __half* c;
  int* err;
  int M, N, K, rounds, xstride;
  int w_static;  // FI_STATIC_WEIGHTS: weight tiles may load before the dependency wait
  float eps;
  int64_t xs0, cs0, cs1, rs0, rs1;
};

constexpr int kSsDeepStages = 6;  // streamed variant, at most one CTA per SM (see below)
struct SgBars {  // sized for the deepest ring (96 of the 256 bytes reserved)
  uint64_t full[kSsDeepStages], empty[kSsDeepStages];
};

template <int NT>
__host__ __device__ constexpr size_t sg_red_bytes() {
  return (size_t)kSgWarps * NT * 8 * (kSgRows + 1) * 4;
}
__host__ __device__ constexpr size_t sg_fixed_bytes() {
  return 1024 + (size_t)kSgStages * kSgStageBytes + 256;
}

template <int NT>
__global__ void __launch_bounds__(kSgThreads, 1)
    small_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const SgArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* stages = smem;
  SgBars* bars = reinterpret_cast<SgBars*>(stages + kSgStages * kSgStageBytes);
  auto red = reinterpret_cast<float(*)[NT * 8][kSgRows + 1]>(reinterpret_cast<uint8_t*>(bars) + 256);
  __half* xs = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(bars) + 256 + sg_red_bytes<NT>());

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int items = (a.N + kSgRows - 1) / kSgRows;
  const int my_items = blockIdx.x < items ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int total = my_items * a.rounds;

  if (tid == 0) {
    for (int i = 0; i < kSgStages; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], kSgWarps * 32);
    }
    fence_barrier_init();
  }
  __syncthreads();
  grid_dep_launch();

  if (warp == kSgWarps) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      // Constant weights (FI_STATIC_WEIGHTS): the first stages load while the previous
      // kernel still runs; otherwise they only go to L2 before the wait.
      const int pre = a.w_static ? (total < kSgStages ? total : kSgStages) : 0;
      for (int q = 0; q < total && q < kSgStages; ++q) {
        const int item = blockIdx.x + (q / a.rounds) * gridDim.x, r = q % a.rounds;
        if (q < pre) {
          mbar_arrive_expect_tx(&bars->full[q], kSgStageBytes);
          sg_load_w(stages + q * kSgStageBytes, &tm_w, &bars->full[q], 0, item * kSgRows,
                    r * kSgWarps);
        } else {
          tma_prefetch_l2_3d(&tm_w, 0, item * kSgRows, r * kSgWarps);
        }
      }
      grid_dep_wait();
      bool dead = false;
      for (int q = pre; q < total; ++q) {
        const int st = q % kSgStages;
        if (q >= kSgStages && !dead)
          dead = !mbar_wait(&bars->empty[st], ((q / kSgStages) - 1) & 1, a.err);
        const int item = blockIdx.x + (q / a.rounds) * gridDim.x, r = q % a.rounds;
        mbar_arrive_expect_tx(&bars->full[st], kSgStageBytes);
        // (element, row, 64-element chunk): 8 chunks x 16 rows x 128 bytes
        sg_load_w(stages + st * kSgStageBytes, &tm_w, &bars->full[st], 0, item * kSgRows,
                  r * kSgWarps);
      }
      for (int q = total > kSgStages ? total - kSgStages : 0; q < total; ++q)
        mbar_wait(&bars->full[q % kSgStages], (q / kSgStages) & 1, a.err);
    }
    return;
  }

  // ---------------------------------------------------------------- math warps
  grid_dep_wait();  // x, the residual and the norm weight may be the previous kernel's output
  {
    // x -> shared memory [M][xstride], zero past K (up to the last round's end), with
    // 8 independent 16-byte loads in flight per thread.
    const int chunks = a.rounds * (kSgRoundK / 8), kchunks = a.K / 8;
    const int total_c = a.M * chunks;
    for (int i0 = tid; i0 < total_c; i0 += 8 * kSgWarps * 32) {
      uint4 u[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + j * kSgWarps * 32;
        const int m = i / chunks, c = i - m * chunks;
        u[j] = make_uint4(0u, 0u, 0u, 0u);
        if (i < total_c && c < kchunks)
          u[j] = *reinterpret_cast<const uint4*>(a.x + m * a.xs0 + c * 8);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + j * kSgWarps * 32;
        if (i >= total_c) break;
        const int m = i / chunks, c = i - m * chunks;
        *reinterpret_cast<uint4*>(xs + m * a.xstride + c * 8) = u[j];
      }
    }
    named_bar_sync(kSgBar, kSgWarps * 32);
    if (a.normw) {
      // RMSNorm in place, one warp per token row, in fi_rms_norm's order: lane l sums
      // x^2 over its 8-element vectors l, l+32, ... with fmaf, then a butterfly
      // shuffle; out = (x * rsqrt(mean + eps)) * w rounded to fp16.
      const int vecs = a.K / 8;
      for (int m = warp; m < a.M; m += kSgWarps) {
        __half* row = xs + m * a.xstride;
        float ss = 0.f;
        for (int v = lane; v < vecs; v += 32) {
          const uint4 u = *reinterpret_cast<const uint4*>(row + v * 8);
          const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h[e]);
            ss = fmaf(f.x, f.x, ss);
            ss = fmaf(f.y, f.y, ss);
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float rms = rsqrtf(ss / (float)a.K + a.eps);
        for (int v = lane; v < vecs; v += 32) {
          uint4 u = *reinterpret_cast<const uint4*>(row + v * 8);
          const uint4 wu = __ldg(reinterpret_cast<const uint4*>(a.normw + v * 8));
          __half2* h = reinterpret_cast<__half2*>(&u);
          const __half2* wh = reinterpret_cast<const __half2*>(&wu);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h[e]);
            const float2 g = __half22float2(wh[e]);
            h[e] = __floats2half2_rn(f.x * rms * g.x, f.y * rms * g.y);
          }
          *reinterpret_cast<uint4*>(row + v * 8) = u;
        }
      }
      named_bar_sync(kSgBar, kSgWarps * 32);
    }
  }

  const int g = lane >> 2, t = lane & 3;
  // ldmatrix row addresses. A: weight rows lane & 15, k half lane >> 4 of each k16
  // step. B: token (lane & 7) of tile nt (tokens past M read row M-1: computed, never
  // stored), k = 8 * (lane >> 3) within a 32-k pair of steps.
  uint32_t xrow[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    xrow[nt] = smem_u32(xs + min(nt * 8 + (lane & 7), a.M - 1) * a.xstride + (lane >> 3) * 8);
  const int arow = lane & 15, ahalf = lane >> 4;

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  bool dead = false;
  int q = 0;
  for (int j = 0; j < my_items; ++j) {
    const int item = blockIdx.x + j * gridDim.x;
    for (int r = 0; r < a.rounds; ++r, ++q) {
      const int st = q % kSgStages;
      if (!dead) dead = !__all_sync(0xffffffffu, mbar_wait(&bars->full[st], (q / kSgStages) & 1, a.err));
      const uint32_t region = smem_u32(stages + st * kSgStageBytes + warp * kSgChunkBytes);
      uint32_t af[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        ldsm_x4(region + arow * 128 + (((kk * 2 + ahalf) ^ (arow & 7)) << 4), af[kk][0],
                af[kk][1], af[kk][2], af[kk][3]);
      // The stage is released once its values are in registers; the next write to
      // it is a TMA (async proxy) write, so order these reads before it.
      fence_proxy_async_smem();
      mbar_arrive(&bars->empty[st]);
      const uint32_t kbyte = (uint32_t)(r * kSgRoundK + warp * kSgChunk) * 2;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(xrow[nt] + kbyte + kp * 64, b0, b1, b2, b3);
          mma_16816(acc[nt], af[2 * kp][0], af[2 * kp][1], af[2 * kp][2], af[2 * kp][3], b0, b1);
          mma_16816(acc[nt], af[2 * kp + 1][0], af[2 * kp + 1][1], af[2 * kp + 1][2],
                    af[2 * kp + 1][3], b2, b3);
        }
      }
    }
    // ---- item done: add the 8 warps' partial sums in warp order, residual, store
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // C^T fragment: weight row g + 8*(e>>1), token nt*8 + 2t + (e&1)
        red[warp][nt * 8 + 2 * t + (e & 1)][g + (e >> 1) * 8] = acc[nt][e];
        acc[nt][e] = 0.f;
      }
    named_bar_sync(kSgBar, kSgWarps * 32);
    const int nbase = item * kSgRows;
    for (int i = tid; i < a.M * kSgRows; i += kSgWarps * 32) {
      const int m = i / kSgRows, rr = i - m * kSgRows, n = nbase + rr;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kSgWarps; ++w) sum += red[w][m][rr];
      if (n < a.N) {
        if (a.res) sum += __half2float(a.res[m * a.rs0 + n * a.rs1]);
        a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(sum);
      }
    }
    named_bar_sync(kSgBar, kSgWarps * 32);
  }
}

template <int NT>
static int launch_small_gemm(cudaStream_t st, const CUtensorMap& tm, const SgArgs& a,
                             size_t smem) {
  static DeviceOnce attr_once;
  {
    const cudaError_t e = attr_once.run([] {
      return cudaFuncSetAttribute(small_gemm_kernel<NT>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    });
    if (e != cudaSuccess) return cuda_fail(e, "fi_small_gemm: cudaFuncSetAttribute");
  }
  const int items = (a.N + kSgRows - 1) / kSgRows;
  int grid = sm_count();
  if (grid > items) grid = items;
  cudaError_t e = launch_pdl(small_gemm_kernel<NT>, dim3((unsigned)grid), dim3(kSgThreads), smem,
                             st, tm, a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_small_gemm launch");
  return FI_OK;
}

// ---------------------------------------------------------------------------
// Streamed variant: x arrives by TMA together with each weight tile (16 KB of
// weights + 16 KB of x per round, 3-stage ring), so nothing is staged before the
// first MMA and two CTAs share an SM. With kFold the weights come pre-multiplied by
// the RMSNorm weight (w'[n, k] = fp16(w[n, k] * g[k])) and the per-token factor
// rsqrt(mean(x^2) + eps) is taken from the x tiles of the CTA's first item and
// applied in the epilogue: out = rms[m] * sum_k x[m, k] w'[n, k].
constexpr int kSsStageBytes = 2 * kSgStageBytes;  // weights | x

struct SsArgs {
  const __half* res;
  __half* c;
  int* err;
  int M, N, K, rounds;
  int w_static;  // FI_STATIC_WEIGHTS: weight tiles may load before the dependency wait
  float eps;
  int64_t cs0, cs1, rs0, rs1;
  // kRope epilogue: RoPE of q / k and the KV-cache slot writes of k / v (one token per
  // sequence; row m of x is sequence m at position start_pos[m])
  const float* cos_tab;
  const float* sin_tab;
  const int32_t* start_pos;
  __half* q_out;
  __half* kc;
  __half* vc;
  const int32_t* bt;
  int nq, nkv;
  int64_t max_pos, tab_stride, num_blocks, block_size, max_blocks;
  int64_t qs[3], kcs[4], vcs[4], bts[2];
  // kReduce epilogue (fi_small_gemm_peer_reduce): the item's partial sums go to every
  // rank's landing area; the output is residual + the ranks' partials in rank order
  uint8_t* peer[8];        // each rank's region as mapped here
  int world, rank;
  int64_t land_off;        // this call's landing buffer within a region
  int64_t land_rank_bytes; // bytes of one source rank's slots within a buffer
  uint32_t* epoch;         // this rank's call counter (local)
  uint32_t* counter;       // CTA arrivals of the current call (local)
};

// kReduce landing slot of one item from one rank: 16 tokens x 16 outputs as fp16,
// three per 8-byte word with the call's 16-bit epoch in the top half of the second
// word (the flag travels inside the data: an 8-byte store reaches the peer whole).
constexpr int kPrSlotWords = 88;  // ceil(256 / 3) = 86, padded

__device__ __forceinline__ void st_word8(uint8_t* p, uint32_t lo, uint32_t hi) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(lo), "r"(hi) : "memory");
}
__device__ __forceinline__ void ld_word8(const uint8_t* p, uint32_t& lo, uint32_t& hi) {
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(lo), "=r"(hi) : "l"(p) : "memory");
}

// kS = 3 ring stages: two CTAs per SM; kS = 2: three (registers capped to fit).
template <int NT, int kS>
__host__ __device__ constexpr size_t ss_smem_bytes() {
  return 1024 + (size_t)kS * kSsStageBytes + 256 + sg_red_bytes<NT>() +
         (size_t)kSgWarps * 16 * 4 + 16 * 4;
}

template <int NT, bool kFold, bool kRope, int kSsStages, bool kReduce = false>
__global__ void __launch_bounds__(kSgThreads, kSsStages == 2 ? 3 : kSsStages == 3 ? 2 : 1)
    small_gemm_stream_kernel(const __grid_constant__ CUtensorMap tm_w,
                             const __grid_constant__ CUtensorMap tm_x, const SsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* stages = smem;
  SgBars* bars = reinterpret_cast<SgBars*>(stages + kSsStages * kSsStageBytes);
  auto red = reinterpret_cast<float(*)[NT * 8][kSgRows + 1]>(reinterpret_cast<uint8_t*>(bars) + 256);
  float* ssq = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256 + sg_red_bytes<NT>());
  float* rmsv = ssq + kSgWarps * 16;  // [16]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int items = (a.N + kSgRows - 1) / kSgRows;
  const int my_items = blockIdx.x < items ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int total = my_items * a.rounds;

  if (tid == 0) {
    for (int i = 0; i < kSsStages; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], kSgWarps * 32);
    }
    fence_barrier_init();
  }
  __syncthreads();
  grid_dep_launch();

  if (warp == kSgWarps) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_x);
      // Constant weights (FI_STATIC_WEIGHTS): the weight halves of the first stages
      // load while the previous kernel still runs (x, its output, after the wait).
      const int pre = a.w_static ? (total < kSsStages ? total : kSsStages) : 0;
      for (int q = 0; q < pre; ++q) {
        mbar_arrive_expect_tx(&bars->full[q], kSsStageBytes);
        sg_load_w(stages + q * kSsStageBytes, &tm_w, &bars->full[q], 0,
                  (blockIdx.x + (q / a.rounds) * gridDim.x) * kSgRows, (q % a.rounds) * kSgWarps);
      }
      for (int q = pre; q < total && q < kSsStages; ++q)  // weights only to L2 before the wait
        tma_prefetch_l2_3d(&tm_w, 0, (blockIdx.x + (q / a.rounds) * gridDim.x) * kSgRows,
                           (q % a.rounds) * kSgWarps);
      grid_dep_wait();  // x is the previous kernel's output
      bool dead = false;
      for (int q = 0; q < total; ++q) {
        const int st = q % kSsStages;
        if (q >= kSsStages && !dead)
          dead = !mbar_wait(&bars->empty[st], ((q / kSsStages) - 1) & 1, a.err);
        const int item = blockIdx.x + (q / a.rounds) * gridDim.x, r = q % a.rounds;
        uint8_t* sp = stages + st * kSsStageBytes;
        if (q >= pre) {
          mbar_arrive_expect_tx(&bars->full[st], kSsStageBytes);
          sg_load_w(sp, &tm_w, &bars->full[st], 0, item * kSgRows, r * kSgWarps);
        }
        // x rows past M read as zeros (outside the tensor)
        tma_load_3d(sp + kSgStageBytes, &tm_x, &bars->full[st], 0, 0, r * kSgWarps);
      }
      for (int q = total > kSsStages ? total - kSsStages : 0; q < total; ++q)
        mbar_wait(&bars->full[q % kSsStages], (q / kSsStages) & 1, a.err);
    }
    return;
  }

  // ---------------------------------------------------------------- math warps
  grid_dep_wait();  // the residual may be the previous kernel's output
  // kReduce: this call's epoch (the previous call's last CTA raised the counter
  // before its grid completed; every CTA reads it before any CTA of this call can)
  const uint32_t epoch = kReduce ? *a.epoch + 1 : 0;
  bool give_up = kReduce && a.err && (*reinterpret_cast<volatile int*>(a.err) & FI_DEVERR_TIMEOUT);
  const int g = lane >> 2, t = lane & 3;
  const int arow = lane & 15, ahalf = lane >> 4;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
  float ss[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) ss[nt] = 0.f;

  bool dead = false;
  int q = 0;
  for (int j = 0; j < my_items; ++j) {
    const int item = blockIdx.x + j * gridDim.x;
    for (int r = 0; r < a.rounds; ++r, ++q) {
      const int st = q % kSsStages;
      if (!dead) dead = !__all_sync(0xffffffffu, mbar_wait(&bars->full[st], (q / kSsStages) & 1, a.err));
      const uint32_t wreg = smem_u32(stages + st * kSsStageBytes + warp * kSgChunkBytes);
      const uint32_t xreg = wreg + kSgStageBytes;
      uint32_t af[4][4], bf[NT][2][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        ldsm_x4(wreg + arow * 128 + (((kk * 2 + ahalf) ^ (arow & 7)) << 4), af[kk][0], af[kk][1],
                af[kk][2], af[kk][3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int xr = nt * 8 + (lane & 7);  // token row of this lane's ldmatrix address
#pragma unroll
        for (int kp = 0; kp < 2; ++kp)
          ldsm_x4(xreg + xr * 128 + (((kp * 4 + (lane >> 3)) ^ (xr & 7)) << 4), bf[nt][kp][0],
                  bf[nt][kp][1], bf[nt][kp][2], bf[nt][kp][3]);
      }
      // Both tiles are in registers: release the stage (the next write to it is a
      // TMA write, so order these reads before it).
      fence_proxy_async_smem();
      mbar_arrive(&bars->empty[st]);
      if (kFold && j == 0) {
        // this thread's x values of token nt*8 + g: 16 of the warp's 64 k per round
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int kp = 0; kp < 2; ++kp)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&bf[nt][kp][e]));
              ss[nt] = fmaf(f.x, f.x, fmaf(f.y, f.y, ss[nt]));
            }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
          mma_16816(acc[nt], af[2 * kp][0], af[2 * kp][1], af[2 * kp][2], af[2 * kp][3],
                    bf[nt][kp][0], bf[nt][kp][1]);
          mma_16816(acc[nt], af[2 * kp + 1][0], af[2 * kp + 1][1], af[2 * kp + 1][2],
                    af[2 * kp + 1][3], bf[nt][kp][2], bf[nt][kp][3]);
        }
    }
    // ---- item done: warp partial sums in warp order (x the rms factor), residual
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        red[warp][nt * 8 + 2 * t + (e & 1)][g + (e >> 1) * 8] = acc[nt][e];
        acc[nt][e] = 0.f;
      }
    if (kFold && j == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float v = ss[nt];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (t == 0) ssq[warp * 16 + nt * 8 + g] = v;
      }
      named_bar_sync(kSgBar, kSgWarps * 32);
      if (tid < 16) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kSgWarps; ++w) v += ssq[w * 16 + tid];
        rmsv[tid] = rsqrtf(v / (float)a.K + a.eps);
      }
    }
    named_bar_sync(kSgBar, kSgWarps * 32);
    if constexpr (kRope) {
      // Weight rows are permuted so that item 8h + ci holds dims ci*8 .. ci*8+7 of
      // head h in rows 0-7 and dims 64 + ci*8 .. in rows 8-15: each thread takes one
      // rotary pair (d, d + 64) of one token, rounds both projection outputs to fp16
      // (the values the unfused path stores) and applies the reference's RoPE and
      // slot writes to them (as fi_rope_kv_write does).
      const int head = item >> 3, ci = item & 7;
      for (int i = tid; i < a.M * 8; i += kSgWarps * 32) {
        const int m = i >> 3, rr = i & 7;
        float lo = 0.f, hi = 0.f;
#pragma unroll
        for (int w = 0; w < kSgWarps; ++w) {
          lo += red[w][m][rr];
          hi += red[w][m][rr + 8];
        }
        if (kFold) {
          lo *= rmsv[m];
          hi *= rmsv[m];
        }
        __half ol = __float2half_rn(lo), oh = __float2half_rn(hi);
        const int d0 = ci * 8 + rr, d1 = 64 + d0;
        const int64_t pos = a.start_pos[m];
        const bool is_v = head >= a.nq + a.nkv;
        if (!is_v) {
          if (pos < 0 || pos >= a.max_pos) {
            set_error(a.err, FI_DEVERR_CONTEXT_LEN);
            continue;
          }
          const float* ct = a.cos_tab + pos * a.tab_stride;
          const float* sn = a.sin_tab + pos * a.tab_stride;
          const float xlo = __half2float(ol), xhi = __half2float(oh);
          ol = rope_elem(xlo, -xhi, __float2half_rn(ct[d0]), __float2half_rn(sn[d0]));
          oh = rope_elem(xhi, xlo, __float2half_rn(ct[d1]), __float2half_rn(sn[d1]));
        }
        if (head < a.nq) {
          __half* dst = a.q_out + m * a.qs[0] + head * a.qs[1];
          dst[d0 * a.qs[2]] = ol;
          dst[d1 * a.qs[2]] = oh;
          continue;
        }
        const int kvh = is_v ? head - a.nq - a.nkv : head - a.nq;
        const int64_t lblk = pos / a.block_size;
        if (pos < 0 || lblk >= a.max_blocks) {
          set_error(a.err, FI_DEVERR_BAD_BLOCK);
          continue;
        }
        const int64_t phys = a.bt[m * a.bts[0] + lblk * a.bts[1]];
        if (phys < 0 || phys >= a.num_blocks) {
          set_error(a.err, FI_DEVERR_BAD_BLOCK);
          continue;
        }
        const int64_t slot = pos % a.block_size;
        const int64_t* cs = is_v ? a.vcs : a.kcs;
        __half* dst = (is_v ? a.vc : a.kc) + phys * cs[0] + slot * cs[1] + kvh * cs[2];
        dst[d0 * cs[3]] = ol;
        dst[d1 * cs[3]] = oh;
      }
    } else if constexpr (kReduce) {
      // Thread w < kWords owns values 3w..3w+2 of the item (value v = token v/16,
      // output v%16): sends its word of this rank's partial to every rank, then sums
      // every rank's word in rank order, adds the residual and stores.
      constexpr int kVals = NT * 8 * kSgRows;
      constexpr int kWords = (kVals + 2) / 3;
      const int nbase = item * kSgRows;
      if (tid < kWords) {
        uint32_t hv[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int v = tid * 3 + j;
          float sum = 0.f;
          if (v < kVals) {
#pragma unroll
            for (int w = 0; w < kSgWarps; ++w) sum += red[w][v >> 4][v & 15];
          }
          hv[j] = __half_as_ushort(__float2half_rn(sum));
        }
        const uint32_t lo = hv[0] | (hv[1] << 16), hi = hv[2] | ((epoch & 0xFFFFu) << 16);
        const int64_t off = a.land_off + a.rank * a.land_rank_bytes +
                            ((int64_t)item * kPrSlotWords + tid) * 8;
        for (int p = 0; p < a.world; ++p) st_word8(a.peer[p] + off, lo, hi);
        float part[3] = {0.f, 0.f, 0.f};
        const unsigned long long t0 = globaltimer_ns();
        for (int p = 0; p < a.world; ++p) {
          const uint8_t* src = a.peer[a.rank] + a.land_off + p * a.land_rank_bytes +
                               ((int64_t)item * kPrSlotWords + tid) * 8;
          uint32_t x, y;
          ld_word8(src, x, y);
          uint32_t spins = 0;
          while ((y >> 16) != (epoch & 0xFFFFu) && !give_up) {
            if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
              set_error(a.err, FI_DEVERR_TIMEOUT);
              give_up = true;
            }
            ld_word8(src, x, y);
          }
          part[0] += __half2float(__ushort_as_half((unsigned short)(x & 0xFFFFu)));
          part[1] += __half2float(__ushort_as_half((unsigned short)(x >> 16)));
          part[2] += __half2float(__ushort_as_half((unsigned short)(y & 0xFFFFu)));
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int v = tid * 3 + j, m = v >> 4, n = nbase + (v & 15);
          if (v < kVals && m < a.M && n < a.N) {
            float out = part[j];
            if (a.res) out += __half2float(a.res[m * a.rs0 + n * a.rs1]);
            a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(out);
          }
        }
      }
    } else {
      const int nbase = item * kSgRows;
      for (int i = tid; i < a.M * kSgRows; i += kSgWarps * 32) {
        const int m = i / kSgRows, rr = i - m * kSgRows, n = nbase + rr;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kSgWarps; ++w) sum += red[w][m][rr];
        if (kFold) sum *= rmsv[m];
        if (n < a.N) {
          if (a.res) sum += __half2float(a.res[m * a.rs0 + n * a.rs1]);
          a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(sum);
        }
      }
    }
    named_bar_sync(kSgBar, kSgWarps * 32);
  }
  if constexpr (kReduce) {
    // the last CTA of this call raises the epoch for the next call
    if (tid == 0 && atomicAdd(a.counter, 1u) == gridDim.x - 1) {
      atomicExch(a.counter, 0u);
      *a.epoch = epoch;
    }
  }
}

template <int NT, bool kFold, bool kRope, int kS, bool kReduce = false>
static int launch_small_gemm_stream_s(cudaStream_t st, const CUtensorMap& tw,
                                      const CUtensorMap& tx, const SsArgs& a) {
  constexpr size_t smem = ss_smem_bytes<NT, kS>();
  static DeviceOnce attr_once;
  {
    const cudaError_t e = attr_once.run([] {
      return cudaFuncSetAttribute(small_gemm_stream_kernel<NT, kFold, kRope, kS, kReduce>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (e != cudaSuccess) return cuda_fail(e, "fi_small_gemm: cudaFuncSetAttribute");
  }
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &nb, small_gemm_stream_kernel<NT, kFold, kRope, kS, kReduce>, kSgThreads, smem) !=
          cudaSuccess ||
      nb < 1)
    nb = 1;
  const int items = (a.N + kSgRows - 1) / kSgRows;
  int grid = nb * sm_count();
  if (grid > items) grid = items;
  cudaError_t e = launch_pdl(small_gemm_stream_kernel<NT, kFold, kRope, kS, kReduce>,
                             dim3((unsigned)grid), dim3(kSgThreads), smem, st, tw, tx, a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_small_gemm launch");
  return FI_OK;
}

// Two 8-token tiles with more work items than two CTAs per SM can hold (but at most
// three per SM): the 2-stage ring at three CTAs per SM avoids a second wave of items
// (QKV 5120 x 3072 at 16 rows: 10.3 -> 8.5 us); otherwise the 3-stage ring is faster.
// At most one item per SM (the per-rank QKV share of a KV-head-sharded stack: N = 640
// at 8 GPUs, 1280 at 4): each CTA's item streams through a 6-stage ring, so more
// weight bytes are in flight per SM than two or three CTAs would keep.
#ifndef FI_SG_DEEP
#define FI_SG_DEEP 1
#endif
template <int NT, bool kFold, bool kRope = false>
static int launch_small_gemm_stream(cudaStream_t st, const CUtensorMap& tw, const CUtensorMap& tx,
                                    const SsArgs& a) {
  const int items = (a.N + kSgRows - 1) / kSgRows;
  if (FI_SG_DEEP && items <= sm_count())
    return launch_small_gemm_stream_s<NT, kFold, kRope, kSsDeepStages>(st, tw, tx, a);
  if (NT == 2 && items > 2 * sm_count() && items <= 3 * sm_count())
    return launch_small_gemm_stream_s<NT, kFold, kRope, 2>(st, tw, tx, a);
  return launch_small_gemm_stream_s<NT, kFold, kRope, 3>(st, tw, tx, a);
}

// Tensor maps of the streamed variant: w [n, k] and x [m, k] as (64-element chunk
// column, row, chunk) with 16-row x 8-chunk boxes, 128B swizzle.
static int stream_maps(const void* x, const void* w, int64_t m, int64_t n, int64_t k,
                       const int64_t* x_strides, const int64_t* w_strides, CUtensorMap* tw,
                       CUtensorMap* tx) {
  const uint32_t box[3] = {(uint32_t)kSgChunk, (uint32_t)kSgRows, (uint32_t)kSgWarps};
  {
    const uint64_t dims[3] = {(uint64_t)kSgChunk, (uint64_t)n, (uint64_t)(k / kSgChunk)};
    const uint64_t sb[2] = {(uint64_t)w_strides[0] * 2, 128};
    const int r = encode_tiled(tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, w, dims, sb, box,
                               CU_TENSOR_MAP_SWIZZLE_128B, "fi_small_gemm w");
    if (r != FI_OK) return r;
  }
  const uint64_t dims[3] = {(uint64_t)kSgChunk, (uint64_t)m, (uint64_t)(k / kSgChunk)};
  const uint64_t sb[2] = {(uint64_t)x_strides[0] * 2, 128};
  return encode_tiled(tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, x, dims, sb, box,
                      CU_TENSOR_MAP_SWIZZLE_128B, "fi_small_gemm x");
}

// Tensor maps and launch of the streamed variant (x [m, k] and w [n, k] already
// checked by the caller).
static int small_gemm_streamed(const void* x, const void* w, void* c, const void* residual,
                               bool fold, float eps, int64_t m, int64_t n, int64_t k,
                               const int64_t* x_strides, const int64_t* w_strides,
                               const int64_t* c_strides, const int64_t* residual_strides,
                               int64_t flags, int32_t* error_flag, cudaStream_t st) {
  CUtensorMap tw, tx;
  {
    const int r = stream_maps(x, w, m, n, k, x_strides, w_strides, &tw, &tx);
    if (r != FI_OK) return r;
  }
  SsArgs a;
  memset(&a, 0, sizeof(a));
  a.res = static_cast<const __half*>(residual);
  a.c = static_cast<__half*>(c);
  a.err = error_flag;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.rounds = (int)((k + kSgRoundK - 1) / kSgRoundK);
  a.w_static = (flags & FI_STATIC_WEIGHTS) != 0;
  a.eps = eps;
  a.cs0 = c_strides[0];
  a.cs1 = c_strides[1];
  if (residual) {
    a.rs0 = residual_strides[0];
    a.rs1 = residual_strides[1];
  }
  if (m <= 8)
    return fold ? launch_small_gemm_stream<1, true>(st, tw, tx, a)
                : launch_small_gemm_stream<1, false>(st, tw, tx, a);
  return fold ? launch_small_gemm_stream<2, true>(st, tw, tx, a)
              : launch_small_gemm_stream<2, false>(st, tw, tx, a);
}

}  // namespace fi

extern "C" int fi_small_gemm(const void* x, const void* w, void* c, const void* residual,
                             const void* norm_weight, float eps, int64_t m, int64_t n, int64_t k,
                             const int64_t* x_strides, const int64_t* w_strides,
                             const int64_t* c_strides, const int64_t* residual_strides,
                             int64_t flags, int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (m < 0 || n < 0 || k <= 0) return fail(FI_ERR_INVALID_ARG, "fi_small_gemm: bad sizes");
  if (flags & ~(int64_t)FI_STATIC_WEIGHTS)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm: unknown flags %lld", (long long)flags);
  if (m > kSgMaxM)
    return fail(FI_ERR_UNSUPPORTED, "fi_small_gemm: M (%lld) > %d; use a dense GEMM",
                (long long)m, kSgMaxM);
  if (k % kSgChunk != 0 || k > (1 << 20) || n > (1 << 30))
    return fail(FI_ERR_UNSUPPORTED, "fi_small_gemm: K must be a multiple of 64 (and <= 2^20)");
  if (m == 0 || n == 0) return FI_OK;
  if (!x || !w || !c || !x_strides || !w_strides || !c_strides || (residual && !residual_strides))
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm: null pointer argument");
  if (x_strides[1] != 1 || x_strides[0] % 8 != 0 || !aligned16(x) || w_strides[1] != 1 ||
      w_strides[0] % 8 != 0 || !aligned16(w) || (norm_weight && !aligned16(norm_weight)))
    return fail(FI_ERR_ALIGNMENT,
                "fi_small_gemm: x / w need 16-byte aligned bases, unit inner strides and row "
                "strides that are multiples of 8 elements");
  if (!norm_weight)  // x straight from global memory by TMA: the streamed variant
    return small_gemm_streamed(x, w, c, residual, false, eps, m, n, k, x_strides, w_strides,
                               c_strides, residual_strides, flags, error_flag,
                               static_cast<cudaStream_t>(stream));
  CUtensorMap tm;
  {
    const uint64_t dims[3] = {(uint64_t)kSgChunk, (uint64_t)n, (uint64_t)(k / kSgChunk)};
    const uint64_t sb[2] = {(uint64_t)w_strides[0] * 2, 128};
    const uint32_t box[3] = {(uint32_t)kSgChunk, (uint32_t)kSgRows, (uint32_t)kSgWarps};
    const int r = encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, w, dims, sb, box,
                               CU_TENSOR_MAP_SWIZZLE_128B, "fi_small_gemm w");
    if (r != FI_OK) return r;
  }
  SgArgs a;
  memset(&a, 0, sizeof(a));
  a.x = static_cast<const __half*>(x);
  a.res = static_cast<const __half*>(residual);
  a.normw = static_cast<const __half*>(norm_weight);
  a.c = static_cast<__half*>(c);
  a.err = error_flag;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.rounds = (int)((k + kSgRoundK - 1) / kSgRoundK);
  a.xstride = a.rounds * kSgRoundK + 8;  // + 16 bytes: conflict-free ldmatrix rows
  a.w_static = (flags & FI_STATIC_WEIGHTS) != 0;
  a.eps = eps;
  a.xs0 = x_strides[0];
  a.cs0 = c_strides[0];
  a.cs1 = c_strides[1];
  if (residual) {
    a.rs0 = residual_strides[0];
    a.rs1 = residual_strides[1];
  }
  const int nt = m <= 8 ? 1 : 2;
  const size_t smem = sg_fixed_bytes() + (nt == 1 ? sg_red_bytes<1>() : sg_red_bytes<2>()) +
                      (size_t)m * a.xstride * 2;
  if (smem > 232448)
    return fail(FI_ERR_UNSUPPORTED, "fi_small_gemm: K too large to stage x in shared memory");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return nt == 1 ? launch_small_gemm<1>(st, tm, a, smem) : launch_small_gemm<2>(st, tm, a, smem);
}

extern "C" int fi_small_gemm_folded(const void* x, const void* w_folded, void* c,
                                    const void* residual, float eps, int64_t m, int64_t n,
                                    int64_t k, const int64_t* x_strides,
                                    const int64_t* w_strides, const int64_t* c_strides,
                                    const int64_t* residual_strides, int64_t flags,
                                    int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (m < 0 || n < 0 || k <= 0) return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_folded: bad sizes");
  if (flags & ~(int64_t)FI_STATIC_WEIGHTS)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_folded: unknown flags %lld", (long long)flags);
  if (m > kSgMaxM)
    return fail(FI_ERR_UNSUPPORTED, "fi_small_gemm_folded: M (%lld) > %d", (long long)m, kSgMaxM);
  if (k % kSgChunk != 0 || k > (1 << 20) || n > (1 << 30))
    return fail(FI_ERR_UNSUPPORTED,
                "fi_small_gemm_folded: K must be a multiple of 64 (and <= 2^20)");
  if (m == 0 || n == 0) return FI_OK;
  if (!x || !w_folded || !c || !x_strides || !w_strides || !c_strides ||
      (residual && !residual_strides))
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_folded: null pointer argument");
  if (x_strides[1] != 1 || x_strides[0] % 8 != 0 || !aligned16(x) || w_strides[1] != 1 ||
      w_strides[0] % 8 != 0 || !aligned16(w_folded))
    return fail(FI_ERR_ALIGNMENT,
                "fi_small_gemm_folded: x / w need 16-byte aligned bases, unit inner strides and "
                "row strides that are multiples of 8 elements");
  return small_gemm_streamed(x, w_folded, c, residual, true, eps, m, n, k, x_strides, w_strides,
                             c_strides, residual_strides, flags, error_flag,
                             static_cast<cudaStream_t>(stream));
}

extern "C" int fi_qkv_rope_kv_write(
    const void* x, const void* w_rope, float eps, int64_t batch, int64_t k, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, const int64_t* x_strides, const int64_t* w_strides,
    const float* cos_table, const float* sin_table, int64_t table_rows, int64_t table_stride,
    const int32_t* start_pos, void* q_out, const int64_t* q_out_strides, void* k_cache,
    void* v_cache, const int32_t* block_table, int64_t num_blocks, int64_t block_size,
    int64_t max_blocks_per_seq, const int64_t* kc_strides, const int64_t* vc_strides,
    const int64_t* bt_strides, int64_t flags, int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (batch < 0 || k <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 ||
      num_blocks <= 0 || max_blocks_per_seq <= 0 || table_rows <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_qkv_rope_kv_write: bad sizes");
  if (flags & ~(int64_t)FI_STATIC_WEIGHTS)
    return fail(FI_ERR_INVALID_ARG, "fi_qkv_rope_kv_write: unknown flags %lld", (long long)flags);
  if (head_dim != 128)
    return fail(FI_ERR_UNSUPPORTED, "fi_qkv_rope_kv_write: head_dim %lld != 128",
                (long long)head_dim);
  if (batch > kSgMaxM)
    return fail(FI_ERR_UNSUPPORTED, "fi_qkv_rope_kv_write: batch (%lld) > %d", (long long)batch,
                kSgMaxM);
  if (k % kSgChunk != 0 || k > (1 << 20))
    return fail(FI_ERR_UNSUPPORTED, "fi_qkv_rope_kv_write: K must be a multiple of 64");
  if (batch == 0) return FI_OK;
  if (!x || !w_rope || !cos_table || !sin_table || !start_pos || !q_out || !k_cache ||
      !v_cache || !block_table || !x_strides || !w_strides || !q_out_strides || !kc_strides ||
      !vc_strides || !bt_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_qkv_rope_kv_write: null pointer argument");
  if (x_strides[1] != 1 || x_strides[0] % 8 != 0 || !aligned16(x) || w_strides[1] != 1 ||
      w_strides[0] % 8 != 0 || !aligned16(w_rope))
    return fail(FI_ERR_ALIGNMENT,
                "fi_qkv_rope_kv_write: x / w need 16-byte aligned bases, unit inner strides and "
                "row strides that are multiples of 8 elements");
  const int64_t n = (num_q_heads + 2 * num_kv_heads) * head_dim;
  CUtensorMap tw, tx;
  {
    const int r = stream_maps(x, w_rope, batch, n, k, x_strides, w_strides, &tw, &tx);
    if (r != FI_OK) return r;
  }
  SsArgs a;
  memset(&a, 0, sizeof(a));
  a.err = error_flag;
  a.M = (int)batch;
  a.N = (int)n;
  a.K = (int)k;
  a.rounds = (int)((k + kSgRoundK - 1) / kSgRoundK);
  a.w_static = (flags & FI_STATIC_WEIGHTS) != 0;
  a.eps = eps;
  a.cos_tab = cos_table;
  a.sin_tab = sin_table;
  a.start_pos = start_pos;
  a.q_out = static_cast<__half*>(q_out);
  a.kc = static_cast<__half*>(k_cache);
  a.vc = static_cast<__half*>(v_cache);
  a.bt = block_table;
  a.nq = (int)num_q_heads;
  a.nkv = (int)num_kv_heads;
  a.max_pos = table_rows;
  a.tab_stride = table_stride;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.max_blocks = max_blocks_per_seq;
  for (int i = 0; i < 3; ++i) a.qs[i] = q_out_strides[i];
  for (int i = 0; i < 4; ++i) {
    a.kcs[i] = kc_strides[i];
    a.vcs[i] = vc_strides[i];
  }
  a.bts[0] = bt_strides[0];
  a.bts[1] = bt_strides[1];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return batch <= 8 ? launch_small_gemm_stream<1, true, true>(st, tw, tx, a)
                    : launch_small_gemm_stream<2, true, true>(st, tw, tx, a);
}

// ---------------------------------------------------------------------------
// O projection sharded by input rows across ranks, reduced over NVLink inside the
// GEMM: c = residual + sum over ranks p (in rank order) of fp16(x_p @ w_p^T), where
// every rank passes its own x_p [m, k] (its heads' attention output) and w_p [n, k]
// (the matching columns of the projection). Each work item (16 outputs) stores its
// partial into every rank's landing area and sums all ranks' partials for those
// outputs, so the exchange costs no launch and no separate rendezvous; every rank
// ends with the same bits in c.
//
// Region of each rank (fi_peer_alloc, shared with fi_peer_open):
//   [landing: nbuf buffers x world source ranks x items x kPrSlotWords x 8 bytes]
//   [local state: call counter, CTA arrival counter]

namespace fi {
static int64_t pr_land_rank_bytes(int64_t n) {
  return ((n + kSgRows - 1) / kSgRows) * kPrSlotWords * 8;
}
}  // namespace fi

extern "C" size_t fi_peer_reduce_bytes(int64_t nbuf, int64_t world, int64_t n) {
  using namespace fi;
  if (nbuf <= 0 || world <= 0 || world > 8 || n <= 0 || n > (1 << 24)) return 0;
  return (size_t)(nbuf * world * pr_land_rank_bytes(n)) + 256;
}

extern "C" int fi_small_gemm_peer_reduce(const void* x, const void* w, void* c,
                                         const void* residual, int64_t m, int64_t n, int64_t k,
                                         const int64_t* x_strides, const int64_t* w_strides,
                                         const int64_t* c_strides,
                                         const int64_t* residual_strides, void* const* bases,
                                         int64_t world, int64_t rank, int64_t buffer,
                                         int64_t nbuf, int64_t flags, int32_t* error_flag,
                                         void* stream) {
  using namespace fi;
  clear_error();
  if (m < 0 || n <= 0 || n > (1 << 24) || k <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: bad sizes");
  if (flags & ~(int64_t)FI_STATIC_WEIGHTS)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: unknown flags %lld",
                (long long)flags);
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: world %lld / rank %lld",
                (long long)world, (long long)rank);
  if (nbuf <= 0 || buffer < 0 || buffer >= nbuf)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: bad buffer index");
  // A rank that has every partial of call k may send call k+1's while a slower rank
  // still reads call k's landing area: consecutive calls need different buffers.
  if (world > 1 && nbuf < 2)
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: %lld ranks need at least 2 buffers",
                (long long)world);
  if (m > kSgMaxM)
    return fail(FI_ERR_UNSUPPORTED, "fi_small_gemm_peer_reduce: M (%lld) > %d", (long long)m,
                kSgMaxM);
  if (k % kSgChunk != 0 || k > (1 << 20))
    return fail(FI_ERR_UNSUPPORTED,
                "fi_small_gemm_peer_reduce: K must be a multiple of 64 (and <= 2^20)");
  if (!x || !w || !c || !x_strides || !w_strides || !c_strides || !bases ||
      (residual && !residual_strides))
    return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: null pointer argument");
  if (x_strides[1] != 1 || x_strides[0] % 8 != 0 || !aligned16(x) || w_strides[1] != 1 ||
      w_strides[0] % 8 != 0 || !aligned16(w))
    return fail(FI_ERR_ALIGNMENT,
                "fi_small_gemm_peer_reduce: x and w rows must be contiguous and 16-byte aligned");
  SsArgs a;
  memset(&a, 0, sizeof(a));
  for (int p = 0; p < world; ++p) {
    if (!bases[p] || !aligned16(bases[p]))
      return fail(FI_ERR_INVALID_ARG, "fi_small_gemm_peer_reduce: region of rank %d missing", p);
    a.peer[p] = static_cast<uint8_t*>(bases[p]);
  }
  if (m == 0) return FI_OK;  // no tokens: every rank skips the call alike
  CUtensorMap tw, tx;
  {
    const int r = stream_maps(x, w, m, n, k, x_strides, w_strides, &tw, &tx);
    if (r != FI_OK) return r;
  }
  a.res = static_cast<const __half*>(residual);
  a.c = static_cast<__half*>(c);
  a.err = error_flag;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.rounds = (int)((k + kSgRoundK - 1) / kSgRoundK);
  a.w_static = (flags & FI_STATIC_WEIGHTS) != 0;
  a.cs0 = c_strides[0];
  a.cs1 = c_strides[1];
  if (residual) {
    a.rs0 = residual_strides[0];
    a.rs1 = residual_strides[1];
  }
  a.world = (int)world;
  a.rank = (int)rank;
  a.land_rank_bytes = pr_land_rank_bytes(n);
  a.land_off = buffer * world * a.land_rank_bytes;
  uint32_t* state = reinterpret_cast<uint32_t*>(a.peer[rank] + nbuf * world * a.land_rank_bytes);
  a.epoch = state;
  a.counter = state + 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return m <= 8 ? launch_small_gemm_stream_s<1, false, false, 3, true>(st, tw, tx, a)
                : launch_small_gemm_stream_s<2, false, false, 3, true>(st, tw, tx, a);
}
