// INT4 group-wise dequant-matmul for decode-sized M, and the storage dequantizer.
//
// Replaces the reference's memory-mode projection path (model.py:15-21 default
// memory_efficient=True; kernels/matmul.py:14-132 `_fused_int4_matmul`, and
// kernels/matmul.py:309-326 `_dequant_storage` / loader.py:157-190
// `dequantize_int4` for the dequantizer).
//
// Weight format (loader.py:9-41): packed int8 [N, K/2], byte j of row n holds
// w[n, 2j] in its low nibble and w[n, 2j+1] in its high nibble, two's complement in
// [-8, 7]; scales fp16 [N, K/groupsize]. A weight is fp16(q * scale) (one rounding),
// exactly as the reference computes it; products and sums are fp32, output fp16.
//
// fi_int4_gemm (M <= 64) is bound by the weight bytes it streams from HBM:
// * A CTA (8 warps) owns 128 weight rows (output columns) and one K slice of at most
//   512. Each thread streams 16-byte chunks (32 nibbles) of two weight rows, all of
//   its slice's loads in flight before any math.
// * Nibbles become fp16 without a conversion instruction: lop3 places a nibble
//   (sign bit flipped) in the mantissa of 1024.0 (0x6400), an exact HSUB2/HFMA2
//   removes the offset, and HMUL2 by the group scale gives fp16(q * scale). One
//   32-bit word yields the pairs (k0,k4) (k1,k5) (k2,k6) (k3,k7).
// * mma.sync m16n8k16 multiplies: the k order inside each 8-group is permuted the
//   same way for x (when x is staged into shared memory, once per CTA) and for the
//   weights, so every fragment comes from one 16-byte shared load or one weight word.
// * Split-K: partial sums (fp32, rows < M only) go to the caller's workspace; the
//   CTA that finishes a column block last sums them in split order (deterministic)
//   and writes fp16. Its per-column-block counter returns to zero for the next call.
#include <cuda_fp16.h>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kI4Threads = 256;  // 8 warps
constexpr int kI4Cols = 128;     // weight rows (output columns) per CTA: 8 warps x 2 x 8
constexpr int kI4KIter = 128;    // k per warp iteration: 4 threads x 32 nibbles
constexpr int kI4MaxIters = 4;   // warp iterations per K slice
constexpr int kI4MaxM = 64;      // four m16 tiles
constexpr int kI4MaxCounters = 65536;  // split-K counters, one per column block: 256 KB

struct I4Args {
  const __half* x;
  const uint8_t* w;
  const __half* s;
  __half* c;
  float* partial;      // [splits, M, Npad] fp32 (splits > 1)
  unsigned* counters;  // [gridDim.x]
  int M, N, K, gs, ks, splits, npad;
  int64_t xs0, ws0, ss0, ss1, cs0, cs1;
};

// (a & b) ^ c
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// One packed word (nibbles k0..k7, k0 lowest) -> fp16(q * scale) as the half2 pairs
// (k0,k4) (k1,k5) (k2,k6) (k3,k7). All steps before the multiply are exact.
__device__ __forceinline__ void dequant_word(uint32_t q, __half2 s2, uint32_t* p) {
  const __half2 off_lo = __floats2half2_rn(1032.f, 1032.f);   // 1024 + 8
  const __half2 sixteenth = __floats2half2_rn(0.0625f, 0.0625f);
  const __half2 off_hi = __floats2half2_rn(-72.f, -72.f);     // (1024 + 16*8) / 16
  const uint32_t q2 = q >> 8;
  // low nibble of each half: 1024 + (u ^ 8); bits 4-7: 1024 + 16 * (u ^ 8)
  const __half2 t0 = u2h(lop3_and_xor(q, 0x000F000Fu, 0x64086408u));
  const __half2 t1 = u2h(lop3_and_xor(q, 0x00F000F0u, 0x64806480u));
  const __half2 t2 = u2h(lop3_and_xor(q2, 0x000F000Fu, 0x64086408u));
  const __half2 t3 = u2h(lop3_and_xor(q2, 0x00F000F0u, 0x64806480u));
  p[0] = h2u(__hmul2(__hsub2(t0, off_lo), s2));
  p[1] = h2u(__hmul2(__hfma2(t1, sixteenth, off_hi), s2));
  p[2] = h2u(__hmul2(__hsub2(t2, off_lo), s2));
  p[3] = h2u(__hmul2(__hfma2(t3, sixteenth, off_hi), s2));
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Shared-memory position (in 16-byte chunks) of chunk c of staged row r: rows are
// padded by one chunk and bit 1 of the chunk index is flipped in odd 8-chunk blocks,
// so the fragment loads of a warp (rows g, g+1 x chunks 4t + wd) never share banks.
__device__ __forceinline__ int xs_pos(int r, int c, int row_chunks) {
  return r * (row_chunks + 1) + (c ^ (((c >> 3) & 1) << 1));
}

template <int MT>
__global__ void __launch_bounds__(kI4Threads) int4_gemm_kernel(const I4Args a) {
  extern __shared__ uint4 xs[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cb = blockIdx.x, split = blockIdx.y;
  const int k0 = split * a.ks;
  const int klen = min(a.ks, a.K - k0);  // > 0, multiple of 32
  const int row_chunks = a.ks / 8;

  // ---- stage x[0:16*MT, k0:k0+klen) with each 8-group in the order 0,4,1,5,2,6,3,7
  for (int i = tid; i < MT * 16 * row_chunks; i += kI4Threads) {
    const int r = i / row_chunks, c = i - r * row_chunks;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < a.M && c * 8 < klen) {
      const uint4 u = *reinterpret_cast<const uint4*>(a.x + r * a.xs0 + k0 + c * 8);
      v.x = __byte_perm(u.x, u.z, 0x5410);  // (h0, h4)
      v.y = __byte_perm(u.x, u.z, 0x7632);  // (h1, h5)
      v.z = __byte_perm(u.y, u.w, 0x5410);  // (h2, h6)
      v.w = __byte_perm(u.y, u.w, 0x7632);  // (h3, h7)
    }
    xs[xs_pos(r, c, row_chunks)] = v;
  }

  // ---- stream this thread's weight chunks (rows na, nb; k = kb + 32t .. +32)
  const int nbase = cb * kI4Cols + warp * 16;
  const int na = nbase + g, nb = nbase + 8 + g;
  const int nit = (klen + kI4KIter - 1) / kI4KIter;
  uint4 wa[kI4MaxIters], wb[kI4MaxIters];
  __half sa[kI4MaxIters], sb[kI4MaxIters];
#pragma unroll
  for (int it = 0; it < kI4MaxIters; ++it) {
    wa[it] = make_uint4(0u, 0u, 0u, 0u);
    wb[it] = make_uint4(0u, 0u, 0u, 0u);
    sa[it] = __float2half(0.f);
    sb[it] = __float2half(0.f);
    const int kk = it * kI4KIter + 32 * t;  // offset inside the slice
    if (it < nit && kk < klen) {
      const int kabs = k0 + kk;
      const int grp = kabs / a.gs;
      if (na < a.N) {
        wa[it] = ldg_stream(a.w + na * a.ws0 + kabs / 2);
        sa[it] = a.s[na * a.ss0 + grp * a.ss1];
      }
      if (nb < a.N) {
        wb[it] = ldg_stream(a.w + nb * a.ws0 + kabs / 2);
        sb[it] = a.s[nb * a.ss0 + grp * a.ss1];
      }
    }
  }
  __syncthreads();

  float acc[MT][2][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;

#pragma unroll
  for (int it = 0; it < kI4MaxIters; ++it) {
    if (it >= nit) break;
    const __half2 s2a = __half2half2(sa[it]), s2b = __half2half2(sb[it]);
    const uint32_t qa[4] = {wa[it].x, wa[it].y, wa[it].z, wa[it].w};
    const uint32_t qb[4] = {wb[it].x, wb[it].y, wb[it].z, wb[it].w};
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
      uint32_t ba[4], bb[4];
      dequant_word(qa[wd], s2a, ba);
      dequant_word(qb[wd], s2b, bb);
      const int c = it * 16 + 4 * t + wd;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 u = xs[xs_pos(mt * 16 + g, c, row_chunks)];
        const uint4 v = xs[xs_pos(mt * 16 + 8 + g, c, row_chunks)];
        mma_16816(acc[mt][0], u.x, v.x, u.y, v.y, ba[0], ba[1]);
        mma_16816(acc[mt][0], u.z, v.z, u.w, v.w, ba[2], ba[3]);
        mma_16816(acc[mt][1], u.x, v.x, u.y, v.y, bb[0], bb[1]);
        mma_16816(acc[mt][1], u.z, v.z, u.w, v.w, bb[2], bb[3]);
      }
    }
  }

  // ---- epilogue: C fragment rows g / g+8, columns 2t, 2t+1 of each 8-column block
  if (a.splits == 1) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = mt * 16 + g + (e >> 1) * 8;
          const int n = nbase + j * 8 + 2 * t + (e & 1);
          if (m < a.M && n < a.N) a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(acc[mt][j][e]);
        }
    return;
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int m = mt * 16 + g + h * 8;
        const int n = nbase + j * 8 + 2 * t;  // < npad
        if (m < a.M)
          *reinterpret_cast<float2*>(a.partial + ((int64_t)split * a.M + m) * a.npad + n) =
              make_float2(acc[mt][j][2 * h], acc[mt][j][2 * h + 1]);
      }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (tid == 0) s_last = atomicAdd(&a.counters[cb], 1u) == (unsigned)(a.splits - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < a.M * kI4Cols; i += kI4Threads) {
    const int m = i / kI4Cols, n = cb * kI4Cols + (i - m * kI4Cols);
    float sum = 0.f;
    for (int sp = 0; sp < a.splits; ++sp)
      sum += __ldcg(a.partial + ((int64_t)sp * a.M + m) * a.npad + n);
    if (n < a.N) a.c[m * a.cs0 + n * a.cs1] = __float2half_rn(sum);
  }
  if (tid == 0) atomicExch(&a.counters[cb], 0u);
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
    dequant_word(q, __half2half2(s[n * ss0 + (k / gs) * ss1]), p);
    uint4 o;  // back to natural order: (k0,k1) (k2,k3) (k4,k5) (k6,k7)
    o.x = __byte_perm(p[0], p[1], 0x5410);
    o.y = __byte_perm(p[2], p[3], 0x5410);
    o.z = __byte_perm(p[0], p[1], 0x7632);
    o.w = __byte_perm(p[2], p[3], 0x7632);
    *reinterpret_cast<uint4*>(out + n * os0 + k) = o;
  }
}

struct I4Plan {
  int cbs, splits, ks, mt, npad;
  size_t counter_bytes, partial_bytes;
};

static I4Plan plan_int4(int64_t m, int64_t n, int64_t k) {
  I4Plan p;
  p.cbs = (int)((n + kI4Cols - 1) / kI4Cols);
  p.npad = p.cbs * kI4Cols;
  p.mt = (int)((m + 15) / 16);
  const int iters_total = (int)((k + kI4KIter - 1) / kI4KIter);
  const int target = 2 * sm_count();
  int splits = (target + p.cbs - 1) / p.cbs;
  if (splits < 1) splits = 1;
  if (splits > iters_total) splits = iters_total;
  int iters = (iters_total + splits - 1) / splits;
  if (iters > kI4MaxIters) iters = kI4MaxIters;
  splits = (iters_total + iters - 1) / iters;
  p.splits = splits;
  p.ks = iters * kI4KIter;
  // The counters sit in a fixed region that only ever holds counters, whatever the
  // shape: a region sized per call would overlap the previous call's partial sums.
  p.counter_bytes = splits > 1 ? (size_t)kI4MaxCounters * 4 : 0;
  p.partial_bytes = splits > 1 ? (size_t)splits * (size_t)m * (size_t)p.npad * 4 : 0;
  return p;
}

// Opts the MT instance in to its largest staging buffer (once per device), launches.
template <int MT>
static int launch_int4_gemm(dim3 grid, size_t smem, cudaStream_t st, const I4Args& a) {
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    const int max_smem = MT * 16 * (kI4MaxIters * kI4KIter / 8 + 1) * 16;
    cudaError_t e = cudaFuncSetAttribute(int4_gemm_kernel<MT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (e != cudaSuccess) return cuda_fail(e, "fi_int4_gemm: cudaFuncSetAttribute");
    attr_done[dev] = true;
  }
  int4_gemm_kernel<MT><<<grid, kI4Threads, smem, st>>>(a);
  return FI_OK;
}

}  // namespace fi

extern "C" size_t fi_int4_gemm_workspace_size(int64_t m, int64_t n, int64_t k,
                                              int64_t groupsize) {
  (void)groupsize;
  if (m <= 0 || n <= 0 || k <= 0 || m > fi::kI4MaxM) return 0;
  const fi::I4Plan p = fi::plan_int4(m, n, k);
  return p.counter_bytes + p.partial_bytes;
}

extern "C" int fi_int4_gemm(const void* x, const void* packed, const void* scales, void* c,
                            int64_t m, int64_t n, int64_t k, int64_t groupsize,
                            const int64_t* x_strides, const int64_t* packed_strides,
                            const int64_t* scales_strides, const int64_t* c_strides,
                            void* workspace, size_t workspace_bytes, void* stream) {
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
  if (n > (int64_t)kI4MaxCounters * kI4Cols || k > (1 << 30))
    return fail(FI_ERR_UNSUPPORTED, "fi_int4_gemm: N above %d or K above 2^30",
                kI4MaxCounters * kI4Cols);
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
  const I4Plan p = plan_int4(m, n, k);
  if (p.splits > 1) {
    if (!workspace || workspace_bytes < p.counter_bytes + p.partial_bytes)
      return fail(FI_ERR_WORKSPACE, "fi_int4_gemm: workspace needs %zu bytes, got %zu",
                  p.counter_bytes + p.partial_bytes, workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
      return fail(FI_ERR_ALIGNMENT, "fi_int4_gemm: workspace must be 256-byte aligned");
  }
  I4Args a;
  a.x = static_cast<const __half*>(x);
  a.w = static_cast<const uint8_t*>(packed);
  a.s = static_cast<const __half*>(scales);
  a.c = static_cast<__half*>(c);
  a.counters = static_cast<unsigned*>(workspace);
  a.partial = p.splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                                      p.counter_bytes)
                           : nullptr;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.gs = (int)groupsize;
  a.ks = p.ks;
  a.splits = p.splits;
  a.npad = p.npad;
  a.xs0 = x_strides[0];
  a.ws0 = packed_strides[0];
  a.ss0 = scales_strides[0];
  a.ss1 = scales_strides[1];
  a.cs0 = c_strides[0];
  a.cs1 = c_strides[1];
  const size_t smem = (size_t)p.mt * 16 * (p.ks / 8 + 1) * 16;
  const dim3 grid((unsigned)p.cbs, (unsigned)p.splits);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int r = FI_OK;
  switch (p.mt) {
    case 1: r = launch_int4_gemm<1>(grid, smem, st, a); break;
    case 2: r = launch_int4_gemm<2>(grid, smem, st, a); break;
    case 3: r = launch_int4_gemm<3>(grid, smem, st, a); break;
    default: r = launch_int4_gemm<4>(grid, smem, st, a); break;
  }
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
