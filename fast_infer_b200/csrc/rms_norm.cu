// RMSNorm for the attention stack: out = x * rsqrt(mean(x^2) + eps) * weight.
//
// Replaces kernels/rms_norm.py:29-43 (`rms_norm(x, weight, eps)`, Triton kernel
// :8-26) as called at model.py:82,141,153: fp16 in, fp32 arithmetic in the
// reference's order ((x * rms) * weight), fp16 out.
//
// One warp per row: the lanes take the row in 16-byte vectors, sum x^2 in fp32,
// reduce with shuffles and scale. Rows of up to 4096 elements are held in registers
// (every load of a lane issued before the first use, one pass over memory); longer
// rows loop and read the row twice. Rows are independent, so any number of rows
// (decode's batch or prefill's tokens) maps to ceil(rows / 8) CTAs of 8 warps.
#include <cuda_fp16.h>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kRmsWarps = 8;

// Rows of hidden <= VPL * 256 elements: each lane holds VPL 16-byte vectors.
template <int VPL>
__global__ void __launch_bounds__(kRmsWarps * 32)
    rms_norm_reg_kernel(const __half* x, const __half* w, __half* out, int64_t rows, int hidden,
                        int64_t xs0, int64_t os0, float eps) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRmsWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* xr = x + row * xs0;
  __half* orow = out + row * os0;
  const int vecs = hidden / 8;
  uint4 xv[VPL], wv[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    xv[i] = make_uint4(0u, 0u, 0u, 0u);
    wv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (v < vecs) {
      xv[i] = *reinterpret_cast<const uint4*>(xr + v * 8);
      wv[i] = __ldg(reinterpret_cast<const uint4*>(w + v * 8));
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const __half2* h = reinterpret_cast<const __half2*>(&xv[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rms = rsqrtf(ss / (float)hidden + eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    if (v >= vecs) break;
    const __half2* h = reinterpret_cast<const __half2*>(&xv[i]);
    const __half2* wh = reinterpret_cast<const __half2*>(&wv[i]);
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      const float2 g = __half22float2(wh[e]);
      oh[e] = __floats2half2_rn(f.x * rms * g.x, f.y * rms * g.y);
    }
    *reinterpret_cast<uint4*>(orow + v * 8) = o;
  }
}

__global__ void __launch_bounds__(kRmsWarps * 32)
    rms_norm_kernel(const __half* x, const __half* w, __half* out, int64_t rows, int hidden,
                    int64_t xs0, int64_t os0, float eps) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRmsWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __half* xr = x + row * xs0;
  __half* orow = out + row * os0;
  const int vecs = hidden / 8;
  float ss = 0.f;
  for (int v = lane; v < vecs; v += 32) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + v * 8);
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
  const float rms = rsqrtf(ss / (float)hidden + eps);
  for (int v = lane; v < vecs; v += 32) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + v * 8);
    const uint4 wu = *reinterpret_cast<const uint4*>(w + v * 8);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    const __half2* wh = reinterpret_cast<const __half2*>(&wu);
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      const float2 g = __half22float2(wh[e]);
      oh[e] = __floats2half2_rn(f.x * rms * g.x, f.y * rms * g.y);
    }
    *reinterpret_cast<uint4*>(orow + v * 8) = o;
  }
}

}  // namespace fi

extern "C" int fi_rms_norm(const void* x, const void* weight, void* out, int64_t rows,
                           int64_t hidden, int64_t x_row_stride, int64_t out_row_stride,
                           float eps, void* stream) {
  using namespace fi;
  clear_error();
  if (rows < 0 || hidden <= 0) return fail(FI_ERR_INVALID_ARG, "fi_rms_norm: bad sizes");
  if (hidden % 8 != 0 || hidden > (1 << 24))
    return fail(FI_ERR_UNSUPPORTED, "fi_rms_norm: hidden size must be a multiple of 8");
  if (rows == 0) return FI_OK;
  if (!x || !weight || !out) return fail(FI_ERR_INVALID_ARG, "fi_rms_norm: null pointer argument");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || x_row_stride % 8 != 0 ||
      out_row_stride % 8 != 0)
    return fail(FI_ERR_ALIGNMENT,
                "fi_rms_norm: needs 16-byte aligned x / weight / out and row strides that are "
                "multiples of 8");
  const int64_t blocks = (rows + kRmsWarps - 1) / kRmsWarps;
  if (blocks > 0x7fffffff) return fail(FI_ERR_UNSUPPORTED, "fi_rms_norm: too many rows");
  const __half* xp = static_cast<const __half*>(x);
  const __half* wp = static_cast<const __half*>(weight);
  __half* op = static_cast<__half*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)blocks, block = kRmsWarps * 32;
  const int vpl = (int)((hidden / 8 + 31) / 32);  // 16-byte vectors per lane
  cudaError_t e;
  if (vpl <= 4)
    e = launch_pdl(rms_norm_reg_kernel<4>, grid, block, 0, st, xp, wp, op, rows, (int)hidden,
                   x_row_stride, out_row_stride, eps);
  else if (vpl <= 8)
    e = launch_pdl(rms_norm_reg_kernel<8>, grid, block, 0, st, xp, wp, op, rows, (int)hidden,
                   x_row_stride, out_row_stride, eps);
  else if (vpl <= 12)
    e = launch_pdl(rms_norm_reg_kernel<12>, grid, block, 0, st, xp, wp, op, rows, (int)hidden,
                   x_row_stride, out_row_stride, eps);
  else if (vpl <= 16)
    e = launch_pdl(rms_norm_reg_kernel<16>, grid, block, 0, st, xp, wp, op, rows, (int)hidden,
                   x_row_stride, out_row_stride, eps);
  else
    e = launch_pdl(rms_norm_kernel, grid, block, 0, st, xp, wp, op, rows, (int)hidden, x_row_stride,
                   out_row_stride, eps);
  if (e != cudaSuccess) return cuda_fail(e, "fi_rms_norm launch");
  return FI_OK;
}
