// Fused rotary embedding + KV-cache slot write.
//
// Replaces, in one launch, the reference's RoPE of q and k (kernels/rope.py:26-44,
// called at model.py:101 with cos/sin cast to fp16 at model.py:74-75) followed by
// the slot writes of k and v (model.py:162-201): from the QKV projection output it
//   * writes rotated q for the attention kernel,
//   * writes rotated k and the unchanged v into their pages of the KV pool,
//   * optionally writes rotated k to a dense tensor (the prefill attention input).
// Arithmetic reproduces the reference's fp16 tensor ops exactly: c = fp16(cos),
// s = fp16(sin), out = fp16(fp16(x * c) + fp16(rotate_half(x) * s)), where every
// product and sum is evaluated in fp32 and rounded to fp16, as PyTorch does.
//
// Work decomposition: a thread owns 8 dims of the first half of one head of one
// token and the matching 8 dims of the second half (rotate_half pairs d with
// d + D/2), so all loads and stores are 16-byte vectors.
#include "common.cuh"
#include "host_common.h"

namespace fi {

struct RopeArgs {
  const __half* qkv;
  const float* cos_tab;
  const float* sin_tab;
  const int32_t* start_pos;
  __half* q_out;
  __half* k_out;
  __half* kc;
  __half* vc;
  const int32_t* bt;
  int* err;
  int64_t start_scalar, max_pos;
  int64_t batch, seq, nq, nkv, hd;
  int64_t num_blocks, block_size, max_blocks;
  int64_t xs[3], qs[4], ks[4], kcs[4], vcs[4], bts[2], tab_stride;
};

__global__ void __launch_bounds__(256) rope_kv_write_kernel(const RopeArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t half_chunks = a.hd / 16;  // 8-dim chunks per half
  const int64_t heads = a.nq + 2 * a.nkv;
  const int64_t total = a.batch * a.seq * heads * half_chunks;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = idx % half_chunks;
    int64_t r = idx / half_chunks;
    const int64_t h = r % heads;
    r /= heads;
    const int64_t t = r % a.seq;
    const int64_t b = r / a.seq;
    const int64_t pos = (a.start_pos ? (int64_t)a.start_pos[b] : a.start_scalar) + t;
    const int64_t d0 = c * 8, d1 = a.hd / 2 + c * 8;
    const __half* src = a.qkv + b * a.xs[0] + t * a.xs[1] + h * a.hd * a.xs[2];
    const uint4 lo_raw = *reinterpret_cast<const uint4*>(src + d0 * a.xs[2]);
    const uint4 hi_raw = *reinterpret_cast<const uint4*>(src + d1 * a.xs[2]);
    uint4 lo_out = lo_raw, hi_out = hi_raw;
    const bool is_v = h >= a.nq + a.nkv;
    if (!is_v) {
      if (pos < 0 || pos >= a.max_pos) {
        if (c == 0) set_error(a.err, FI_DEVERR_CONTEXT_LEN);
        continue;
      }
      const float* ct = a.cos_tab + pos * a.tab_stride;
      const float* st = a.sin_tab + pos * a.tab_stride;
      const __half* xl = reinterpret_cast<const __half*>(&lo_raw);
      const __half* xh = reinterpret_cast<const __half*>(&hi_raw);
      __half* ol = reinterpret_cast<__half*>(&lo_out);
      __half* oh = reinterpret_cast<__half*>(&hi_out);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xlo = __half2float(xl[e]), xhi = __half2float(xh[e]);
        // rotate_half(x) = [-x_hi, x_lo]
        ol[e] = rope_elem(xlo, -xhi, __float2half_rn(ct[d0 + e]), __float2half_rn(st[d0 + e]));
        oh[e] = rope_elem(xhi, xlo, __float2half_rn(ct[d1 + e]), __float2half_rn(st[d1 + e]));
      }
    }
    if (h < a.nq) {
      __half* dst = a.q_out + b * a.qs[0] + t * a.qs[1] + h * a.qs[2];
      *reinterpret_cast<uint4*>(dst + d0 * a.qs[3]) = lo_out;
      *reinterpret_cast<uint4*>(dst + d1 * a.qs[3]) = hi_out;
      continue;
    }
    const int64_t kvh = is_v ? h - a.nq - a.nkv : h - a.nq;
    if (!is_v && a.k_out) {
      __half* dst = a.k_out + b * a.ks[0] + t * a.ks[1] + kvh * a.ks[2];
      *reinterpret_cast<uint4*>(dst + d0 * a.ks[3]) = lo_out;
      *reinterpret_cast<uint4*>(dst + d1 * a.ks[3]) = hi_out;
    }
    const int64_t lblk = pos / a.block_size;
    if (pos < 0 || lblk >= a.max_blocks) {
      if (c == 0) set_error(a.err, FI_DEVERR_BAD_BLOCK);
      continue;
    }
    const int64_t phys = a.bt[b * a.bts[0] + lblk * a.bts[1]];
    if (phys < 0 || phys >= a.num_blocks) {
      if (c == 0) set_error(a.err, FI_DEVERR_BAD_BLOCK);
      continue;
    }
    const int64_t slot = pos % a.block_size;
    const int64_t* cs = is_v ? a.vcs : a.kcs;
    __half* dst = (is_v ? a.vc : a.kc) + phys * cs[0] + slot * cs[1] + kvh * cs[2];
    *reinterpret_cast<uint4*>(dst + d0 * cs[3]) = lo_out;
    *reinterpret_cast<uint4*>(dst + d1 * cs[3]) = hi_out;
  }
}

}  // namespace fi

extern "C" int fi_rope_kv_write(const void* qkv, int64_t batch, int64_t seq, int64_t num_q_heads,
                                int64_t num_kv_heads, int64_t head_dim, const int64_t* qkv_strides,
                                const float* cos_table, const float* sin_table, int64_t table_rows,
                                int64_t table_stride, const int32_t* start_pos,
                                int64_t start_pos_scalar, void* q_out, const int64_t* q_out_strides,
                                void* k_out, const int64_t* k_out_strides, void* k_cache,
                                void* v_cache, const int32_t* block_table, int64_t num_blocks,
                                int64_t block_size, int64_t max_blocks_per_seq,
                                const int64_t* kc_strides, const int64_t* vc_strides,
                                const int64_t* bt_strides, int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (batch < 0 || seq < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      block_size <= 0 || max_blocks_per_seq <= 0 || table_rows <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_rope_kv_write: non-positive size");
  if (head_dim <= 0 || head_dim % 16 != 0 || head_dim > 512)
    return fail(FI_ERR_UNSUPPORTED, "fi_rope_kv_write: head_dim must be a multiple of 16 (<= 512)");
  if (batch == 0 || seq == 0) return FI_OK;
  if (!qkv || !cos_table || !sin_table || !q_out || !k_cache || !v_cache || !block_table ||
      !qkv_strides || !q_out_strides || !kc_strides || !vc_strides || !bt_strides ||
      (k_out && !k_out_strides))
    return fail(FI_ERR_INVALID_ARG, "fi_rope_kv_write: null pointer argument");
  if (table_stride < head_dim) return fail(FI_ERR_INVALID_ARG, "fi_rope_kv_write: table_stride < head_dim");
  if (!start_pos && (start_pos_scalar < 0 || start_pos_scalar + seq > table_rows))
    return fail(FI_ERR_INVALID_ARG, "fi_rope_kv_write: positions beyond the rotary table");
  RopeArgs a;
  a.qkv = static_cast<const __half*>(qkv);
  a.cos_tab = cos_table;
  a.sin_tab = sin_table;
  a.start_pos = start_pos;
  a.q_out = static_cast<__half*>(q_out);
  a.k_out = static_cast<__half*>(k_out);
  a.kc = static_cast<__half*>(k_cache);
  a.vc = static_cast<__half*>(v_cache);
  a.bt = block_table;
  a.err = error_flag;
  a.start_scalar = start_pos_scalar;
  a.max_pos = table_rows;
  a.batch = batch;
  a.seq = seq;
  a.nq = num_q_heads;
  a.nkv = num_kv_heads;
  a.hd = head_dim;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.max_blocks = max_blocks_per_seq;
  a.tab_stride = table_stride;
  for (int i = 0; i < 3; ++i) a.xs[i] = qkv_strides[i];
  for (int i = 0; i < 4; ++i) {
    a.qs[i] = q_out_strides[i];
    a.ks[i] = k_out ? k_out_strides[i] : 0;
    a.kcs[i] = kc_strides[i];
    a.vcs[i] = vc_strides[i];
  }
  a.bts[0] = bt_strides[0];
  a.bts[1] = bt_strides[1];
  // 16-byte vectors everywhere: unit innermost strides, other strides multiples of 8.
  bool ok = a.xs[2] == 1 && a.qs[3] == 1 && a.kcs[3] == 1 && a.vcs[3] == 1 &&
            (!k_out || a.ks[3] == 1);
  ok = ok && a.xs[0] % 8 == 0 && a.xs[1] % 8 == 0;
  for (int i = 0; i < 3; ++i)
    ok = ok && a.qs[i] % 8 == 0 && a.kcs[i] % 8 == 0 && a.vcs[i] % 8 == 0 &&
         (!k_out || a.ks[i] % 8 == 0);
  ok = ok && aligned16(qkv) && aligned16(q_out) && aligned16(k_cache) && aligned16(v_cache) &&
       (!k_out || aligned16(k_out));
  if (!ok)
    return fail(FI_ERR_ALIGNMENT,
                "fi_rope_kv_write: tensors need 16-byte aligned bases, unit innermost strides and "
                "other strides that are multiples of 8 elements");
  const int64_t total = batch * seq * (num_q_heads + 2 * num_kv_heads) * (head_dim / 16);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  const cudaError_t e = launch_pdl(rope_kv_write_kernel, dim3((unsigned)blocks), dim3(threads), 0,
                                   static_cast<cudaStream_t>(stream), a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_rope_kv_write launch");
  return FI_OK;
}
