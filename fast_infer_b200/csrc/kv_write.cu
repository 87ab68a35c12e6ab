// KV-cache slot write: scatter new tokens' K/V rows into their pages.
//
// Replaces the per-(layer, sequence, block) torch copies of the reference
// (model.py:176-183 for prefill, model.py:196-201 for decode, kv_cache.py:69-102)
// with one launch that copies K and V together. The copy is byte-exact.
//
// Work decomposition: one thread moves one 16-byte chunk of one (token, head) row
// (head_dim 128 fp16 = 256 B = 16 chunks), so a warp covers two rows and every
// global access is a full, aligned 16-byte vector. When a stride is not a multiple
// of 8 elements the same grid runs with 2-byte element copies instead.
#include "common.cuh"
#include "host_common.h"

namespace fi {

struct KvWriteArgs {
  const __half* k;
  const __half* v;
  __half* kc;
  __half* vc;
  const int32_t* bt;
  const int32_t* start_pos;
  const int32_t* n_new;
  int* err;
  int64_t start_scalar;
  int64_t batch, num_new, heads, head_dim, num_blocks, block_size, max_blocks;
  int64_t ks[4], vs[4], kcs[4], vcs[4], bts[2];
};

template <bool kVec>
__global__ void __launch_bounds__(256) kv_write_kernel(const KvWriteArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t chunks_per_row = kVec ? a.head_dim / 8 : a.head_dim;
  const int64_t total = a.batch * a.num_new * a.heads * chunks_per_row;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = idx % chunks_per_row;
    int64_t r = idx / chunks_per_row;
    const int64_t h = r % a.heads;
    r /= a.heads;
    const int64_t t = r % a.num_new;
    const int64_t b = r / a.num_new;
    if (a.n_new && t >= a.n_new[b]) continue;
    const int64_t pos = (a.start_pos ? (int64_t)a.start_pos[b] : a.start_scalar) + t;
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
    const int64_t e = kVec ? c * 8 : c;
    const int64_t src_k = b * a.ks[0] + t * a.ks[1] + h * a.ks[2] + e * a.ks[3];
    const int64_t src_v = b * a.vs[0] + t * a.vs[1] + h * a.vs[2] + e * a.vs[3];
    const int64_t dst_k = phys * a.kcs[0] + slot * a.kcs[1] + h * a.kcs[2] + e * a.kcs[3];
    const int64_t dst_v = phys * a.vcs[0] + slot * a.vcs[1] + h * a.vcs[2] + e * a.vcs[3];
    if (kVec) {
      const uint4 kv = __ldg(reinterpret_cast<const uint4*>(a.k + src_k));
      const uint4 vv = __ldg(reinterpret_cast<const uint4*>(a.v + src_v));
      *reinterpret_cast<uint4*>(a.kc + dst_k) = kv;
      *reinterpret_cast<uint4*>(a.vc + dst_v) = vv;
    } else {
      a.kc[dst_k] = a.k[src_k];
      a.vc[dst_v] = a.v[src_v];
    }
  }
}

}  // namespace fi

extern "C" int fi_kv_write(const void* k, const void* v, void* k_cache, void* v_cache,
                           const int32_t* block_table, const int32_t* start_pos,
                           int64_t start_pos_scalar, const int32_t* n_new, int64_t batch,
                           int64_t num_new, int64_t num_kv_heads, int64_t head_dim,
                           int64_t num_blocks, int64_t block_size, int64_t max_blocks_per_seq,
                           const int64_t* k_strides, const int64_t* v_strides,
                           const int64_t* kc_strides, const int64_t* vc_strides,
                           const int64_t* bt_strides, int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (batch < 0 || num_new < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_blocks <= 0 ||
      block_size <= 0 || max_blocks_per_seq <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_kv_write: non-positive size");
  if (batch == 0 || num_new == 0) return FI_OK;
  if (!k || !v || !k_cache || !v_cache || !block_table || !k_strides || !v_strides ||
      !kc_strides || !vc_strides || !bt_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_kv_write: null pointer argument");
  KvWriteArgs a;
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.kc = static_cast<__half*>(k_cache);
  a.vc = static_cast<__half*>(v_cache);
  a.bt = block_table;
  a.start_pos = start_pos;
  a.n_new = n_new;
  a.err = error_flag;
  a.start_scalar = start_pos_scalar;
  a.batch = batch;
  a.num_new = num_new;
  a.heads = num_kv_heads;
  a.head_dim = head_dim;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.max_blocks = max_blocks_per_seq;
  bool vec = (head_dim % 8 == 0);
  for (int i = 0; i < 4; ++i) {
    a.ks[i] = k_strides[i];
    a.vs[i] = v_strides[i];
    a.kcs[i] = kc_strides[i];
    a.vcs[i] = vc_strides[i];
    if (i < 3)
      vec = vec && (a.ks[i] % 8 == 0) && (a.vs[i] % 8 == 0) && (a.kcs[i] % 8 == 0) &&
            (a.vcs[i] % 8 == 0);
  }
  vec = vec && a.ks[3] == 1 && a.vs[3] == 1 && a.kcs[3] == 1 && a.vcs[3] == 1;
  vec = vec && aligned16(k) && aligned16(v) && aligned16(k_cache) && aligned16(v_cache);
  a.bts[0] = bt_strides[0];
  a.bts[1] = bt_strides[1];
  if (!start_pos && start_pos_scalar < 0)
    return fail(FI_ERR_INVALID_ARG, "fi_kv_write: negative start position");
  if (!start_pos && !n_new && (start_pos_scalar + num_new + block_size - 1) / block_size >
                                  max_blocks_per_seq)
    return fail(FI_ERR_INVALID_ARG, "fi_kv_write: positions beyond the block table (%lld tokens)",
                (long long)(start_pos_scalar + num_new));
  const int64_t chunks = vec ? head_dim / 8 : head_dim;
  const int64_t total = batch * num_new * num_kv_heads * chunks;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      vec ? launch_pdl(kv_write_kernel<true>, dim3((unsigned)blocks), dim3(threads), 0, s, a)
          : launch_pdl(kv_write_kernel<false>, dim3((unsigned)blocks), dim3(threads), 0, s, a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_kv_write launch");
  return FI_OK;
}
