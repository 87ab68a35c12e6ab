// Paged decode with no device allocation: the split-KV scratch lives in a
// file-scope static device array instead of a caller-provided workspace.
//
// Who needs this: callers that reach the C ABI without a device allocator of their
// own — a C/C++ host that links only this library (no caching allocator) and must
// not pay cudaMalloc's implicit device synchronisation on the per-token decode
// path, or a serving runtime that forbids allocation after start-up so its memory
// footprint stays fixed. They still pass every input and output buffer; only the
// scratch is provided here.
//
// Limits and sharing:
// * The array holds FI_NOALLOC_SCRATCH_BYTES (16 MiB). Every GPU that loads the
//   library keeps that much device memory until the process exits.
// * Sizes whose split-KV scratch (fi_paged_decode_workspace_size) exceeds it are
//   rejected with FI_ERR_WORKSPACE before anything is launched.
// * All calls on a device share the one array. Nothing in it has to start at zero
//   (each call writes every partial it reads back), but calls whose kernels
//   overlap on the GPU — e.g. issued on different streams without ordering — race
//   on it. Order such calls on one stream or use fi_paged_decode with separate
//   workspaces.
// * The first call on each device resolves the array's device address with
//   cudaGetSymbolAddress (that device current); make that first call before any
//   stream capture. The address is kept per device together with the unique ID of
//   the CUDA context it was resolved in: a call from another context on that device
//   (after cudaDeviceReset, or a caller's own non-primary context) resolves it again
//   in that context, which is then a first call too.
#include <mutex>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[FI_NOALLOC_SCRATCH_BYTES];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique ID of the calling thread's current CUDA context (cuCtxGetId: never reused
// within a process, unlike the context handle). False if there is none or the
// driver lacks the call.
static bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

struct ScratchAddress {
  unsigned long long ctx_id;  // context the address was resolved in
  void* ptr;                  // nullptr: not resolved yet
};
static std::mutex g_scratch_mu;
static ScratchAddress g_scratch[kNoAllocMaxDevices] = {};

// Device address of g_decode_scratch in the current device's current context
// (resolved once per device and context). In host code the symbol name is only a
// host-side stand-in, never a device address.
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "fi_paged_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(FI_ERR_UNSUPPORTED, "fi_paged_decode_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  unsigned long long id = 0;
  bool have_id = current_context_id(&id);
  ScratchAddress& c = g_scratch[dev];
  if (have_id && c.ptr != nullptr && c.ctx_id == id) {
    *out = c.ptr;
    return FI_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "fi_paged_decode_noalloc: cudaGetSymbolAddress");
  if (!have_id) have_id = current_context_id(&id);  // the lookup may have made the context
  // without a context ID nothing is cached: the next call looks the address up again
  c = have_id ? ScratchAddress{id, p} : ScratchAddress{0, nullptr};
  *out = p;
  return FI_OK;
}

}  // namespace fi

extern "C" int fi_paged_decode_noalloc(
    const void* q, const void* k_cache, const void* v_cache, void* o, const int32_t* block_table,
    const int32_t* context_lens, int64_t num_tokens, int64_t max_context_len, int64_t batch,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t block_size, int64_t max_blocks_per_seq, const int64_t* q_strides,
    const int64_t* kc_strides, const int64_t* vc_strides, const int64_t* o_strides,
    const int64_t* bt_strides, float sm_scale, int64_t pages_per_split, int32_t* error_flag,
    void* stream) {
  using namespace fi;
  clear_error();
  // The launch bound fi_paged_decode itself uses: the scalar token count when no
  // per-sequence lengths are given, never more than the block table spans.
  int64_t bound = context_lens ? max_context_len : num_tokens;
  if (bound > max_blocks_per_seq * block_size) bound = max_blocks_per_seq * block_size;
  const size_t need = fi_paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                     bound, block_size, pages_per_split);
  if (need > (size_t)FI_NOALLOC_SCRATCH_BYTES)
    return fail(FI_ERR_WORKSPACE,
                "fi_paged_decode_noalloc: these sizes need %zu bytes of split-KV scratch, more "
                "than the %d-byte static scratch; use fi_paged_decode with a workspace or a "
                "larger pages_per_split",
                need, (int)FI_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    const int r = scratch_address(&scratch);
    if (r != FI_OK) return r;
  }
  return fi_paged_decode(q, k_cache, v_cache, o, block_table, context_lens, num_tokens,
                         max_context_len, batch, num_q_heads, num_kv_heads, head_dim, num_blocks,
                         block_size, max_blocks_per_seq, q_strides, kc_strides, vc_strides,
                         o_strides, bt_strides, sm_scale, pages_per_split, scratch,
                         need > 0 ? (size_t)FI_NOALLOC_SCRATCH_BYTES : 0, error_flag, stream);
}
