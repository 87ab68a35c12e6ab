// Host helpers: thread-local error messages, tensor-map encoding, device queries.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>

#include "host_common.h"

namespace fi {

static thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = '\0'; }

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle, const char* what) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return fail(FI_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  if (!aligned16(base)) return fail(FI_ERR_ALIGNMENT, "%s: base pointer not 16-byte aligned", what);
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) {
      if (strides_bytes[i] % 16 != 0)
        return fail(FI_ERR_ALIGNMENT, "%s: stride of dim %u (%llu bytes) not a multiple of 16",
                    what, i + 1, (unsigned long long)strides_bytes[i]);
      s[i] = strides_bytes[i];
    }
  }
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FI_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return FI_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("FI_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int sm_count() {
  static std::atomic<int> counts[kMaxCachedDevices];  // zero-initialised (static storage)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  const bool cached = dev >= 0 && dev < kMaxCachedDevices;
  if (cached) {
    const int c = counts[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (cached) counts[dev].store(n, std::memory_order_relaxed);  // every writer stores the same n
  return n;
}

}  // namespace fi

extern "C" int fi_version(void) { return 100; }

extern "C" const char* fi_last_error(void) { return fi::g_last_error; }
