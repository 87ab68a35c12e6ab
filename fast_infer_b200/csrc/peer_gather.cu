// All-gather of per-rank attention outputs over NVLink peer memory (CUDA IPC).
//
// Replaces, for the decode step of a KV-head-sharded stack, the NCCL all-gather of
// the per-rank head outputs before the replicated O projection (the one exchange of
// the sharded path, model.py:123-134 run with heads split over GPUs). One kernel per
// gather writes this rank's [rows, row_bytes] block straight into every rank's
// gather buffer (plain 16-byte stores through the peer mapping, NVLink), then
// raises this rank's flag in every peer and waits (bounded) until every peer's flag
// for the same call has arrived: no library collective, no host involvement, one
// launch, CUDA-graph capturable.
//
// Each rank owns one region (fi_peer_alloc, shared with the others through
// cudaIpcGetMemHandle / cudaIpcOpenMemHandle):
//   [nbuf gather buffers: nbuf x max_rows x row_total bytes]
//   [flags: 64 x uint32, flags[p] = number of gathers rank p has delivered here]
//   [local: epoch (gathers done by this rank), CTA arrival counter]
// Calls are counted on the device (epoch), so a replayed graph waits for the
// matching call of every peer. A buffer must not be rewritten while a peer may still
// read it: callers rotate buffers so that two uses of one buffer have another
// gather between them (the stack uses one buffer per layer).
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kPgMaxWorld = 8;
constexpr int kPgFlags = 64;       // uint32 flag slots (world <= 8, padded to 256 bytes)
constexpr int kPgThreads = 256;

struct PeerGatherArgs {
  const uint8_t* src;
  int64_t rows, row_bytes, src_stride;  // bytes
  uint8_t* base[kPgMaxWorld];           // each rank's region as mapped here
  int world, rank;
  int64_t data_off;                     // this call's buffer within a region
  int64_t row_total;                    // world * row_bytes
  int64_t flags_off;                    // flags array within a region
  uint32_t* epoch;                      // this rank's local state
  uint32_t* counter;
  int* err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__global__ void __launch_bounds__(kPgThreads) peer_gather_kernel(const PeerGatherArgs a) {
  grid_dep_wait();  // the rows come from the previous kernel
  const int64_t vpr = a.row_bytes / 16;
  const int64_t total = a.rows * vpr;
  for (int64_t i = blockIdx.x * (int64_t)kPgThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kPgThreads) {
    const int64_t r = i / vpr, c = i - r * vpr;
    const uint4 v = *reinterpret_cast<const uint4*>(a.src + r * a.src_stride + c * 16);
    const int64_t off = a.data_off + r * a.row_total + a.rank * a.row_bytes + c * 16;
    for (int p = 0; p < a.world; ++p) *reinterpret_cast<uint4*>(a.base[p] + off) = v;
  }
  // One system-scope fence per CTA: the barrier orders the CTA's stores before it.
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  if (gridDim.x > 1) {
    if (atomicAdd(a.counter, 1u) != gridDim.x - 1) return;
    // Last CTA: every CTA's stores were fenced before its arrival.
    atomicExch(a.counter, 0u);
    __threadfence_system();
  }
  // Publish this call to every rank, then wait for the same call of every rank.
  const uint32_t e = *a.epoch + 1;
  *a.epoch = e;
  for (int p = 0; p < a.world; ++p)
    st_release_sys(reinterpret_cast<uint32_t*>(a.base[p] + a.flags_off) + a.rank, e);
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.base[a.rank] + a.flags_off);
  // After one wait has run out (a peer gone or stuck) later calls do not wait again:
  // a persistent error word turns a broken rendezvous into one 2 s delay, not one
  // per call.
  if (a.err && (*reinterpret_cast<volatile int*>(a.err) & FI_DEVERR_TIMEOUT)) return;
  const unsigned long long t0 = globaltimer_ns();
  for (int p = 0; p < a.world; ++p) {
    uint32_t spins = 0;
    while ((int32_t)(ld_relaxed_sys(mine + p) - e) < 0) {
      if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        set_error(a.err, FI_DEVERR_TIMEOUT);
        return;
      }
    }
  }
  fence_acq_rel_sys();  // the peers' rows are visible to this kernel's successors
}

static int64_t pg_data_bytes(int64_t nbuf, int64_t max_rows, int64_t row_total) {
  return (nbuf * max_rows * row_total + 255) / 256 * 256;
}

}  // namespace fi

extern "C" size_t fi_peer_gather_bytes(int64_t nbuf, int64_t max_rows, int64_t row_total_bytes) {
  using namespace fi;
  if (nbuf <= 0 || max_rows <= 0 || row_total_bytes <= 0) return 0;
  return (size_t)(pg_data_bytes(nbuf, max_rows, row_total_bytes) + kPgFlags * 4 + 256);
}

extern "C" int fi_peer_alloc(size_t bytes, void** ptr, void* handle) {
  using namespace fi;
  clear_error();
  if (!ptr || !handle || bytes == 0) return fail(FI_ERR_INVALID_ARG, "fi_peer_alloc: bad argument");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "fi_peer_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "fi_peer_alloc");
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return FI_OK;
}

extern "C" int fi_peer_open(const void* handle, void** ptr) {
  using namespace fi;
  clear_error();
  if (!ptr || !handle) return fail(FI_ERR_INVALID_ARG, "fi_peer_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "fi_peer_open: cudaIpcOpenMemHandle");
  *ptr = p;
  return FI_OK;
}

extern "C" int fi_peer_close(void* ptr) {
  using namespace fi;
  clear_error();
  if (!ptr) return FI_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? FI_OK : cuda_fail(e, "fi_peer_close");
}

extern "C" int fi_peer_free(void* ptr) {
  using namespace fi;
  clear_error();
  if (!ptr) return FI_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? FI_OK : cuda_fail(e, "fi_peer_free");
}

extern "C" int fi_peer_gather(const void* src, int64_t rows, int64_t row_bytes,
                              int64_t src_row_stride_bytes, void* const* bases, int64_t world,
                              int64_t rank, int64_t buffer, int64_t nbuf, int64_t max_rows,
                              int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (world < 1 || world > kPgMaxWorld || rank < 0 || rank >= world)
    return fail(FI_ERR_INVALID_ARG, "fi_peer_gather: world %lld / rank %lld", (long long)world,
                (long long)rank);
  if (rows < 0 || rows > max_rows || row_bytes <= 0 || nbuf <= 0 || buffer < 0 || buffer >= nbuf)
    return fail(FI_ERR_INVALID_ARG, "fi_peer_gather: bad sizes or buffer index");
  if (row_bytes % 16 != 0 || src_row_stride_bytes % 16 != 0 || !aligned16(src))
    return fail(FI_ERR_ALIGNMENT,
                "fi_peer_gather: rows must be 16-byte aligned multiples of 16 bytes");
  if (!src || !bases) return fail(FI_ERR_INVALID_ARG, "fi_peer_gather: null pointer argument");
  PeerGatherArgs a;
  memset(&a, 0, sizeof(a));
  for (int p = 0; p < world; ++p) {
    if (!bases[p] || !aligned16(bases[p]))
      return fail(FI_ERR_INVALID_ARG, "fi_peer_gather: region of rank %d missing or unaligned", p);
    a.base[p] = static_cast<uint8_t*>(bases[p]);
  }
  a.src = static_cast<const uint8_t*>(src);
  a.rows = rows;
  a.row_bytes = row_bytes;
  a.src_stride = src_row_stride_bytes;
  a.world = (int)world;
  a.rank = (int)rank;
  a.row_total = world * row_bytes;
  a.data_off = buffer * max_rows * a.row_total;
  a.flags_off = pg_data_bytes(nbuf, max_rows, a.row_total);
  uint32_t* local = reinterpret_cast<uint32_t*>(a.base[rank] + a.flags_off) + kPgFlags;
  a.epoch = local;
  a.counter = local + 1;
  a.err = error_flag;
  const int64_t total = rows * (row_bytes / 16);
  int64_t blocks = (total + kPgThreads * 8 - 1) / (kPgThreads * 8);  // ~8 vectors a thread
  if (blocks < 1) blocks = 1;
  const int64_t cap = (int64_t)sm_count() * 4;
  if (blocks > cap) blocks = cap;
  cudaError_t e = launch_pdl(peer_gather_kernel, dim3((unsigned)blocks), dim3(kPgThreads), 0,
                             static_cast<cudaStream_t>(stream), a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_peer_gather launch");
  return FI_OK;
}
