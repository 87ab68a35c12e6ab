// All-gather of per-rank attention outputs over NVLink peer memory (CUDA IPC).
//
// Replaces, for the decode step of a KV-head-sharded stack, the NCCL all-gather of
// the per-rank head outputs before the replicated O projection (the one exchange of
// the sharded path, model.py:123-134 run with heads split over GPUs). One kernel per
// gather, no library collective, no host involvement, CUDA-graph capturable.
//
// Protocol: flags travel inside the data. Every 4-byte word of this rank's rows is
// sent to every rank as one 8-byte store {word, epoch} (an 8-byte store reaches the
// peer whole), so no system-scope fence is needed: each rank polls the words of its
// own landing area until every word carries the current call's epoch, unpacking
// them into its output rows. The epoch counts calls on the device, so a replayed
// graph matches calls across ranks, and a stale word (an older call) never passes.
//
// Each rank owns one region (fi_peer_alloc, shared with the others through
// cudaIpcGetMemHandle / cudaIpcOpenMemHandle):
//   [output: nbuf buffers x max_rows x row_total bytes]   (row_total = world x row)
//   [landing area: nbuf x max_rows x world x row words, 8 bytes each]
//   [local: epoch (calls made by this rank), CTA arrival counter]
// A buffer must not be rewritten while a peer may still read it: callers rotate
// buffers so that two uses of one buffer have another gather between them (the
// stack uses one buffer per layer).
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
  int64_t rows, row_words, src_stride;  // row_words: 4-byte words per row; stride in bytes
  uint8_t* base[kPgMaxWorld];           // each rank's region as mapped here
  int world, rank;
  int64_t out_off;                      // this call's output buffer within a region
  int64_t land_off;                     // this call's landing area within a region
  uint32_t* epoch;                      // this rank's local state
  uint32_t* counter;
  int* err;
};

__device__ __forceinline__ void st_pair(uint32_t* p, uint32_t v, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v), "r"(flag) : "memory");
}
__device__ __forceinline__ void ld_pair(const uint32_t* p, uint32_t& v, uint32_t& flag) {
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v), "=r"(flag) : "l"(p) : "memory");
}

__global__ void __launch_bounds__(kPgThreads) peer_gather_kernel(const PeerGatherArgs a) {
  grid_dep_wait();  // the rows come from the previous kernel; the last call has finished
  const uint32_t e = *a.epoch + 1;  // this call's epoch (raised by the last CTA below)
  const int64_t rw = a.row_words;
  const int64_t nthreads = (int64_t)gridDim.x * kPgThreads;
  const int64_t t0i = blockIdx.x * (int64_t)kPgThreads + threadIdx.x;
  // ---- send: word w of row r -> landing slot (r, rank, w) of every rank
  for (int64_t i = t0i; i < a.rows * rw; i += nthreads) {
    const int64_t r = i / rw, w = i - r * rw;
    const uint32_t v = *reinterpret_cast<const uint32_t*>(a.src + r * a.src_stride + w * 4);
    const int64_t slot = (r * a.world + a.rank) * rw + w;
    for (int p = 0; p < a.world; ++p)
      st_pair(reinterpret_cast<uint32_t*>(a.base[p] + a.land_off) + 2 * slot, v, e);
  }
  // ---- receive: every rank's words of every row, unpacked to [row][rank][word]
  uint32_t* land = reinterpret_cast<uint32_t*>(a.base[a.rank] + a.land_off);
  uint32_t* out = reinterpret_cast<uint32_t*>(a.base[a.rank] + a.out_off);
  // after one wait has run out (a peer gone or stuck) later calls do not wait again
  bool give_up = a.err && (*reinterpret_cast<volatile int*>(a.err) & FI_DEVERR_TIMEOUT);
  const unsigned long long t0 = globaltimer_ns();
  for (int64_t i = t0i; i < a.rows * a.world * rw; i += nthreads) {
    uint32_t v, f;
    ld_pair(land + 2 * i, v, f);
    uint32_t spins = 0;
    while (f != e && !give_up) {
      if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        set_error(a.err, FI_DEVERR_TIMEOUT);
        give_up = true;
      }
      ld_pair(land + 2 * i, v, f);
    }
    out[i] = v;  // landing slot (r, p, w) and output word (r, p*rw + w) share the index
  }
  // ---- the last CTA to finish raises the epoch for the next call
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.counter, 1u) == gridDim.x - 1) {
    atomicExch(a.counter, 0u);
    *a.epoch = e;
  }
}

// Output buffers, then the landing area (8 bytes per 4-byte word).
static int64_t pg_out_bytes(int64_t nbuf, int64_t max_rows, int64_t row_total) {
  return (nbuf * max_rows * row_total + 255) / 256 * 256;
}
static int64_t pg_data_bytes(int64_t nbuf, int64_t max_rows, int64_t row_total) {
  return pg_out_bytes(nbuf, max_rows, row_total) + 2 * pg_out_bytes(nbuf, max_rows, row_total);
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
  // A rank that has received every word of call k may start call k+1 while a slower
  // rank still reads call k's landing area; with one buffer its sends would overwrite
  // words the slower rank has not read yet.
  if (world > 1 && nbuf < 2)
    return fail(FI_ERR_INVALID_ARG, "fi_peer_gather: %lld ranks need at least 2 buffers",
                (long long)world);
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
  a.row_words = row_bytes / 4;
  a.src_stride = src_row_stride_bytes;
  a.world = (int)world;
  a.rank = (int)rank;
  const int64_t row_total = world * row_bytes;
  a.out_off = buffer * max_rows * row_total;
  a.land_off = pg_out_bytes(nbuf, max_rows, row_total) + 2 * buffer * max_rows * row_total;
  uint32_t* local = reinterpret_cast<uint32_t*>(a.base[rank] +
                                                pg_data_bytes(nbuf, max_rows, row_total)) +
                    kPgFlags;
  a.epoch = local;
  a.counter = local + 1;
  a.err = error_flag;
  const int64_t total = rows * world * (row_bytes / 4);  // words received
  int64_t blocks = (total + kPgThreads * 16 - 1) / (kPgThreads * 16);  // ~16 words a thread
  if (blocks < 1) blocks = 1;
  const int64_t cap = (int64_t)sm_count() * 4;
  if (blocks > cap) blocks = cap;
  cudaError_t e = launch_pdl(peer_gather_kernel, dim3((unsigned)blocks), dim3(kPgThreads), 0,
                             static_cast<cudaStream_t>(stream), a);
  if (e != cudaSuccess) return cuda_fail(e, "fi_peer_gather launch");
  return FI_OK;
}
