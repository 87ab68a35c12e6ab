// Causal prefill attention (FlashAttention forward) on sm_100a tensor cores.
//
// Replaces the Triton kernel `_flash_attn_fwd` and its launcher `flash_attention`
// (reference kernels/attention.py:8-113). Semantics, per (batch b, query head h,
// query row i):  o[b,h,i] = sum_{j<=i} softmax_j(q[b,h,i].k[b,hk,j] * scale) v[b,hk,j]
// with hk = h / (Hq / Hk); fp16 in, fp32 softmax/accumulation, fp16 out.
//
// B200 design:
// * A CTA owns 256 consecutive query rows of one head as two 128-row tiles (T0, T1)
//   that share every K/V tile fetched; work units are issued longest-first so the
//   causal triangle load-balances across the 148 SMs.
// * Warp roles (320 threads): warps 0-3 = softmax/epilogue of T0, warps 4-7 = T1,
//   warp 8 = TMA producer, warp 9 = UMMA issuer (one thread).
// * Tensor memory (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each.
//   S_t = Q_t K^T is a 128x128x128 tcgen05.mma (A, B from 128B-swizzled shared
//   memory, K-major). Softmax threads own one row each (TMEM lane = row), read S
//   with tcgen05.ld, write P as packed fp16 over the first 64 columns of S_t, and
//   the PV product O_t += P V reads P straight from tensor memory (A operand in
//   TMEM, V as an MN-major shared-memory operand). No S/P round trip through
//   shared memory or registers of other warps.
// * Online softmax in base 2 with a lazy rescale: O_t and l are rescaled only when
//   a row's running max grows by more than 8 (2^8 headroom in fp16 P), which after
//   the first tiles almost never happens. The result is exact either way because
//   numerator and denominator use the same stale max.
// * The MMA issue order S0(j), S1(j), PV0(j), S0(j+1), PV1(j), S1(j+1), ... lets
//   the tensor core work on one tile while the other tile's softmax runs.
// * Epilogue: O/l -> fp16 into the (now idle) Q tile's shared memory in the same
//   swizzled layout, then one TMA store per 64-column half (rows past seq_len are
//   clipped by the tensor map).
#include <math.h>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kBM = 128;            // query rows per tile
constexpr int kBN = 128;            // keys per KV tile
constexpr int kHD = 128;            // head dim
constexpr int kHalfBytes = kBM * 128;      // 128 rows x 64 fp16 (one swizzle column)
constexpr int kTileBytes = 2 * kHalfBytes; // 32 KB: a 128 x 128 fp16 tile
constexpr int kPfThreads = 320;
constexpr int kPfStages = 2;
// Q0, Q1, K[2], V[2] tiles + barriers + tmem slot, plus 1 KB for alignment.
constexpr int kPfSmemBytes = 1024 + (2 + 2 * kPfStages) * kTileBytes + 256;

constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillParams {
  int batch, hq, hk, group, seq_len, npairs;
  float scale_log2;
  int* err;
};

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 "version 1" format).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: f16 x f16 -> f32, M = 128, N = 128.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t a_mn_major, uint32_t b_mn_major) {
  return (1u << 4) | (a_mn_major << 15) | (b_mn_major << 16) | ((uint32_t)(kBN >> 3) << 17) |
         ((uint32_t)(kBM >> 4) << 24);
}

struct PfBarriers {
  uint64_t q_full;
  uint64_t k_full[kPfStages], k_empty[kPfStages];
  uint64_t v_full[kPfStages], v_empty[kPfStages];
  uint64_t s_full[2], p_full[2], o_full[2];
  uint64_t mma_done;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // 2 tiles
  uint8_t* sK = smem + 2 * kTileBytes;                 // kPfStages tiles
  uint8_t* sV = sK + kPfStages * kTileBytes;           // kPfStages tiles
  PfBarriers* bars = reinterpret_cast<PfBarriers*>(sV + kPfStages * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Work unit: longest (largest pair index) first; heads of one KV group adjacent.
  const int per_pair = p.batch * p.hq;
  const int pair = p.npairs - 1 - (int)(blockIdx.x / per_pair);
  const int rem = (int)(blockIdx.x % per_pair);
  const int b = rem / p.hq, h = rem % p.hq;
  const int hk = h / p.group;
  int n_tiles[2];
  bool live[2];
  for (int t = 0; t < 2; ++t) {
    const int r0 = pair * 2 * kBM + t * kBM;
    live[t] = r0 < p.seq_len;
    n_tiles[t] = live[t] ? r0 / kBN + 1 : 0;
  }
  const int nkv = live[1] ? n_tiles[1] : n_tiles[0];

  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 4);
      mbar_init(&bars->o_full[t], 1);
    }
    mbar_init(&bars->mma_done, 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      const int q_bytes = (live[0] ? kTileBytes : 0) + (live[1] ? kTileBytes : 0);
      mbar_arrive_expect_tx(&bars->q_full, q_bytes);
      for (int t = 0; t < 2; ++t) {
        if (!live[t]) continue;
        const int r0 = pair * 2 * kBM + t * kBM;
        tma_load_4d(sQ + t * kTileBytes, &tm_q, &bars->q_full, 0, r0, h, b);
        tma_load_4d(sQ + t * kTileBytes + kHalfBytes, &tm_q, &bars->q_full, 64, r0, h, b);
      }
      for (int j = 0; j < nkv; ++j) {
        const int s = j % kPfStages;
        const uint32_t par = ((j / kPfStages) - 1) & 1;
        if (j >= kPfStages && !mbar_wait(&bars->k_empty[s], par, p.err)) break;
        mbar_arrive_expect_tx(&bars->k_full[s], kTileBytes);
        tma_load_4d(sK + s * kTileBytes, &tm_k, &bars->k_full[s], 0, j * kBN, hk, b);
        tma_load_4d(sK + s * kTileBytes + kHalfBytes, &tm_k, &bars->k_full[s], 64, j * kBN, hk, b);
        if (j >= kPfStages && !mbar_wait(&bars->v_empty[s], par, p.err)) break;
        mbar_arrive_expect_tx(&bars->v_full[s], kTileBytes);
        tma_load_4d(sV + s * kTileBytes, &tm_v, &bars->v_full[s], 0, j * kBN, hk, b);
        tma_load_4d(sV + s * kTileBytes + kHalfBytes, &tm_v, &bars->v_full[s], 64, j * kBN, hk, b);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_f16(0, 0);
      constexpr uint32_t idesc_pv = umma_idesc_f16(0, 1);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(&bars->q_full, 0, p.err);
      auto issue_s = [&](int t, int j) {
        const uint32_t qa = q_addr + t * kTileBytes;
        const uint32_t ka = k_addr + (j % kPfStages) * kTileBytes;
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_ss(tmem + t * kBN, umma_desc_sw128(qa + off, 16, 1024),
                  umma_desc_sw128(ka + off, 16, 1024), idesc_qk, k > 0);
        }
        umma_commit(&bars->s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t va = v_addr + (j % kPfStages) * kTileBytes;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          umma_ts(tmem + 256 + t * kHD, tmem + t * kBN + k * 8,
                  umma_desc_sw128(va + k * 16 * 128, kHalfBytes, 1024), idesc_pv,
                  (j > 0 || k > 0) ? 1u : 0u);
        }
      };
      if (ok && nkv > 0) {
        ok = mbar_wait(&bars->k_full[0], 0, p.err);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < 2; ++t)
            if (live[t]) issue_s(t, 0);
        }
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const bool has_next = j + 1 < nkv;
        if (has_next) {
          ok = mbar_wait(&bars->k_full[(j + 1) % kPfStages], ((j + 1) / kPfStages) & 1, p.err);
          if (!ok) break;
        }
        ok = mbar_wait(&bars->v_full[j % kPfStages], (j / kPfStages) & 1, p.err);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t) {
          if (!live[t] || j >= n_tiles[t]) continue;
          ok = mbar_wait(&bars->p_full[t], j & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, j);
          if (j == n_tiles[t] - 1)
            umma_commit(&bars->o_full[t]);
          else
            issue_s(t, j + 1);
        }
        umma_commit(&bars->v_empty[j % kPfStages]);
        if (has_next) umma_commit(&bars->k_empty[(j + 1) % kPfStages]);
        // K tile 0 is only released here once tile-0/1 S MMAs of j = 0 finished.
        if (j == 0) umma_commit(&bars->k_empty[0]);
      }
      umma_commit(&bars->mma_done);
      mbar_wait(&bars->mma_done, 0, p.err);
    }
  } else {
    // ------------------------------------------- softmax + epilogue, warps 0-7
    const int t = warp >> 2;             // Q tile of this warpgroup
    const int quarter = warp & 3;        // TMEM lane quarter
    const int row = quarter * 32 + lane; // row within the tile
    const int r0 = pair * 2 * kBM + t * kBM;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * kBN;
    const uint32_t tO = tmem + lane_off + 256 + t * kHD;
    const float sl2 = p.scale_log2;
    const int n_my = t ? n_tiles[1] : n_tiles[0];
    float m = -INFINITY, l = 0.f;
    bool ok = t ? live[1] : live[0];
    for (int j = 0; ok && j < n_my; ++j) {
      ok = mbar_wait(&bars->s_full[t], j & 1, p.err);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[kBN];
      tmem_ld32(tS + 0, sr + 0);
      tmem_ld32(tS + 32, sr + 32);
      tmem_ld32(tS + 64, sr + 64);
      tmem_ld32(tS + 96, sr + 96);
      tmem_wait_ld();
      reg_fence<kBN>(sr);
      if (j == n_my - 1) {
        // Diagonal tile: key column c (absolute r0 + c) is visible iff c <= row.
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c > row) sr[c] = __float_as_uint(-INFINITY);
      }
      float mx = __uint_as_float(sr[0]);
#pragma unroll
      for (int c = 1; c < kBN; ++c) mx = fmaxf(mx, __uint_as_float(sr[c]));
      const float m_tile = mx * sl2;
      const float m_new = fmaxf(m, m_tile);
      // Lazy rescale: only rows whose max grew by more than the threshold move
      // their reference point (and then O_t and l are rescaled by alpha).
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m = m_new;
      } else {
        const bool need = m_new > m + kRescaleThreshold;
        rescale = __any_sync(0xffffffffu, need);
        if (need) {
          alpha = fast_exp2(m - m_new);
          m = m_new;
          l *= alpha;
        }
      }
      const float mref = (m == -INFINITY) ? 0.f : m;
      float rs = 0.f;
      // P packed in place: entry c/2 is written after entries c and c+1 were read.
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c]), sl2, -mref));
        const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c + 1]), sl2, -mref));
        rs += p0 + p1;
        sr[c >> 1] = pack_half2(p0, p1);
      }
      l += rs;
      tmem_st32(tS + 0, sr);
      tmem_st32(tS + 32, sr + 32);
      if (rescale) {
        // PV_t(j-1) is complete: s_full for step j was committed after it.
#pragma unroll
        for (int cc = 0; cc < kHD; cc += 32) {
          uint32_t ov[32];
          tmem_ld32(tO + cc, ov);
          tmem_wait_ld();
          reg_fence<32>(ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(tO + cc, ov);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[t]);
    }
    // ------------------------------------------------------------- epilogue
    if (ok) ok = mbar_wait(&bars->o_full[t], 0, p.err);
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint8_t* so = sQ + t * kTileBytes;  // Q tile is dead once O is complete
#pragma unroll
      for (int cc = 0; cc < kHD; cc += 32) {
        uint32_t ov[32];
        tmem_ld32(tO + cc, ov);
        tmem_wait_ld();
        reg_fence<32>(ov);
        uint32_t hv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          hv[e] = pack_half2(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv);
        const int half = cc >> 6;
        const uint32_t base = smem_u32(so + half * kHalfBytes) + row * 128;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int chunk = ((cc & 63) >> 3) + q4;
          const uint32_t addr = base + ((chunk ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                       "r"(hv[4 * q4]), "r"(hv[4 * q4 + 1]), "r"(hv[4 * q4 + 2]),
                       "r"(hv[4 * q4 + 3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1 + t, 128);
      if (quarter == 0 && lane == 0) {
        tma_store_4d(&tm_o, so, 0, r0, h, b);
        tma_store_4d(&tm_o, so + kHalfBytes, 64, r0, h, b);
        tma_store_commit();
        tma_store_wait_all();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// 4-D tensor map over a [B, H, S, 128] fp16 tensor with element strides st[4]
// (b, h, s, d). Box: 64 columns x 128 rows, 128B swizzle.
static int make_bhsd_map(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t S,
                         const int64_t* st, const char* what) {
  if (st[3] != 1) return fail(FI_ERR_ALIGNMENT, "%s: innermost stride must be 1", what);
  uint64_t dims[4] = {(uint64_t)kHD, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t sb[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  // A size-1 dimension is never stepped over; give it any legal stride.
  uint64_t prev = (uint64_t)kHD * 2;
  for (int i = 0; i < 3; ++i) {
    if (dims[i + 1] == 1) sb[i] = (prev + 15) / 16 * 16;
    prev = sb[i] * dims[i + 1];
  }
  const uint32_t box[4] = {64, (uint32_t)kBM, 1, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims, sb, box,
                      CU_TENSOR_MAP_SWIZZLE_128B, what);
}

}  // namespace fi

extern "C" int fi_prefill_fwd(const void* q, const void* k, const void* v, void* o,
                              int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                              int64_t seq_len, int64_t head_dim, const int64_t* q_strides,
                              const int64_t* k_strides, const int64_t* v_strides,
                              const int64_t* o_strides, float sm_scale, int32_t* error_flag,
                              void* stream) {
  using namespace fi;
  clear_error();
  if (batch < 0 || seq_len < 0 || num_q_heads <= 0 || num_kv_heads <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_prefill_fwd: bad sizes");
  if (head_dim != kHD)
    return fail(FI_ERR_UNSUPPORTED, "fi_prefill_fwd: head_dim %lld != 128", (long long)head_dim);
  if (num_q_heads % num_kv_heads != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_prefill_fwd: num_q_heads %% num_kv_heads != 0");
  if (batch == 0 || seq_len == 0) return FI_OK;
  if (!q || !k || !v || !o || !q_strides || !k_strides || !v_strides || !o_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_prefill_fwd: null pointer argument");
  if (seq_len > (1 << 30) || batch > 65535 || num_q_heads > 65535)
    return fail(FI_ERR_UNSUPPORTED, "fi_prefill_fwd: sizes too large");
  CUtensorMap tq, tk, tv, to;
  int r = make_bhsd_map(&tq, q, batch, num_q_heads, seq_len, q_strides, "fi_prefill_fwd q");
  if (r != FI_OK) return r;
  r = make_bhsd_map(&tk, k, batch, num_kv_heads, seq_len, k_strides, "fi_prefill_fwd k");
  if (r != FI_OK) return r;
  r = make_bhsd_map(&tv, v, batch, num_kv_heads, seq_len, v_strides, "fi_prefill_fwd v");
  if (r != FI_OK) return r;
  r = make_bhsd_map(&to, o, batch, num_q_heads, seq_len, o_strides, "fi_prefill_fwd o");
  if (r != FI_OK) return r;

  PrefillParams p;
  p.batch = (int)batch;
  p.hq = (int)num_q_heads;
  p.hk = (int)num_kv_heads;
  p.group = (int)(num_q_heads / num_kv_heads);
  p.seq_len = (int)seq_len;
  p.npairs = (int)((seq_len + 2 * kBM - 1) / (2 * kBM));
  p.scale_log2 = (float)((double)sm_scale * 1.4426950408889634);
  p.err = error_flag;
  const int64_t units = (int64_t)p.npairs * batch * num_q_heads;
  if (units > 0x7fffffff) return fail(FI_ERR_UNSUPPORTED, "fi_prefill_fwd: grid too large");

  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_fwd_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "fi_prefill_fwd: cudaFuncSetAttribute");
    attr_done[dev] = true;
  }
  prefill_fwd_kernel<<<(unsigned)units, kPfThreads, kPfSmemBytes, static_cast<cudaStream_t>(stream)>>>(
      tq, tk, tv, to, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fi_prefill_fwd: launch");
  return FI_OK;
}
