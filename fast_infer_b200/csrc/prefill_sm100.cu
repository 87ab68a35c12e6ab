// Causal prefill attention (FlashAttention forward) on sm_100a tensor cores.
//
// Replaces the Triton kernel `_flash_attn_fwd` and its launcher `flash_attention`
// (reference kernels/attention.py:8-113). Semantics, per (batch b, query head h,
// query row i):  o[b,h,i] = sum_{j<=i} softmax_j(q[b,h,i].k[b,hk,j] * scale) v[b,hk,j]
// with hk = h / (Hq / Hk); fp16 in, fp32 softmax/accumulation, fp16 out.
//
// B200 design:
// * Persistent kernel, one CTA per SM. A work unit is 256 consecutive query rows of
//   one head as two 128-row tiles (T0, T1) that share every K/V tile fetched; units
//   are numbered longest-first and dealt to CTAs in snake order, so the causal
//   triangle load-balances across the 148 SMs. Barrier phases carry across units,
//   so the next unit's K/V and Q loads and first S MMA overlap this unit's tail.
// * Warp roles (384 threads): warps 0-3 = softmax/epilogue of T0, warps 4-7 = T1,
//   warp 8 = TMA producer, warp 9 = UMMA issuer (one thread), warps 10-11 only give
//   their registers to the softmax warpgroups (setmaxnreg 184 / 136).
// * Tensor memory (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each.
//   S_t = Q_t K^T is a 128x128x128 tcgen05.mma (A, B from 128B-swizzled shared
//   memory, K-major). Softmax threads own one row each (TMEM lane = row), read S
//   with tcgen05.ld, write P as packed fp16 over the first 64 columns of S_t, and
//   the PV product O_t += P V reads P straight from tensor memory (A operand in
//   TMEM, V as an MN-major shared-memory operand).
// * Online softmax in base 2 with a lazy rescale: O_t and l are rescaled only when
//   a row's running max grows by more than 8 (2^8 headroom in fp16 P), which after
//   the first tiles almost never happens. The result is exact either way because
//   numerator and denominator use the same stale max. A share of the exponentials
//   runs as a polynomial on the FMA pipe (exp2_poly_x2) next to MUFU.
// * The MMA issue order S0(j), S1(j), PV0(j), S0(j+1), PV1(j), S1(j+1), ... lets
//   the tensor core work on one tile while the other tile's softmax runs.
// * Epilogue: O_t is read from TMEM (then released for the next unit), divided by
//   l, and each thread stores its fp16 row straight to global memory.
// * Packed variable-length batches (fi_prefill_fwd_varlen) run the same kernel with
//   3-D TMA maps over [tokens, H, D] and per-sequence lengths from cu_seqlens.

#include <math.h>

#include "common.cuh"
#include "host_common.h"

namespace fi {

constexpr int kBM = 128;            // query rows per tile
constexpr int kBN = 128;            // keys per KV tile
constexpr int kHD = 128;            // head dim
constexpr int kHalfBytes = kBM * 128;      // 128 rows x 64 fp16 (one swizzle column)
constexpr int kTileBytes = 2 * kHalfBytes; // 32 KB: a 128 x 128 fp16 tile
// 3 warpgroups: two softmax warpgroups (one per Q tile) and one for the TMA
// producer (warp 8) and UMMA issuer (warp 9); warps 10-11 only hand their
// registers to the softmax warpgroups (setmaxnreg).
constexpr int kPfThreads = 384;
constexpr int kRegsSoftmax = 184;  // 2 x 128 x 184 + 128 x 136 = 384 x 168
constexpr int kRegsOther = 136;
constexpr int kTeardownBar = 15;   // named barrier: all roles done, TMEM can be freed
constexpr int kPfStages = 2;
// Q0, Q1, K[2], V[2] tiles + barriers + tmem slot, plus 1 KB for alignment.
constexpr int kPfSmemBytes = 1024 + (2 + 2 * kPfStages) * kTileBytes + 256;

constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Of every 8 column pairs of S, this many take exp2 on the FMA pipe (polynomial)
// instead of MUFU, so the two units share the softmax's exponentials.
#ifndef FI_PF_EMU_PAIRS
#define FI_PF_EMU_PAIRS 2
#endif
constexpr int kEmuPairsPer8 = FI_PF_EMU_PAIRS;
#ifndef FI_PF_SPIN
#define FI_PF_SPIN 0
#endif
// Critical-path waits (S ready, P ready) busy-poll instead of suspending.
__device__ __forceinline__ bool crit_wait(uint64_t* bar, uint32_t parity, int* err) {
#if FI_PF_SPIN
  return mbar_wait_spin(bar, parity, err);
#else
  return mbar_wait(bar, parity, err);
#endif
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 "version 1" format):
// start address, leading / stride byte offsets (16-byte units), layout type 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: f16 x f16 -> f32 accumulate, M = 128, N = 128,
// operand majorness per argument (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t a_mn_major, uint32_t b_mn_major) {
  return (1u << 4) | (a_mn_major << 15) | (b_mn_major << 16) | ((uint32_t)(kBN >> 3) << 17) |
         ((uint32_t)(kBM >> 4) << 24);
}

struct PrefillParams {
  int batch, hq, hk, group, seq_len, npairs, units;
  const int32_t* cu_seqlens;  // packed (varlen) layout: sequence b = tokens [cu[b], cu[b+1])
  float scale_log2;
  __half* o;
  int64_t os[4];
  int* err;
};

struct PfBarriers {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kPfStages], k_empty[kPfStages];
  uint64_t v_full[kPfStages], v_empty[kPfStages];
  uint64_t s_full[2], p_full[2], o_full[2], o_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
};

// One work unit = 256 consecutive query rows (two 128-row tiles) of one head.
struct PfUnit {
  int b, h, hk, pair;
  int start, len;  // first token of the sequence in the packed layout (0 if not packed), length
  int n[2];  // KV tiles each Q tile needs (0 = tile beyond seq_len)
  int nkv;   // KV tiles the unit streams = max(n[0], n[1])
};

// Units are numbered longest-first (largest pair index first; the heads of one
// KV group adjacent, so they share K/V in L2). Persistent CTA c of G takes unit
// k = r*G + (r even ? c : G-1-c) in round r — a snake order that keeps the
// per-CTA total work within one unit of greedy longest-processing-time.
__device__ __forceinline__ int pf_unit_index(int round, int cta, int G) {
  return round * G + ((round & 1) ? (G - 1 - cta) : cta);
}

__device__ __forceinline__ PfUnit pf_unit(const PrefillParams& p, int k) {
  PfUnit u;
  const int per_pair = p.batch * p.hq;
  u.pair = p.npairs - 1 - k / per_pair;
  const int rem = k % per_pair;
  u.b = rem / p.hq;
  u.h = rem % p.hq;
  u.hk = u.h / p.group;
  if (p.cu_seqlens) {
    u.start = p.cu_seqlens[u.b];
    u.len = p.cu_seqlens[u.b + 1] - u.start;
  } else {
    u.start = 0;
    u.len = p.seq_len;
  }
  for (int t = 0; t < 2; ++t) {
    const int r0 = u.pair * 2 * kBM + t * kBM;
    u.n[t] = r0 < u.len ? r0 / kBN + 1 : 0;
  }
  u.nkv = u.n[1] > 0 ? u.n[1] : u.n[0];
  return u;
}

// Loads one 64-column half of a 128-row tile: (batch, head, row) coordinates for
// [B, H, S, D] tensors, (head, packed token) coordinates for packed [T, H, D] ones.
template <bool kPacked>
__device__ __forceinline__ void tma_tile_half(void* dst, const CUtensorMap* m, uint64_t* bar,
                                              int d0, int row, int h, const PfUnit& u) {
  if (kPacked)
    tma_load_3d(dst, m, bar, d0, h, u.start + row);
  else
    tma_load_4d(dst, m, bar, d0, row, h, u.b);
}

// One pass of the online softmax over a row of S held in registers (one thread =
// one row): p = 2^(s*sl2 - mref) with the scaling on packed FFMA2 and exp2 on MUFU
// (and, for kEmuPairsPer8 of every 8 column pairs, on the FMA pipe); the row sum in 4
// packed FADD2 chains; P packed to fp16 in place (entry c/2 written after entries c
// and c+1 were read).
__device__ __forceinline__ void softmax_pass(uint32_t* sr, float sl2, float mref, float& lsum) {
  const uint64_t sc2 = f32x2(sl2, sl2), nm2 = f32x2(-mref, -mref);
  uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c = 0; c < kBN; c += 2) {
    const uint64_t xp =
        fma_f32x2(f32x2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, nm2);
    float p0, p1;
    if (((c >> 1) & 7) < kEmuPairsPer8) {
      exp2_poly_x2(xp, p0, p1);
    } else {
      float x0, x1;
      f32x2_split(xp, x0, x1);
      p0 = fast_exp2(x0);
      p1 = fast_exp2(x1);
    }
    sum2[(c >> 1) & 3] = add_f32x2(sum2[(c >> 1) & 3], f32x2(p0, p1));
    sr[c >> 1] = pack_half2(p0, p1);
  }
  const uint64_t s01 = add_f32x2(add_f32x2(sum2[0], sum2[1]), add_f32x2(sum2[2], sum2[3]));
  float lo, hi;
  f32x2_split(s01, lo, hi);
  lsum = lo + hi;
}

template <bool kPacked>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* sQ = smem;                                  // 2 tiles
  uint8_t* sK = smem + 2 * kTileBytes;                 // kPfStages tiles
  uint8_t* sV = sK + kPfStages * kTileBytes;           // kPfStages tiles
  PfBarriers* bars = reinterpret_cast<PfBarriers*>(sV + kPfStages * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;

  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->q_full[t], 1);
      mbar_init(&bars->q_empty[t], 1);
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 4);
      mbar_init(&bars->o_full[t], 1);
      mbar_init(&bars->o_empty[t], 4);
    }
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->mma_done, 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp >= 8) {
    // Warpgroup 2 gives registers to the softmax warpgroups, runs the producer
    // and UMMA roles (lane 0 of warps 8 and 9) and leaves through its own exit:
    // every .sync.aligned instruction below is reached by whole, converged warps.
    setmaxnreg_dec<kRegsOther>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------- TMA producer
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      int qc[2] = {0, 0};  // Q loads per tile so far
      int g = 0;           // K/V tiles streamed so far (all units)
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int k = pf_unit_index(r, cta, G);
        if (k >= p.units) break;
        const PfUnit u = pf_unit(p, k);
        if (u.pair == p.npairs - 1 && u.h == 0 && (u.len < 0 || u.len > p.npairs * 2 * kBM))
          set_error(p.err, FI_DEVERR_CONTEXT_LEN);  // cu_seqlens beyond max_seqlen
        if (u.nkv == 0) continue;  // ragged batch: this sequence is shorter
        // K/V tile 0 of the unit goes out before the Q loads: its ring slot frees
        // two steps before the previous unit ends, while the Q buffers only free
        // after that unit's last S MMA.
        auto load_q = [&]() {
          for (int t = 0; t < 2 && ok; ++t) {
            if (u.n[t] == 0) continue;
            if (qc[t] > 0) ok = mbar_wait(&bars->q_empty[t], (qc[t] - 1) & 1, p.err);
            if (!ok) break;
            const int r0 = u.pair * 2 * kBM + t * kBM;
            mbar_arrive_expect_tx(&bars->q_full[t], kTileBytes);
            tma_tile_half<kPacked>(sQ + t * kTileBytes, &tm_q, &bars->q_full[t], 0, r0, u.h, u);
            tma_tile_half<kPacked>(sQ + t * kTileBytes + kHalfBytes, &tm_q, &bars->q_full[t], 64,
                                   r0, u.h, u);
            ++qc[t];
          }
        };
        for (int j = 0; ok && j < u.nkv; ++j, ++g) {
          const int s = g % kPfStages;
          const uint32_t par = ((g / kPfStages) - 1) & 1;
          if (g >= kPfStages && !(ok = mbar_wait(&bars->k_empty[s], par, p.err))) break;
          mbar_arrive_expect_tx(&bars->k_full[s], kTileBytes);
          tma_tile_half<kPacked>(sK + s * kTileBytes, &tm_k, &bars->k_full[s], 0, j * kBN, u.hk, u);
          tma_tile_half<kPacked>(sK + s * kTileBytes + kHalfBytes, &tm_k, &bars->k_full[s], 64,
                                 j * kBN, u.hk, u);
          if (g >= kPfStages && !(ok = mbar_wait(&bars->v_empty[s], par, p.err))) break;
          mbar_arrive_expect_tx(&bars->v_full[s], kTileBytes);
          tma_tile_half<kPacked>(sV + s * kTileBytes, &tm_v, &bars->v_full[s], 0, j * kBN, u.hk, u);
          tma_tile_half<kPacked>(sV + s * kTileBytes + kHalfBytes, &tm_v, &bars->v_full[s], 64,
                                 j * kBN, u.hk, u);
          if (j == 0) load_q();
        }
      }
    } else if (warp == 9 && lane == 0) {
      // ---------------------------------------------------------- UMMA issuer
      constexpr uint32_t idesc_qk = umma_idesc_f16(0, 0);
      constexpr uint32_t idesc_pv = umma_idesc_f16(0, 1);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      int qc[2] = {0, 0};   // units seen per tile (q_full / o_full / o_empty phases)
      int sc[2] = {0, 0};   // S tiles issued per tile (s_full / p_full phases)
      int g = 0;            // K/V tiles consumed so far
      bool ok = true;
      // Descriptors are built once per operand; a K step only advances the start
      // address field (16-byte units, no carry: shared addresses are < 2^18).
      auto issue_s = [&](int t, int kstage) {
        const uint64_t da = umma_desc_sw128(q_addr + t * kTileBytes, 16, 1024);
        const uint64_t db = umma_desc_sw128(k_addr + kstage * kTileBytes, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
          umma_ss(tmem + t * kBN, da + off, db + off, idesc_qk, kk > 0);
        }
        umma_commit(&bars->s_full[t]);
      };
      auto issue_pv = [&](int t, int vstage, bool first) {
        const uint64_t db = umma_desc_sw128(v_addr + vstage * kTileBytes, kHalfBytes, 1024);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          umma_ts(tmem + 256 + t * kHD, tmem + t * kBN + kk * 8, db + (uint32_t)(kk * 16 * 128 / 16),
                  idesc_pv, (!first || kk > 0) ? 1u : 0u);
        }
      };
      for (int r = 0; ok; ++r) {
        const int k = pf_unit_index(r, cta, G);
        if (k >= p.units) break;
        const PfUnit u = pf_unit(p, k);
        if (u.nkv == 0) continue;
        // First K tile of the unit, then S_t(0) for each live tile.
        ok = mbar_wait(&bars->k_full[g % kPfStages], (g / kPfStages) & 1, p.err);
        for (int t = 0; t < 2 && ok; ++t) {
          if (u.n[t] == 0) continue;
          ok = mbar_wait(&bars->q_full[t], qc[t] & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          issue_s(t, g % kPfStages);
          ++sc[t];
          if (u.n[t] == 1) umma_commit(&bars->q_empty[t]);
        }
        for (int j = 0; ok && j < u.nkv; ++j, ++g) {
          const bool has_next = j + 1 < u.nkv;
          if (has_next) {
            ok = mbar_wait(&bars->k_full[(g + 1) % kPfStages], ((g + 1) / kPfStages) & 1, p.err);
            if (!ok) break;
          }
          ok = mbar_wait(&bars->v_full[g % kPfStages], (g / kPfStages) & 1, p.err);
          if (!ok) break;
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= u.n[t]) continue;
            ok = crit_wait(&bars->p_full[t], (sc[t] - 1) & 1, p.err);
            // PV_t(0) overwrites O_t: the previous unit's epilogue must have read it.
            if (ok && j == 0 && qc[t] > 0)
              ok = mbar_wait(&bars->o_empty[t], (qc[t] - 1) & 1, p.err);
            if (!ok) break;
            tc_fence_after();
            issue_pv(t, g % kPfStages, j == 0);
            if (j == u.n[t] - 1) {
              umma_commit(&bars->o_full[t]);
            } else {
              issue_s(t, (g + 1) % kPfStages);
              ++sc[t];
              if (j + 1 == u.n[t] - 1) umma_commit(&bars->q_empty[t]);
            }
          }
          umma_commit(&bars->v_empty[g % kPfStages]);
          // Free each K stage as soon as the S MMAs reading it complete: K tile g+1
          // was read by the S(j+1) issued above, the unit's first K tile by S(0).
          if (j == 0) umma_commit(&bars->k_empty[g % kPfStages]);
          if (has_next) umma_commit(&bars->k_empty[(g + 1) % kPfStages]);
        }
        for (int t = 0; t < 2; ++t)
          if (u.n[t] > 0) ++qc[t];
      }
      umma_commit(&bars->mma_done);
      mbar_wait(&bars->mma_done, 0, p.err);
    }
    __syncwarp();
    named_bar_arrive(kTeardownBar, kPfThreads);
    return;
  }

  // ------------------------------------------- softmax + epilogue, warps 0-7
  setmaxnreg_inc<kRegsSoftmax>();
  {
    const int t = warp >> 2;             // Q tile of this warpgroup
    const int quarter = warp & 3;        // TMEM lane quarter
    const int row = quarter * 32 + lane; // row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * kBN;
    const uint32_t tO = tmem + lane_off + 256 + t * kHD;
    const float sl2 = p.scale_log2;
    int sc = 0;  // S tiles consumed (s_full / p_full phases)
    int uc = 0;  // units finished (o_full / o_empty phases)
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int k = pf_unit_index(r, cta, G);
      if (k >= p.units) break;
      const PfUnit u = pf_unit(p, k);
      const int n_my = u.n[t];
      if (n_my == 0) continue;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; ok && j < n_my; ++j, ++sc) {
        ok = __all_sync(0xffffffffu, crit_wait(&bars->s_full[t], sc & 1, p.err));
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
        // Lazy rescale: only rows whose max grew by more than the threshold move
        // their reference point (and then O_t and l are rescaled by alpha).
        bool rescale = false;
        float alpha = 1.f, lt;
        // Row max as 8 independent chains of 3-input max (short dependency chains).
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a = __uint_as_float(sr[i]);
#pragma unroll
          for (int kk = 1; kk < 15; kk += 2)
            a = fmax3f(a, __uint_as_float(sr[i + 8 * kk]), __uint_as_float(sr[i + 8 * (kk + 1)]));
          mx8[i] = fmaxf(a, __uint_as_float(sr[i + 120]));
        }
        const float mx = fmaxf(fmax3f(mx8[0], mx8[1], mx8[2]),
                               fmax3f(fmax3f(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7]));
        const float m_new = fmaxf(m, mx * sl2);
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
        softmax_pass(sr, sl2, (m == -INFINITY) ? 0.f : m, lt);
        l += lt;
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
      // ----------------------------------------------------------- epilogue
      // O_t -> registers (then O_t is released for the next unit's first PV),
      // normalise, and store fp16 rows straight to global memory.
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_full[t], uc & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      uint32_t ov[kHD];
      tmem_ld32(tO + 0, ov + 0);
      tmem_ld32(tO + 32, ov + 32);
      tmem_ld32(tO + 64, ov + 64);
      tmem_ld32(tO + 96, ov + 96);
      tmem_wait_ld();
      reg_fence<kHD>(ov);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->o_empty[t]);
      ++uc;
      const int grow = u.pair * 2 * kBM + t * kBM + row;
      if (grow < u.len) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __half* orow = kPacked ? p.o + (int64_t)(u.start + grow) * p.os[0] + u.h * p.os[1]
                               : p.o + u.b * p.os[0] + u.h * p.os[1] + (int64_t)grow * p.os[2];
#pragma unroll
        for (int c8 = 0; c8 < kHD; c8 += 8) {
          uint4 pk;
          pk.x = pack_half2(__uint_as_float(ov[c8 + 0]) * inv, __uint_as_float(ov[c8 + 1]) * inv);
          pk.y = pack_half2(__uint_as_float(ov[c8 + 2]) * inv, __uint_as_float(ov[c8 + 3]) * inv);
          pk.z = pack_half2(__uint_as_float(ov[c8 + 4]) * inv, __uint_as_float(ov[c8 + 5]) * inv);
          pk.w = pack_half2(__uint_as_float(ov[c8 + 6]) * inv, __uint_as_float(ov[c8 + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c8) = pk;
        }
      }
    }
  }

  tc_fence_before();
  named_bar_sync(kTeardownBar, kPfThreads);
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

// 3-D tensor map over a packed [T, H, 128] fp16 tensor with element strides st[3]
// (token, head, d). Box: 64 columns x 1 head x 128 tokens, 128B swizzle.
static int make_thd_map(CUtensorMap* m, const void* base, int64_t T, int64_t H,
                        const int64_t* st, const char* what) {
  if (st[2] != 1) return fail(FI_ERR_ALIGNMENT, "%s: innermost stride must be 1", what);
  uint64_t dims[3] = {(uint64_t)kHD, (uint64_t)H, (uint64_t)T};
  uint64_t sb[2] = {(uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  if (H == 1) sb[0] = (uint64_t)kHD * 2;
  const uint32_t box[3] = {64, 1, (uint32_t)kBM};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, sb, box,
                      CU_TENSOR_MAP_SWIZZLE_128B, what);
}

static bool o_layout_ok(const void* o, const int64_t* os, int n) {
  if (os[n - 1] != 1 || (reinterpret_cast<uintptr_t>(o) & 15) != 0) return false;
  for (int i = 0; i + 1 < n; ++i)
    if (os[i] % 8 != 0) return false;
  return true;
}

template <bool kPacked>
static int launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          PrefillParams& p, int64_t batch, int64_t num_q_heads, void* stream) {
  const int64_t units = (int64_t)p.npairs * batch * num_q_heads;
  if (units > 0x7fffffff) return fail(FI_ERR_UNSUPPORTED, "fi_prefill_fwd: too many work units");
  p.units = (int)units;
  const int grid = (int)(units < sm_count() ? units : sm_count());
  static DeviceOnce attr_once;
  {
    const cudaError_t e = attr_once.run([] {
      return cudaFuncSetAttribute(prefill_fwd_kernel<kPacked>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmemBytes);
    });
    if (e != cudaSuccess) return cuda_fail(e, "fi_prefill_fwd: cudaFuncSetAttribute");
  }
  prefill_fwd_kernel<kPacked><<<(unsigned)grid, kPfThreads, kPfSmemBytes,
                                static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fi_prefill_fwd: launch");
  return FI_OK;
}

static void fill_common(PrefillParams& p, int64_t batch, int64_t hq, int64_t hk, int64_t max_len,
                        float sm_scale, void* o, const int64_t* os, int nos, int32_t* err) {
  p.batch = (int)batch;
  p.hq = (int)hq;
  p.hk = (int)hk;
  p.group = (int)(hq / hk);
  p.seq_len = (int)max_len;
  p.npairs = (int)((max_len + 2 * kBM - 1) / (2 * kBM));
  p.scale_log2 = (float)((double)sm_scale * 1.4426950408889634);
  p.err = err;
  p.o = static_cast<__half*>(o);
  for (int i = 0; i < 4; ++i) p.os[i] = i < nos ? os[i] : 0;
  p.cu_seqlens = nullptr;
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
  CUtensorMap tq, tk, tv;
  int r = make_bhsd_map(&tq, q, batch, num_q_heads, seq_len, q_strides, "fi_prefill_fwd q");
  if (r != FI_OK) return r;
  r = make_bhsd_map(&tk, k, batch, num_kv_heads, seq_len, k_strides, "fi_prefill_fwd k");
  if (r != FI_OK) return r;
  r = make_bhsd_map(&tv, v, batch, num_kv_heads, seq_len, v_strides, "fi_prefill_fwd v");
  if (r != FI_OK) return r;
  if (!o_layout_ok(o, o_strides, 4))
    return fail(FI_ERR_ALIGNMENT,
                "fi_prefill_fwd o: needs a 16-byte aligned base, unit innermost stride and "
                "other strides multiple of 8");
  PrefillParams p;
  fill_common(p, batch, num_q_heads, num_kv_heads, seq_len, sm_scale, o, o_strides, 4, error_flag);
  return launch_prefill<false>(tq, tk, tv, p, batch, num_q_heads, stream);
}

extern "C" int fi_prefill_fwd_varlen(const void* q, const void* k, const void* v, void* o,
                                     const int32_t* cu_seqlens, int64_t batch,
                                     int64_t num_q_heads, int64_t num_kv_heads,
                                     int64_t max_seqlen, int64_t total_tokens, int64_t head_dim,
                                     const int64_t* q_strides, const int64_t* k_strides,
                                     const int64_t* v_strides, const int64_t* o_strides,
                                     float sm_scale, int32_t* error_flag, void* stream) {
  using namespace fi;
  clear_error();
  if (batch < 0 || max_seqlen < 0 || total_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0)
    return fail(FI_ERR_INVALID_ARG, "fi_prefill_fwd_varlen: bad sizes");
  if (head_dim != kHD)
    return fail(FI_ERR_UNSUPPORTED, "fi_prefill_fwd_varlen: head_dim %lld != 128",
                (long long)head_dim);
  if (num_q_heads % num_kv_heads != 0)
    return fail(FI_ERR_INVALID_ARG, "fi_prefill_fwd_varlen: num_q_heads %% num_kv_heads != 0");
  if (batch == 0 || max_seqlen == 0 || total_tokens == 0) return FI_OK;
  if (!q || !k || !v || !o || !cu_seqlens || !q_strides || !k_strides || !v_strides || !o_strides)
    return fail(FI_ERR_INVALID_ARG, "fi_prefill_fwd_varlen: null pointer argument");
  if (max_seqlen > (1 << 30) || total_tokens > (1ll << 31) || batch > 65535 ||
      num_q_heads > 65535)
    return fail(FI_ERR_UNSUPPORTED, "fi_prefill_fwd_varlen: sizes too large");
  CUtensorMap tq, tk, tv;
  int r = make_thd_map(&tq, q, total_tokens, num_q_heads, q_strides, "fi_prefill_fwd_varlen q");
  if (r != FI_OK) return r;
  r = make_thd_map(&tk, k, total_tokens, num_kv_heads, k_strides, "fi_prefill_fwd_varlen k");
  if (r != FI_OK) return r;
  r = make_thd_map(&tv, v, total_tokens, num_kv_heads, v_strides, "fi_prefill_fwd_varlen v");
  if (r != FI_OK) return r;
  if (!o_layout_ok(o, o_strides, 3))
    return fail(FI_ERR_ALIGNMENT,
                "fi_prefill_fwd_varlen o: needs a 16-byte aligned base, unit innermost stride "
                "and other strides multiple of 8");
  PrefillParams p;
  fill_common(p, batch, num_q_heads, num_kv_heads, max_seqlen, sm_scale, o, o_strides, 3,
              error_flag);
  p.cu_seqlens = cu_seqlens;
  return launch_prefill<true>(tq, tk, tv, p, batch, num_q_heads, stream);
}
