/*
 * fast_infer_b200 — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Drop-in boundary for Fast_Infer's attention path. Every entry point takes raw
 * device pointers, element strides (int64, in elements, one per tensor dimension,
 * outermost first), shapes, a softmax scale and a CUDA stream (cudaStream_t passed
 * as void*). Nothing here allocates or synchronises the stream, and the only state
 * kept between calls is per-device set-up (kernel attributes, SM counts), made once
 * under a lock: calls are asynchronous on `stream`, re-entrant and thread-safe, and
 * every buffer belongs to the caller (the peer-gather set-up calls at the end are
 * the exception: they allocate and map the shared regions once). Each call returns FI_OK or an FI_ERR_* code
 * after validating its
 * arguments on the host; fi_last_error() then gives a one-line message
 * (thread-local).
 *
 * Device-side faults the host cannot see before launch (a block-table entry
 * outside the page pool, a pipeline wait that ran out of time) are OR-ed into the
 * optional `error_flag` word (device int32, caller-zeroed) as FI_DEVERR_* bits.
 * Pages with an invalid block-table entry are skipped, never dereferenced.
 *
 * Supported: fp16 Q/K/V/O, head_dim 128, KV page (block) size 64, GQA with
 * num_q_heads % num_kv_heads == 0 and num_q_heads / num_kv_heads <= 8 for decode.
 */
#ifndef FAST_INFER_B200_H
#define FAST_INFER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FI_OK 0
#define FI_ERR_INVALID_ARG 1 /* null pointer, bad shape, inconsistent sizes */
#define FI_ERR_UNSUPPORTED 2 /* valid input outside what the kernels implement */
#define FI_ERR_ALIGNMENT 3   /* pointer or stride not 16-byte aligned where required */
#define FI_ERR_WORKSPACE 4   /* workspace missing or too small */
#define FI_ERR_CUDA 5        /* a CUDA runtime / driver call failed */

/* ---- device error bits (OR-ed into *error_flag) ------------------------ */
#define FI_DEVERR_TIMEOUT 1    /* an mbarrier wait exceeded its time bound; output undefined */
#define FI_DEVERR_BAD_BLOCK 2  /* block_table entry outside [0, num_blocks) for a live token */
#define FI_DEVERR_CONTEXT_LEN 4 /* a context length beyond max_context_len or the block table;
                                  that sequence was truncated */

/* ---- call flags (the `flags` argument of the decode GEMMs) -------------- */
/* The weight operand is constant: no kernel that may still be running when the call
 * is made writes it. The call's first weight tiles then load while the previous
 * kernel on the stream finishes (programmatic dependent launch), instead of after
 * it. Results are the same bits either way; without the flag the weights are read
 * only after the dependency wait, so they may be the previous kernel's output. */
#define FI_STATIC_WEIGHTS 1

/* Library version (major*10000 + minor*100 + patch). */
int fi_version(void);

/* Message describing the last non-FI_OK return on this thread ("" if none). */
const char* fi_last_error(void);

/*
 * Causal prefill attention (FlashAttention forward), tcgen05 UMMA + TMEM.
 *
 * Replaces: kernels/attention.py:80-113 `flash_attention(q, k, v, sm_scale)` and
 * its Triton kernel `_flash_attn_fwd` (kernels/attention.py:8-77).
 *
 * q, o : [batch, num_q_heads, seq_len, 128] fp16, strides q_strides / o_strides
 *        (4 entries each; innermost stride must be 1, the others multiples of 8).
 * k, v : [batch, num_kv_heads, seq_len, 128] fp16. num_kv_heads may equal
 *        num_q_heads (K/V already expanded, as the reference caller passes them)
 *        or divide it (GQA without expansion: query head h reads K/V head
 *        h / (num_q_heads / num_kv_heads)).
 * o[b,h,i,:] = softmax_j<=i(q[b,h,i,:].k[b,hk,j,:] * sm_scale) . v[b,hk,:,:].
 */
int fi_prefill_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                   int64_t num_q_heads, int64_t num_kv_heads, int64_t seq_len, int64_t head_dim,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                   const int64_t* o_strides, float sm_scale, int32_t* error_flag, void* stream);

/*
 * Causal prefill over a ragged batch packed along the token axis (no counterpart
 * in the reference, whose flash_attention takes one shared length; the per-sequence
 * state it lacks is noted at model.py:59,67-72 and kv_cache.py:39).
 *
 * q, o : [total_tokens, num_q_heads, 128] fp16 (strides: 3 entries, token/head/dim);
 * k, v : [total_tokens, num_kv_heads, 128] fp16; sequence b owns tokens
 *        [cu_seqlens[b], cu_seqlens[b+1]) (device int32 [batch + 1], non-decreasing).
 * max_seqlen bounds every length (longer sequences set FI_DEVERR_CONTEXT_LEN and are
 * only partly computed). Same arithmetic and GQA rule as fi_prefill_fwd.
 */
int fi_prefill_fwd_varlen(const void* q, const void* k, const void* v, void* o,
                          const int32_t* cu_seqlens, int64_t batch, int64_t num_q_heads,
                          int64_t num_kv_heads, int64_t max_seqlen, int64_t total_tokens,
                          int64_t head_dim, const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* v_strides, const int64_t* o_strides, float sm_scale,
                          int32_t* error_flag, void* stream);

/*
 * Bytes of split-KV workspace fi_paged_decode needs for these sizes
 * (pages_per_split = 0 selects the library's automatic split size).
 */
size_t fi_paged_decode_workspace_size(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                      int64_t head_dim, int64_t max_context_len,
                                      int64_t block_size, int64_t pages_per_split);

/*
 * Paged decode attention (one query token per sequence) with GQA and split-KV.
 *
 * Replaces: kernels/attention.py:191-233 `paged_attention(q, k_cache, v_cache,
 * block_table, block_size, num_tokens, sm_scale)` and its Triton kernel
 * `_paged_attention_kernel` (kernels/attention.py:116-188).
 *
 * q, o        : [batch, num_q_heads, 128] fp16 (q_strides / o_strides: 3 entries).
 * k_cache,
 * v_cache     : [num_blocks, block_size=64, num_kv_heads, 128] fp16 page pools
 *               (kc_strides / vc_strides: 4 entries; the layout of one layer of
 *               kv_cache.py:25-28).
 * block_table : [batch, max_blocks_per_seq] int32 (bt_strides: 2 entries), logical
 *               page -> physical page; -1 marks an unused slot (kv_cache.py:33-34).
 * context_lens: optional [batch] int32 device array of per-sequence token counts.
 *               NULL = every sequence has `num_tokens` tokens (the reference's
 *               scalar). `max_context_len` is a host-side upper bound of the
 *               lengths, used only to size the launch (ignored when NULL).
 *               Sequences with 0 tokens produce zeros (kernels/attention.py:205-206).
 * workspace   : caller-owned device buffer of at least
 *               fi_paged_decode_workspace_size(...) bytes (may be NULL when that is 0).
 * pages_per_split: KV pages per split-KV partition; 0 = automatic. Deterministic:
 *               a call repeated on the same inputs gives the same bits.
 */
int fi_paged_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
                    const int32_t* block_table, const int32_t* context_lens, int64_t num_tokens,
                    int64_t max_context_len, int64_t batch, int64_t num_q_heads,
                    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                    int64_t block_size, int64_t max_blocks_per_seq, const int64_t* q_strides,
                    const int64_t* kc_strides, const int64_t* vc_strides,
                    const int64_t* o_strides, const int64_t* bt_strides, float sm_scale,
                    int64_t pages_per_split, void* workspace, size_t workspace_bytes,
                    int32_t* error_flag, void* stream);

/*
 * Paged decode that allocates nothing: identical arguments and results to
 * fi_paged_decode minus the workspace, whose split-KV scratch comes from a
 * file-scope static device array of FI_NOALLOC_SCRATCH_BYTES instead.
 *
 * No counterpart in the reference. For callers that cannot allocate device memory
 * themselves: a C/C++ host linking only this library (no caching allocator, and
 * cudaMalloc would synchronise the device on the decode path) or a runtime that
 * forbids allocation after start-up to keep its footprint fixed.
 *
 * Sizes needing more scratch than FI_NOALLOC_SCRATCH_BYTES return FI_ERR_WORKSPACE.
 * Every GPU that loads the library holds the array until exit; all calls on a
 * device share it, so calls that overlap on the GPU race (order them on one
 * stream). The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make it before any stream capture. The address is kept
 * per device and CUDA context: the first call from another context on that device
 * (after cudaDeviceReset, or a non-primary context of the caller's) looks it up
 * again, so it too belongs before any capture.
 */
#define FI_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
int fi_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o,
                            const int32_t* block_table, const int32_t* context_lens,
                            int64_t num_tokens, int64_t max_context_len, int64_t batch,
                            int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                            int64_t num_blocks, int64_t block_size, int64_t max_blocks_per_seq,
                            const int64_t* q_strides, const int64_t* kc_strides,
                            const int64_t* vc_strides, const int64_t* o_strides,
                            const int64_t* bt_strides, float sm_scale, int64_t pages_per_split,
                            int32_t* error_flag, void* stream);

/*
 * KV-cache slot write: copy new tokens' K and V rows into their pages.
 *
 * Replaces: the slot writes of model.py:162-183 (`_store_kv_prefill`), model.py:185-201
 * (`_store_kv_decode`) and kv_cache.py:69-102 (`KVCache.store`, `store_batch`), which the
 * reference performs as one torch copy (plus a host sync) per (layer, sequence, block).
 *
 * k, v     : [batch, num_new, num_kv_heads, head_dim] fp16 (k_strides / v_strides:
 *            4 entries, innermost 1).
 * Token t of sequence b is written to logical position p = start_pos[b] + t (or
 * start_pos_scalar + t when start_pos is NULL), i.e. to page
 * block_table[b, p / block_size], row p % block_size, for t < n_new[b] (or all
 * num_new tokens when n_new is NULL). Bytes are copied unchanged (bit-exact).
 * Pages must already be allocated; an entry outside [0, num_blocks) sets
 * FI_DEVERR_BAD_BLOCK and that row is skipped.
 */
int fi_kv_write(const void* k, const void* v, void* k_cache, void* v_cache,
                const int32_t* block_table, const int32_t* start_pos, int64_t start_pos_scalar,
                const int32_t* n_new, int64_t batch, int64_t num_new, int64_t num_kv_heads,
                int64_t head_dim, int64_t num_blocks, int64_t block_size,
                int64_t max_blocks_per_seq, const int64_t* k_strides, const int64_t* v_strides,
                const int64_t* kc_strides, const int64_t* vc_strides, const int64_t* bt_strides,
                int32_t* error_flag, void* stream);

/*
 * Fused rotary embedding + KV-cache slot write, from the QKV projection output.
 *
 * Replaces: kernels/rope.py:26-44 `apply_rope(q, k, cos, sin)` as called at
 * model.py:101 (cos/sin rows cast to fp16, model.py:74-75) plus the slot writes of
 * model.py:162-201, in one launch.
 *
 * qkv       : [batch, seq, (nq + 2*nkv) * head_dim] fp16, heads in the order q | k | v
 *             (qkv_strides: 3 entries, innermost 1) — the fused projection output.
 * cos_table,
 * sin_table : fp32 [table_rows, table_stride] rotary tables (kernels/rope.py:9-16);
 *             token t of sequence b uses row start_pos[b] + t (or start_pos_scalar + t).
 * q_out     : [batch, seq, nq, head_dim] fp16 rotated q (q_out_strides: 4 entries).
 * k_out     : optional dense [batch, seq, nkv, head_dim] rotated k (NULL = cache only).
 * Rotated k and unchanged v go to page block_table[b, p / block_size], row
 * p % block_size of k_cache / v_cache (layouts as in fi_kv_write).
 * Every product and sum is rounded to fp16 as PyTorch's fp16 ops do, so results are
 * bit-identical to the reference's apply_rope followed by its copies.
 */
int fi_rope_kv_write(const void* qkv, int64_t batch, int64_t seq, int64_t num_q_heads,
                     int64_t num_kv_heads, int64_t head_dim, const int64_t* qkv_strides,
                     const float* cos_table, const float* sin_table, int64_t table_rows,
                     int64_t table_stride, const int32_t* start_pos, int64_t start_pos_scalar,
                     void* q_out, const int64_t* q_out_strides, void* k_out,
                     const int64_t* k_out_strides, void* k_cache, void* v_cache,
                     const int32_t* block_table, int64_t num_blocks, int64_t block_size,
                     int64_t max_blocks_per_seq, const int64_t* kc_strides,
                     const int64_t* vc_strides, const int64_t* bt_strides, int32_t* error_flag,
                     void* stream);

/*
 * RMSNorm: out[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * weight, fp16 in/out,
 * fp32 arithmetic. x, out: [rows, hidden] with row strides (elements, multiples of 8;
 * unit inner stride); weight: [hidden]. hidden a multiple of 8; 16-byte aligned bases.
 *
 * Replaces: kernels/rms_norm.py:29-43 `rms_norm(x, weight, eps)` (called at
 * model.py:82,141,153), used here by the attention-stack harness.
 */
int fi_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int64_t hidden,
                int64_t x_row_stride, int64_t out_row_stride, float eps, void* stream);

/* ---- INT4 group-wise weights (the projections around attention) ---------- */

/*
 * Weight format of every INT4 entry point (reference loader.py:9-41,
 * `quantize_int4_groupwise`): packed int8 [N, K/2], byte j of row n holds w[n, 2j] in
 * its low nibble and w[n, 2j+1] in its high nibble (two's complement, [-8, 7]);
 * scales fp16 [N, K/groupsize]; weight value fp16(q * scale). K % groupsize == 0.
 */

/*
 * C[M, N] = x[M, K] @ dequant(W)^T, fp16 in / fp16 out, fp32 accumulation, for
 * decode-sized M (1..64; larger M returns FI_ERR_UNSUPPORTED — dequantize with
 * fi_int4_dequant and use a dense GEMM). Uses no workspace; deterministic.
 * error_flag: optional device int32; FI_DEVERR_TIMEOUT if a pipeline wait ran out.
 *
 * Replaces: kernels/matmul.py:14-132 `_fused_int4_matmul` (reached through
 * `int4_matmul(x, (packed, scales), groupsize)`, kernels/matmul.py:217-231, from
 * model.py:91-93,134 and kernels/mlp.py:49,52 in the default memory mode).
 *
 * x       : [M, K] fp16, x_strides {row, 1}; 16-byte aligned base, row stride a
 *           multiple of 8.
 * packed  : [N, K/2] int8, packed_strides {row bytes, 1}; 16-byte aligned base and
 *           row stride.
 * scales  : [N, K/groupsize] fp16, any strides. groupsize a multiple of 32.
 * c       : [M, N] fp16, any strides.
 */
int fi_int4_gemm(const void* x, const void* packed, const void* scales, void* c, int64_t m,
                 int64_t n, int64_t k, int64_t groupsize, const int64_t* x_strides,
                 const int64_t* packed_strides, const int64_t* scales_strides,
                 const int64_t* c_strides, int32_t* error_flag, void* stream);

/*
 * Dequantize INT4 weights to fp16 [N, K] (out_strides {row, 1}; 16-byte aligned base,
 * row stride a multiple of 8), bit-identical to the reference.
 *
 * Replaces: kernels/matmul.py:309-326 `_dequant_storage` and loader.py:157-190
 * `dequantize_int4` (the speed-mode weight preparation, kernels/matmul.py:236-266).
 * packed: 4-byte aligned base and row stride; groupsize a multiple of 8.
 */
int fi_int4_dequant(const void* packed, const void* scales, void* out, int64_t n, int64_t k,
                    int64_t groupsize, const int64_t* packed_strides,
                    const int64_t* scales_strides, const int64_t* out_strides, void* stream);

/*
 * Quantize fp16 weights w [N, K] (w_strides: 2 entries, any) to the INT4 format
 * above, bit-identical to the reference: per group, scale = fp16(max(max|w|,
 * fp16(1e-6)) / 7), q = round-half-even(fp16(w / scale)) clamped to [-8, 7].
 *
 * Replaces: loader.py:9-41 `quantize_int4_groupwise` (run once per linear weight at
 * load time, loader.py:150-154). packed_strides {row bytes, 1}; groupsize even.
 */
int fi_int4_quantize(const void* w, void* packed, void* scales, int64_t n, int64_t k,
                     int64_t groupsize, const int64_t* w_strides, const int64_t* packed_strides,
                     const int64_t* scales_strides, void* stream);

/*
 * Decode-sized fp16 GEMM with optional RMSNorm prologue and residual epilogue:
 *   c[i, :] = residual[i, :] + rmsnorm(x[i, :]) @ w^T   (i < m <= 16)
 * x [m, k], w [n, k] (the reference's linear-weight layout), c / residual [m, n], all
 * fp16 (strides: 2 entries; x and w with unit inner stride, row strides multiples of
 * 8 elements, 16-byte aligned bases); fp32 accumulation, one fp16 rounding at the
 * end. norm_weight [k] (NULL: no norm) applies fi_rms_norm's arithmetic with eps;
 * residual NULL: no add (it may alias c). k a multiple of 64; m > 16 returns
 * FI_ERR_UNSUPPORTED (use a dense GEMM). flags: 0 or FI_STATIC_WEIGHTS.
 *
 * Replaces, at decode batch sizes: kernels/rms_norm.py:29-43 followed by
 * kernels/matmul.py:187-212 `_fp16_matmul` (the QKV projection of model.py:82-93),
 * and `_fp16_matmul` followed by the residual add (the O projection, model.py:134-141).
 */
int fi_small_gemm(const void* x, const void* w, void* c, const void* residual,
                  const void* norm_weight, float eps, int64_t m, int64_t n, int64_t k,
                  const int64_t* x_strides, const int64_t* w_strides, const int64_t* c_strides,
                  const int64_t* residual_strides, int64_t flags, int32_t* error_flag,
                  void* stream);

/*
 * The same with the RMSNorm weight folded into the weights: w_folded[n, j] =
 * fp16(w[n, j] * norm_weight[j]) (prepared once), and
 *   c[i, :] = residual[i, :] + rsqrt(mean(x[i, :]^2) + eps) * (x[i, :] @ w_folded^T).
 * Mathematically rmsnorm(x) @ w^T; the rounding differs from the reference's (the
 * normalised x is not rounded to fp16, the folded weights are), within fp16 noise.
 * x reaches the kernel by TMA with each weight tile instead of being staged and
 * normalised first. Same layouts and limits as fi_small_gemm.
 */
int fi_small_gemm_folded(const void* x, const void* w_folded, void* c, const void* residual,
                         float eps, int64_t m, int64_t n, int64_t k, const int64_t* x_strides,
                         const int64_t* w_strides, const int64_t* c_strides,
                         const int64_t* residual_strides, int64_t flags, int32_t* error_flag,
                         void* stream);

/*
 * Decode-step QKV projection with RMSNorm, RoPE and the KV-cache slot writes in one
 * launch: for each sequence b (< batch <= 16; one token each, row b of x [batch, k])
 *   qkv = rsqrt(mean(x[b]^2) + eps) * (x[b] @ w^T)  rounded to fp16,
 * then RoPE of the q and k heads at position start_pos[b] and the writes, exactly as
 * fi_rope_kv_write does with that qkv: rotated q to q_out [batch, nq, 128] (strides: 3
 * entries), rotated k and raw v to page block_table[b, pos / block_size], row
 * pos % block_size of k_cache / v_cache (layouts as in fi_kv_write).
 * w_rope is the folded weight of fi_small_gemm_folded ([(nq + 2 nkv) * 128, k]) with
 * its rows permuted per head: for head h and c in 0..7, rows 128h + 16c .. +7 hold
 * dims 8c .. 8c+7 and rows 128h + 16c + 8 .. +15 hold dims 64 + 8c .. (so each
 * 16-row tile carries its rotary pairs). head_dim 128; cos/sin fp32 [table_rows,
 * table_stride]. flags: 0 or FI_STATIC_WEIGHTS (for w_rope).
 *
 * Replaces, at decode batch sizes: the RMSNorm + QKV projection (model.py:82-93) and
 * the RoPE + slot writes (kernels/rope.py:26-44, model.py:101,185-201).
 */
int fi_qkv_rope_kv_write(const void* x, const void* w_rope, float eps, int64_t batch, int64_t k,
                         int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                         const int64_t* x_strides, const int64_t* w_strides,
                         const float* cos_table, const float* sin_table, int64_t table_rows,
                         int64_t table_stride, const int32_t* start_pos, void* q_out,
                         const int64_t* q_out_strides, void* k_cache, void* v_cache,
                         const int32_t* block_table, int64_t num_blocks, int64_t block_size,
                         int64_t max_blocks_per_seq, const int64_t* kc_strides,
                         const int64_t* vc_strides, const int64_t* bt_strides, int64_t flags,
                         int32_t* error_flag, void* stream);

/*
 * Head-output all-gather over NVLink peer memory, for a stack sharded by KV head.
 *
 * Replaces: the NCCL all-gather of per-rank attention outputs [rows, heads_r * 128]
 * before the replicated O projection (model.py:123-134 with the heads split over
 * GPUs; the one exchange of the sharded path). Set-up (these allocate and
 * synchronise; call once): every rank calls fi_peer_alloc for a region of
 * fi_peer_gather_bytes(nbuf, max_rows, world * row_bytes) bytes and shares the
 * 64-byte `handle` with the others (e.g. through torch.distributed), which map it
 * with fi_peer_open. bases[p] is rank p's region as mapped on this rank
 * (bases[rank] = this rank's own pointer).
 *
 * fi_peer_gather: writes src [rows, row_bytes] (16-byte aligned rows) into buffer
 * `buffer` of every rank's region at [row, rank * row_bytes], then waits on the device
 * until every rank has delivered the same call (bounded: FI_DEVERR_TIMEOUT after 2 s).
 * On return of the kernel this rank's buffer holds [rows, world * row_bytes] with rank
 * p's block at p. Calls are counted on the device, so a CUDA graph replays correctly;
 * every rank must make the same sequence of calls, and two uses of one buffer need
 * another gather between them, so world > 1 needs nbuf >= 2 (FI_ERR_INVALID_ARG
 * otherwise). world <= 8. A call whose error_flag already holds
 * FI_DEVERR_TIMEOUT does not wait (pass one persistent word to every call so a broken
 * rendezvous costs one time-out).
 */
size_t fi_peer_gather_bytes(int64_t nbuf, int64_t max_rows, int64_t row_total_bytes);
int fi_peer_alloc(size_t bytes, void** ptr, void* handle);
int fi_peer_open(const void* handle, void** ptr);
int fi_peer_close(void* ptr);
int fi_peer_free(void* ptr);
int fi_peer_gather(const void* src, int64_t rows, int64_t row_bytes, int64_t src_row_stride_bytes,
                   void* const* bases, int64_t world, int64_t rank, int64_t buffer, int64_t nbuf,
                   int64_t max_rows, int32_t* error_flag, void* stream);

/*
 * O projection of a stack sharded by KV head, reduced across ranks over NVLink peer
 * memory inside the GEMM (no separate gather, no replicated projection).
 *
 * Replaces, for the decode step of a KV-head-sharded stack, the all-gather of the
 * per-rank head outputs plus the replicated O projection and residual add
 * (model.py:123-135 with the heads split over GPUs): every rank multiplies only its
 * own heads' output by the matching input columns of the projection.
 *
 * c[i, :] = residual[i, :] + sum over ranks p, in rank order, of fp16(x_p[i, :] @ w_p^T)
 *   x_p : [m, k] fp16 on rank p, m <= 16 (x_strides: 2 entries, innermost 1)
 *   w_p : [n, k] fp16 on rank p, the projection's input columns of rank p's heads
 *   c, residual : [m, n] fp16 (may be the same buffer); identical bits on every rank.
 * k a multiple of 64. Set-up as for fi_peer_gather: fi_peer_alloc a region of
 * fi_peer_reduce_bytes(nbuf, world, n) bytes on every rank, fi_peer_open the others'.
 * Each call uses landing buffer `buffer`; consecutive calls must use different
 * buffers (world > 1 needs nbuf >= 2, FI_ERR_INVALID_ARG otherwise). Calls are
 * counted on the device, so a CUDA graph replays correctly; every rank makes the same
 * sequence of calls. A rank waits for the others' partials (bounded: 2 s, then
 * FI_DEVERR_TIMEOUT in error_flag; later calls given a word holding it do not wait).
 * flags: FI_STATIC_WEIGHTS as for fi_small_gemm.
 */
size_t fi_peer_reduce_bytes(int64_t nbuf, int64_t world, int64_t n);
int fi_small_gemm_peer_reduce(const void* x, const void* w, void* c, const void* residual,
                              int64_t m, int64_t n, int64_t k, const int64_t* x_strides,
                              const int64_t* w_strides, const int64_t* c_strides,
                              const int64_t* residual_strides, void* const* bases, int64_t world,
                              int64_t rank, int64_t buffer, int64_t nbuf, int64_t flags,
                              int32_t* error_flag, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FAST_INFER_B200_H */
