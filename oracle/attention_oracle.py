"""CPU oracle for the Fast_Infer attention hot path (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy with fp32 arithmetic, the three pieces of the
reference's attention path:

* causal FlashAttention-v2 prefill   (reference kernels/attention.py:8-113)
* PagedAttention decode               (reference kernels/attention.py:116-233)
* paged KV-cache block allocation and slot writes
                                      (reference kv_cache.py:12-113, model.py:162-201)

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The CUDA library under ``fast_infer_b200/`` never calls into this file.

Pinning: the functions here are checked against golden vectors produced by
running the reference's own Triton kernels under ``TRITON_INTERPRET=1`` and the
reference's own ``KVCache`` / ``LlamaForCausalLM._store_kv_*`` methods
(``tests/golden/make_golden.py`` generates them; ``tests/test_oracle_golden.py``
checks them).

Inputs are numpy arrays; fp16 inputs are upcast to fp32 exactly as the reference
does before its dot products (kernels/attention.py:45,53,146,165,181).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

BLOCK_SIZE_DEFAULT = 64


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


# ---------------------------------------------------------------------------
# Seeded inputs (shared by the golden generator, the tests and the bench).
# ---------------------------------------------------------------------------

def randn_f16(rng: np.random.Generator, shape) -> np.ndarray:
    """N(0,1) samples rounded to fp16 (the distribution every config names)."""
    return rng.standard_normal(size=shape, dtype=np.float32).astype(np.float16)


# ---------------------------------------------------------------------------
# Prefill: causal FlashAttention-v2, blockwise like the reference kernel.
# ---------------------------------------------------------------------------

def flash_attention_blockwise(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                              sm_scale: float | None = None) -> np.ndarray:
    """Blockwise causal FA-v2 forward, following reference kernels/attention.py:8-113.

    q: [B, Hq, S, D] fp16; k, v: [B, Hk, S, D] fp16 with Hq % Hk == 0. When Hk < Hq
    the K/V head for query head h is h // (Hq // Hk), which is what the reference
    caller's ``repeat_interleave`` (model.py:110-111) produces.

    Block sizes follow the launcher (attention.py:95-96): BLOCK_M = BLOCK_N =
    max(16, min(32, next_pow2(S))). Per Q tile: m=-inf, l=0, acc=0 (:39-41); KV
    loop to the causal bound start_m+BLOCK_M (:47); scores q.k^T*scale (:55);
    causal and bounds masks to -inf (:58-59); online softmax with exp (:61-66);
    acc += p.v (:70); result acc/l cast to fp16 (:74).
    """
    B, Hq, S, D = q.shape
    Hk = k.shape[1]
    assert Hq % Hk == 0
    G = Hq // Hk
    if sm_scale is None:
        sm_scale = D ** -0.5
    bm = bn = max(16, min(32, _next_pow2(S)))
    out = np.empty((B, Hq, S, D), dtype=np.float16)
    scale = np.float32(sm_scale)
    for b in range(B):
        for h in range(Hq):
            qh = q[b, h].astype(np.float32)
            kh = k[b, h // G].astype(np.float32)
            vh = v[b, h // G].astype(np.float32)
            for sm in range(0, S, bm):
                m_offs = np.arange(sm, sm + bm)
                m_mask = m_offs < S
                qt = np.zeros((bm, D), np.float32)
                qt[m_mask] = qh[m_offs[m_mask]]
                m_i = np.full(bm, -np.inf, np.float32)
                l_i = np.zeros(bm, np.float32)
                acc = np.zeros((bm, D), np.float32)
                for sn in range(0, sm + bm, bn):
                    n_offs = np.arange(sn, sn + bn)
                    n_mask = n_offs < S
                    kt = np.zeros((bn, D), np.float32)
                    vt = np.zeros((bn, D), np.float32)
                    kt[n_mask] = kh[n_offs[n_mask]]
                    vt[n_mask] = vh[n_offs[n_mask]]
                    qk = (qt @ kt.T) * scale
                    ok = (m_offs[:, None] >= n_offs[None, :]) & m_mask[:, None] & n_mask[None, :]
                    qk = np.where(ok, qk, np.float32(-np.inf))
                    with np.errstate(invalid="ignore"):
                        m_new = np.maximum(m_i, qk.max(axis=1))
                        alpha = np.exp(m_i - m_new)
                        p = np.exp(qk - m_new[:, None])
                    l_i = l_i * alpha + p.sum(axis=1)
                    acc = acc * alpha[:, None] + p @ vt
                    m_i = m_new
                with np.errstate(invalid="ignore", divide="ignore"):
                    res = (acc / l_i[:, None]).astype(np.float16)
                out[b, h, m_offs[m_mask]] = res[m_mask]
    return out


def attention_fp32(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = True,
                   sm_scale: float | None = None) -> np.ndarray:
    """Dense fp32 softmax attention (the 'fp32 PyTorch attention' comparison point).

    q: [B, Hq, Sq, D]; k, v: [B, Hk, Sk, D]; GQA head h -> h // (Hq // Hk).
    With causal=True query i attends to keys 0..i (Sq == Sk).
    Returns fp32 [B, Hq, Sq, D].
    """
    B, Hq, Sq, D = q.shape
    Hk, Sk = k.shape[1], k.shape[2]
    G = Hq // Hk
    if sm_scale is None:
        sm_scale = D ** -0.5
    out = np.empty((B, Hq, Sq, D), np.float32)
    for b in range(B):
        for kh in range(Hk):
            kk = k[b, kh].astype(np.float32)
            vv = v[b, kh].astype(np.float32)
            qq = q[b, kh * G:(kh + 1) * G].astype(np.float32)  # [G, Sq, D]
            s = np.einsum("gqd,kd->gqk", qq, kk) * np.float32(sm_scale)
            if causal:
                mask = np.tril(np.ones((Sq, Sk), bool))
                s = np.where(mask[None], s, -np.inf)
            s = s - s.max(axis=-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=-1, keepdims=True)
            out[b, kh * G:(kh + 1) * G] = np.einsum("gqk,kd->gqd", p, vv)
    return out


# ---------------------------------------------------------------------------
# Decode: PagedAttention over the [NB, block_size, Hkv, D] pool.
# ---------------------------------------------------------------------------

def paged_attention_blockwise(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                              block_table: np.ndarray, block_size: int,
                              num_tokens: int | None = None,
                              context_lens: np.ndarray | None = None,
                              sm_scale: float | None = None) -> np.ndarray:
    """Paged decode, a literal per-(sequence, head) restatement of reference
    kernels/attention.py:116-233 (bit-identical to the reference run under
    TRITON_INTERPRET=1).

    q: [B, Hq, D] fp16; k_cache, v_cache: [NB, block_size, Hkv, D] fp16;
    block_table: [B, max_blocks] int32 (-1 = unused). One scalar ``num_tokens``
    for the batch as in the reference launcher (:191-233), or per-sequence
    ``context_lens`` (the ragged extension; equal to calling the reference once
    per sequence). num_tokens == 0 returns zeros (:205-206).

    Per (b, q_head): kv_head = q_head // (Hq // Hkv) (:138-139); loop over
    ceil(n/block_size) logical blocks (:155); phys = block_table[b, blk] (:156);
    K rows beyond n load as 0 (:164-165); scores = sum(q*k)*scale, masked to -inf
    beyond n (:168-169); online softmax with exp (:172-176); acc += sum(p*v)
    (:179-182); output acc/l in fp16 (:186).
    """
    B, Hq, D = q.shape
    NB, bs, Hkv, _ = k_cache.shape
    assert bs == block_size
    G = Hq // Hkv
    if sm_scale is None:
        sm_scale = D ** -0.5
    scale = np.float32(sm_scale)
    if context_lens is None:
        if num_tokens == 0:
            return np.zeros_like(q)
        lens = np.full(B, num_tokens, np.int64)
    else:
        lens = np.asarray(context_lens, np.int64)
    out = np.zeros((B, Hq, D), np.float16)
    offs = np.arange(block_size)
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            continue
        for h in range(Hq):
            kvh = h // G
            qh = q[b, h].astype(np.float32)
            m_i = np.float32(-np.inf)
            l_i = np.float32(0.0)
            acc = np.zeros(D, np.float32)
            for blk in range((n + block_size - 1) // block_size):
                phys = int(block_table[b, blk])
                tmask = (blk * block_size + offs) < n
                kt = np.where(tmask[:, None], k_cache[phys, :, kvh].astype(np.float32),
                              np.float32(0.0))
                scores = np.sum(qh[None, :] * kt, axis=1) * scale
                scores = np.where(tmask, scores, np.float32(-np.inf))
                m_new = np.maximum(m_i, np.max(scores))
                alpha = np.exp(m_i - m_new)
                p = np.exp(scores - m_new)
                l_i = l_i * alpha + np.sum(p)
                acc = acc * alpha
                vt = np.where(tmask[:, None], v_cache[phys, :, kvh].astype(np.float32),
                              np.float32(0.0))
                acc = acc + np.sum(p[:, None] * vt, axis=0)
                m_i = m_new
            out[b, h] = (acc / l_i).astype(np.float16)
    return out


def paged_attention_vectorized(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                               block_table: np.ndarray, block_size: int,
                               context_lens: np.ndarray,
                               sm_scale: float | None = None) -> np.ndarray:
    """The same per-block online-softmax algorithm as ``paged_attention_blockwise``
    with all query heads of a sequence processed together (numpy einsum), so it runs
    fast enough to be timed as the CPU baseline. Differs from the literal version
    only in fp32 summation order (at most a few fp16 ulps)."""
    B, Hq, D = q.shape
    NB, bs, Hkv, _ = k_cache.shape
    G = Hq // Hkv
    if sm_scale is None:
        sm_scale = D ** -0.5
    scale = np.float32(sm_scale)
    out = np.zeros((B, Hq, D), np.float16)
    for b in range(B):
        n = int(context_lens[b])
        if n == 0:
            continue
        qb = q[b].astype(np.float32).reshape(Hkv, G, D)
        m_i = np.full((Hkv, G), -np.inf, np.float32)
        l_i = np.zeros((Hkv, G), np.float32)
        acc = np.zeros((Hkv, G, D), np.float32)
        for blk in range((n + block_size - 1) // block_size):
            phys = int(block_table[b, blk])
            nv = min(block_size, n - blk * block_size)
            kt = k_cache[phys, :nv].astype(np.float32)  # [nv, Hkv, D]
            vt = v_cache[phys, :nv].astype(np.float32)
            scores = np.einsum("kgd,tkd->kgt", qb, kt) * scale
            m_new = np.maximum(m_i, scores.max(axis=-1))
            alpha = np.exp(m_i - m_new)
            p = np.exp(scores - m_new[..., None])
            l_i = l_i * alpha + p.sum(axis=-1)
            acc = acc * alpha[..., None] + np.einsum("kgt,tkd->kgd", p, vt)
            m_i = m_new
        out[b] = (acc / l_i[..., None]).reshape(Hq, D).astype(np.float16)
    return out


def paged_attention_fp32(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                         block_table: np.ndarray, context_lens: np.ndarray,
                         sm_scale: float | None = None) -> np.ndarray:
    """Dense fp32 softmax decode attention over the gathered pages (fp32 reference)."""
    B, Hq, D = q.shape
    NB, bs, Hkv, _ = k_cache.shape
    G = Hq // Hkv
    if sm_scale is None:
        sm_scale = D ** -0.5
    out = np.zeros((B, Hq, D), np.float32)
    for b in range(B):
        n = int(context_lens[b])
        if n == 0:
            continue
        nblk = (n + bs - 1) // bs
        phys = np.asarray(block_table[b, :nblk], np.int64)
        kk = k_cache[phys].reshape(nblk * bs, Hkv, D)[:n].astype(np.float32)
        vv = v_cache[phys].reshape(nblk * bs, Hkv, D)[:n].astype(np.float32)
        qb = q[b].astype(np.float32).reshape(Hkv, G, D)
        s = np.einsum("kgd,tkd->kgt", qb, kk) * np.float32(sm_scale)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = np.einsum("kgt,tkd->kgd", p, vv).reshape(Hq, D)
    return out


# ---------------------------------------------------------------------------
# KV cache: block allocation and slot writes.
# ---------------------------------------------------------------------------

@dataclass
class KVCacheOracle:
    """Host restatement of reference kv_cache.py:6-113 (pool, block table, FIFO free list).

    Pool tensors k, v: [L, NB, block_size, H, D] fp16, zero-initialised (:25-28);
    NB = ceil(max_seq_len / block_size) (:21-22); block_table [B, NB] int32 with
    -1 = unallocated (:33-34); free list FIFO ``pop(0)`` (:37,54); ``alloc_block``
    fills the first -1 slot of the row (:56-61).
    """
    num_layers: int
    num_heads: int
    head_dim: int
    max_seq_len: int
    block_size: int = BLOCK_SIZE_DEFAULT
    k: np.ndarray = field(init=False)
    v: np.ndarray = field(init=False)
    block_table: np.ndarray = field(init=False)

    def __post_init__(self):
        self.num_blocks = (self.max_seq_len + self.block_size - 1) // self.block_size
        self.max_blocks_per_seq = self.num_blocks
        shape = (self.num_layers, self.num_blocks, self.block_size, self.num_heads, self.head_dim)
        self.k = np.zeros(shape, np.float16)
        self.v = np.zeros(shape, np.float16)
        self.block_table = np.full((1, self.max_blocks_per_seq), -1, np.int32)
        self.free_blocks = list(range(self.num_blocks))
        self._allocated = 0
        self.num_tokens = 0

    def grow_batch(self, batch_size: int):
        """reference kv_cache.py:41-48."""
        if batch_size <= self.block_table.shape[0]:
            return
        nt = np.full((batch_size, self.max_blocks_per_seq), -1, np.int32)
        nt[: self.block_table.shape[0]] = self.block_table
        self.block_table = nt

    def alloc_block(self, batch_idx: int = 0) -> int:
        """reference kv_cache.py:50-63."""
        if not self.free_blocks:
            raise RuntimeError("KV cache out of memory")
        phys = self.free_blocks.pop(0)
        row = self.block_table[batch_idx]
        empty = np.nonzero(row == -1)[0]
        if len(empty) == 0:
            raise RuntimeError("Sequence block table full")
        logical = int(empty[0])
        row[logical] = phys
        self._allocated += 1
        return logical

    def reset(self):
        """reference kv_cache.py:108-113."""
        self.block_table.fill(-1)
        self.free_blocks = list(range(self.num_blocks))
        self._allocated = 0
        self.num_tokens = 0


def store_kv_prefill(cache: KVCacheOracle, layer_idx: int, k: np.ndarray, v: np.ndarray):
    """reference model.py:162-183. k, v: [B, S, H, D] fp16."""
    B, S = k.shape[0], k.shape[1]
    bs = cache.block_size
    num_needed = (S + bs - 1) // bs
    if layer_idx == 0:
        cache.num_tokens = S
    for b in range(B):
        while int((cache.block_table[b] >= 0).sum()) < num_needed:
            cache.alloc_block(b)
        for blk in range(num_needed):
            start = blk * bs
            end = min(start + bs, S)
            phys = int(cache.block_table[b, blk])
            cache.k[layer_idx, phys, : end - start] = k[b, start:end]
            cache.v[layer_idx, phys, : end - start] = v[b, start:end]


def store_kv_decode(cache: KVCacheOracle, layer_idx: int, k: np.ndarray, v: np.ndarray,
                    token_count: int):
    """reference model.py:185-201. k, v: [B, H, D]; token_count = model._token_count."""
    B = k.shape[0]
    pos = token_count - 1
    bs = cache.block_size
    blk, off = pos // bs, pos % bs
    if layer_idx == 0:
        cache.num_tokens += 1
    for b in range(B):
        while int((cache.block_table[b] >= 0).sum()) <= blk:
            cache.alloc_block(b)
        phys = int(cache.block_table[b, blk])
        cache.k[layer_idx, phys, off] = k[b]
        cache.v[layer_idx, phys, off] = v[b]


def slot_write(k_cache: np.ndarray, v_cache: np.ndarray, k: np.ndarray, v: np.ndarray,
               block_table: np.ndarray, start_pos: np.ndarray, n_new: np.ndarray,
               block_size: int):
    """Generic paged slot write: token t of sequence b goes to logical position
    start_pos[b] + t, i.e. page block_table[b, pos // block_size], row pos % block_size
    (the index math of model.py:176-183 and :188-201). k, v: [B, T, H, D]; only the
    first n_new[b] tokens of row b are written. Mutates k_cache / v_cache in place.
    """
    B = k.shape[0]
    for b in range(B):
        for t in range(int(n_new[b])):
            pos = int(start_pos[b]) + t
            phys = int(block_table[b, pos // block_size])
            k_cache[phys, pos % block_size] = k[b, t]
            v_cache[phys, pos % block_size] = v[b, t]


# ---------------------------------------------------------------------------
# Rotary embedding (the producer of the K written by the slot writes).
# ---------------------------------------------------------------------------

def rope_tables(head_dim: int, max_seq_len: int, theta: float = 500000.0):
    """fp32 cos/sin tables [max_seq_len, head_dim], reference kernels/rope.py:9-16."""
    freq = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                         / np.float32(head_dim)))).astype(np.float32)
    ang = np.outer(np.arange(max_seq_len, dtype=np.float32), freq).astype(np.float32)
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope_fp16(x: np.ndarray, cos16: np.ndarray, sin16: np.ndarray) -> np.ndarray:
    """x * cos + rotate_half(x) * sin with fp16 tensors, every op rounded to fp16
    (reference kernels/rope.py:19-44). x: [B, S, H, D] fp16; cos16/sin16: [S, D] fp16."""
    d = x.shape[-1]
    rot = np.concatenate([-x[..., d // 2:], x[..., : d // 2]], axis=-1)
    c = cos16[None, :, None, :].astype(np.float32)
    s = sin16[None, :, None, :].astype(np.float32)
    a = (x.astype(np.float32) * c).astype(np.float16)
    b = (rot.astype(np.float32) * s).astype(np.float16)
    return (a.astype(np.float32) + b.astype(np.float32)).astype(np.float16)


# ---------------------------------------------------------------------------
# Error metrics used by every parity test (north_star tolerances).
# ---------------------------------------------------------------------------

MAX_ABS_TOL = 2e-3
REL_L2_TOL = 1e-3


def error_stats(out: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """(max-abs, relative-L2) of ``out`` against an fp32 ``ref``."""
    o = np.asarray(out, np.float64)
    r = np.asarray(ref, np.float64)
    max_abs = float(np.max(np.abs(o - r))) if o.size else 0.0
    den = float(np.linalg.norm(r))
    rel = float(np.linalg.norm(o - r) / den) if den > 0 else float(np.linalg.norm(o - r))
    return max_abs, rel


def causal_prefill_flops(batch: int, num_q_heads: int, seq_len: int, head_dim: int) -> float:
    """Algorithmic FLOPs of causal attention: B*Hq*4*D*S(S+1)/2 (QK^T and PV, exact causal)."""
    return float(batch) * num_q_heads * 4.0 * head_dim * seq_len * (seq_len + 1) / 2.0


def decode_bytes(context_lens, num_kv_heads: int, head_dim: int, num_q_heads: int,
                 block_size: int = BLOCK_SIZE_DEFAULT) -> float:
    """Algorithmic HBM bytes of one paged decode pass: each K and V byte once, plus
    Q and O (fp16) and the block-table entries read."""
    lens = np.asarray(context_lens, np.int64)
    kv = float(lens.sum()) * num_kv_heads * head_dim * 2 * 2
    qo = float(len(lens)) * num_q_heads * head_dim * 2 * 2
    bt = float(sum(math.ceil(int(n) / block_size) for n in lens)) * 4
    return kv + qo + bt
