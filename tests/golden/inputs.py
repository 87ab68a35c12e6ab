"""Seeded inputs of the golden fixtures (shared by make_golden.py, the tests and smoke()).

numpy's ``default_rng`` makes them bit-identical on every machine, so only the
reference's outputs need to be stored.
"""

from __future__ import annotations

import numpy as np

from oracle.attention_oracle import randn_f16


def c1_inputs():
    """Config 1 inputs (shared with tests): returns dict of numpy arrays."""
    rng = np.random.default_rng(0)
    B, Hq, Hkv, S, D, steps, NB = 1, 24, 8, 128, 128, 16, 64
    return dict(
        q=randn_f16(rng, (B, Hq, S, D)),
        k=randn_f16(rng, (B, Hkv, S, D)),
        v=randn_f16(rng, (B, Hkv, S, D)),
        dq=randn_f16(rng, (steps, B, Hq, D)),
        dk=randn_f16(rng, (steps, B, Hkv, D)),
        dv=randn_f16(rng, (steps, B, Hkv, D)),
        block_table=rng.permutation(NB).astype(np.int32)[None, :],
        num_blocks=np.int64(NB),
    )


def prefill_small_inputs(S: int):
    rng = np.random.default_rng(100 + S)
    B, Hq, Hkv, D = 2, 6, 2, 128
    return (randn_f16(rng, (B, Hq, S, D)), randn_f16(rng, (B, Hkv, S, D)),
            randn_f16(rng, (B, Hkv, S, D)))


PREFILL_SMALL_S = (1, 77, 200)
DECODE_RAGGED_LENS = (1, 63, 64, 65, 300, 0, 129)


def decode_ragged_inputs():
    rng = np.random.default_rng(7)
    Hq, Hkv, D, bs = 24, 8, 128, 64
    lens = np.array(DECODE_RAGGED_LENS, np.int32)
    B = len(lens)
    nblk = [(int(n) + bs - 1) // bs for n in lens]
    NB = sum(nblk) + 3  # a few spare pages that nobody references
    perm = rng.permutation(NB).astype(np.int32)
    max_blocks = max(nblk) + 1
    bt = np.full((B, max_blocks), -1, np.int32)
    p = 0
    for b in range(B):
        bt[b, : nblk[b]] = perm[p: p + nblk[b]]
        p += nblk[b]
    return dict(
        q=randn_f16(rng, (B, Hq, D)),
        k_cache=randn_f16(rng, (NB, bs, Hkv, D)),
        v_cache=randn_f16(rng, (NB, bs, Hkv, D)),
        block_table=bt,
        context_lens=lens,
    )


KV_WRITE = dict(layers=2, heads=2, head_dim=128, max_seq_len=512, block=64,
                batch=2, prefill=100, decode_steps=30)


def kv_write_inputs():
    c = KV_WRITE
    rng = np.random.default_rng(11)
    L, B, S, H, D = c["layers"], c["batch"], c["prefill"], c["heads"], c["head_dim"]
    T = c["decode_steps"]
    return dict(
        pk=randn_f16(rng, (L, B, S, H, D)), pv=randn_f16(rng, (L, B, S, H, D)),
        dk=randn_f16(rng, (T, L, B, H, D)), dv=randn_f16(rng, (T, L, B, H, D)),
    )


ROPE_PREFILL_POS = tuple(range(6))
ROPE_DECODE_POS = 300


def rope_inputs():
    """q/k for the RoPE fixture: a 6-token prefill and one decode token (B2, 24/8 heads)."""
    rng = np.random.default_rng(31)
    return dict(
        q=randn_f16(rng, (2, 6, 24, 128)), k=randn_f16(rng, (2, 6, 8, 128)),
        dq=randn_f16(rng, (2, 1, 24, 128)), dk=randn_f16(rng, (2, 1, 8, 128)),
    )


# INT4 dequant-matmul fixture: (name, N, K, groupsize, M values).
INT4_CASES = (
    ("a", 192, 384, 128, (1, 5, 16, 33)),
    ("b", 100, 256, 128, (3,)),
    ("g64", 64, 256, 64, (2,)),
)


def int4_inputs(name: str):
    """Weights N(0, 0.02) and activations N(0, 1), fp16, for one INT4_CASES entry.

    Case "a" plants an all-zero quantization group (scale clamp) and one outlier.
    """
    case = {c[0]: c for c in INT4_CASES}[name]
    _, n, k, g, ms = case
    rng = np.random.default_rng(41 + n + k)
    w = (rng.standard_normal(size=(n, k), dtype=np.float32) * 0.02).astype(np.float16)
    if name == "a":
        w[0, :g] = 0
        w[1, 3] = np.float16(5.0)
    xs = {m: randn_f16(rng, (m, k)) for m in ms}
    return w, xs, g


# RMSNorm fixture: (rows, hidden) shapes; row 0 of the first case carries large values.
RMS_CASES = ((4, 3072), (7, 128))


def rms_inputs(rows: int, hidden: int):
    rng = np.random.default_rng(71 + rows + hidden)
    x = randn_f16(rng, (rows, hidden))
    if hidden == 3072:
        x[0] = (x[0].astype(np.float32) * 40.0).astype(np.float16)
    w = (1.0 + 0.1 * rng.standard_normal(size=(hidden,), dtype=np.float32)).astype(np.float16)
    return x, w


# Reference model forward (model.py:50-160) with 2 layers of the Llama-3.2-3B shape
# (hidden 3072, 24/8 heads, intermediate 8192) and a small vocabulary: a 62-token
# prompt for 2 sequences, then 4 decode tokens (positions 62..65; the 65th token
# starts a new page). The pool (max_seq_len 512) has 8 pages shared by the batch.
MODEL = dict(layers=2, vocab=512, hidden=3072, intermediate=8192, heads=24, kv_heads=8,
             head_dim=128, batch=2, prompt=62, decode_steps=4, max_seq_len=512)


def model_weights():
    """Seeded fp16 weights (numpy): embedding N(0,1) (tied LM head), norm weights
    1 + 0.1 N(0,1), linear weights [out, in] N(0, 0.02) per layer."""
    c = MODEL
    rng = np.random.default_rng(61)
    H, I, V = c["hidden"], c["intermediate"], c["vocab"]
    kv = c["kv_heads"] * c["head_dim"]

    def lin(n, k):
        return (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16)

    def norm():
        return (1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32)).astype(np.float16)

    embed = randn_f16(rng, (V, H))
    layers = []
    for _ in range(c["layers"]):
        layers.append(dict(input_layernorm=norm(), post_attention_layernorm=norm(),
                           q_proj=lin(H, H), k_proj=lin(kv, H), v_proj=lin(kv, H),
                           o_proj=lin(H, H), gate_proj=lin(I, H), up_proj=lin(I, H),
                           down_proj=lin(H, I)))
    return dict(embed=embed, layers=layers, norm=norm())


def model_token_ids():
    """Prompt ids [batch, prompt] and the decode steps' ids [steps, batch, 1]."""
    c = MODEL
    rng = np.random.default_rng(62)
    prompt = rng.integers(0, c["vocab"], size=(c["batch"], c["prompt"])).astype(np.int64)
    steps = rng.integers(0, c["vocab"], size=(c["decode_steps"], c["batch"], 1)).astype(np.int64)
    return prompt, steps
