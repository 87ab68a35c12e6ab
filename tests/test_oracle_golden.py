"""The CPU oracle reproduces the reference's own outputs (golden vectors made by
running the reference Triton kernels under TRITON_INTERPRET=1 and its KV-cache
methods; see tests/golden/make_golden.py)."""

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle.attention_oracle import (MAX_ABS_TOL, REL_L2_TOL, KVCacheOracle, attention_fp32,
                                     error_stats, flash_attention_blockwise,
                                     paged_attention_blockwise, paged_attention_fp32,
                                     paged_attention_vectorized, slot_write, store_kv_decode,
                                     store_kv_prefill)
from tests.golden.inputs import (KV_WRITE, PREFILL_SMALL_S, c1_inputs, decode_ragged_inputs,
                                 kv_write_inputs, prefill_small_inputs)

GOLDEN = Path(__file__).resolve().parent / "golden"


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_c1_prefill_bit_identical_to_reference():
    c1 = c1_inputs()
    g = np.load(GOLDEN / "c1.npz")
    out = flash_attention_blockwise(c1["q"], c1["k"], c1["v"])
    assert np.array_equal(out, g["o_prefill"])


def test_c1_reference_within_north_star_tolerance_of_fp32():
    c1 = c1_inputs()
    g = np.load(GOLDEN / "c1.npz")
    ref32 = attention_fp32(c1["q"], c1["k"], c1["v"])
    max_abs, rel = error_stats(g["o_prefill"], ref32)
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL


def _c1_pool():
    c1 = c1_inputs()
    NB = int(c1["num_blocks"])
    kc = np.zeros((NB, 64, 8, 128), np.float16)
    vc = np.zeros_like(kc)
    bt = c1["block_table"]
    k = c1["k"][0].transpose(1, 0, 2)[None]  # [1, S, H, D]
    v = c1["v"][0].transpose(1, 0, 2)[None]
    slot_write(kc, vc, k, v, bt, np.array([0]), np.array([128]), 64)
    return c1, kc, vc, bt


def test_c1_decode_steps_bit_identical_to_reference():
    c1, kc, vc, bt = _c1_pool()
    g = np.load(GOLDEN / "c1.npz")
    for t in range(c1["dq"].shape[0]):
        pos = 128 + t
        slot_write(kc, vc, c1["dk"][t][:, None], c1["dv"][t][:, None], bt,
                   np.array([pos]), np.array([1]), 64)
        out = paged_attention_blockwise(c1["dq"][t], kc, vc, bt, 64, num_tokens=pos + 1)
        assert np.array_equal(out, g["o_decode"][t]), f"step {t}"
    assert _sha(kc) == str(g["k_pool_sha"]) and _sha(vc) == str(g["v_pool_sha"])


@pytest.mark.parametrize("S", PREFILL_SMALL_S)
def test_small_gqa_prefill_bit_identical(S):
    q, k, v = prefill_small_inputs(S)
    g = np.load(GOLDEN / "prefill_small.npz")
    assert np.array_equal(flash_attention_blockwise(q, k, v), g[f"o_S{S}"])


def test_ragged_decode_bit_identical_and_zero_length():
    d = decode_ragged_inputs()
    g = np.load(GOLDEN / "decode_ragged.npz")
    out = paged_attention_blockwise(d["q"], d["k_cache"], d["v_cache"], d["block_table"], 64,
                                    context_lens=d["context_lens"])
    assert np.array_equal(out, g["o"])
    assert not out[d["context_lens"] == 0].any()
    o64 = paged_attention_blockwise(d["q"][2:5], d["k_cache"], d["v_cache"],
                                    d["block_table"][2:5], 64, num_tokens=64)
    assert np.array_equal(o64, g["o_batch64"])


def test_num_tokens_zero_returns_zeros():
    d = decode_ragged_inputs()
    out = paged_attention_blockwise(d["q"], d["k_cache"], d["v_cache"], d["block_table"], 64,
                                    num_tokens=0)
    assert out.shape == d["q"].shape and not out.any()


def test_vectorized_and_fp32_decode_agree_with_reference():
    d = decode_ragged_inputs()
    g = np.load(GOLDEN / "decode_ragged.npz")
    vec = paged_attention_vectorized(d["q"], d["k_cache"], d["v_cache"], d["block_table"], 64,
                                     d["context_lens"])
    f32 = paged_attention_fp32(d["q"], d["k_cache"], d["v_cache"], d["block_table"],
                               d["context_lens"])
    for out in (vec, g["o"]):
        max_abs, rel = error_stats(out, f32)
        assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL


def test_kv_cache_allocation_and_slot_writes_match_reference():
    c = KV_WRITE
    w = kv_write_inputs()
    g = np.load(GOLDEN / "kv_write.npz")
    cache = KVCacheOracle(c["layers"], c["heads"], c["head_dim"], c["max_seq_len"], c["block"])
    cache.grow_batch(c["batch"])
    for layer in range(c["layers"]):
        store_kv_prefill(cache, layer, w["pk"][layer], w["pv"][layer])
    assert np.array_equal(cache.block_table, g["bt_after_prefill"])
    tc = c["prefill"]
    for t in range(c["decode_steps"]):
        tc += 1
        for layer in range(c["layers"]):
            store_kv_decode(cache, layer, w["dk"][t, layer], w["dv"][t, layer], tc)
    assert np.array_equal(cache.block_table, g["bt_final"])
    assert cache.num_tokens == int(g["num_tokens"])
    assert cache.free_blocks == list(g["free_blocks"])
    assert _sha(cache.k) == str(g["k_sha"]) and _sha(cache.v) == str(g["v_sha"])


def test_kv_cache_out_of_memory_and_reset():
    cache = KVCacheOracle(1, 1, 8, 128, 64)
    cache.alloc_block(0)
    cache.alloc_block(0)
    with pytest.raises(RuntimeError):
        cache.alloc_block(0)
    cache.reset()
    assert cache.free_blocks == [0, 1] and (cache.block_table == -1).all()


def test_rope_oracle_bit_identical_to_reference():
    from oracle.attention_oracle import apply_rope_fp16, rope_tables
    from tests.golden.inputs import ROPE_DECODE_POS, rope_inputs
    g = np.load(GOLDEN / "rope.npz")
    r = rope_inputs()
    assert np.array_equal(apply_rope_fp16(r["q"], g["cos16"], g["sin16"]), g["q_rot"])
    assert np.array_equal(apply_rope_fp16(r["k"], g["cos16"], g["sin16"]), g["k_rot"])
    assert np.array_equal(apply_rope_fp16(r["dq"], g["dcos16"], g["dsin16"]), g["dq_rot"])
    assert np.array_equal(apply_rope_fp16(r["dk"], g["dcos16"], g["dsin16"]), g["dk_rot"])
    cos, _ = rope_tables(128, 4096)
    # fp32 cos of arguments up to ~300 rad: implementations differ by ~1e-5
    assert np.allclose(cos[ROPE_DECODE_POS], g["cos_fp32_row300"], atol=1e-4)


def test_model_call_sequence_bit_identical_to_reference():
    """The reference model's whole forward (tests/golden/model_forward.npz: 2 layers,
    a 62-token prefill of 2 sequences, 4 decode tokens, the last starting a new page),
    replayed call by call through the oracle with the inputs the reference's own calls
    got: every attention output, block table, free list, num_tokens and pool digest of
    the reference's run, bit for bit."""
    from tests.golden.inputs import MODEL
    c = MODEL
    g = np.load(GOLDEN / "model_forward.npz")
    cache = KVCacheOracle(c["layers"], c["kv_heads"], c["head_dim"], c["max_seq_len"], 64)
    cache.grow_batch(c["batch"])
    token_count = 0
    for i in range(1 + c["decode_steps"]):
        token_count = c["prompt"] if i == 0 else token_count + 1
        for layer in range(c["layers"]):
            key = f"f{i}_l{layer}_"
            q, k, v = g[key + "q"], g[key + "k"], g[key + "v"]
            if i == 0:  # model.py:104-117: BHSD views, K/V expanded for the kernel
                G = c["heads"] // c["kv_heads"]
                out = flash_attention_blockwise(
                    q.transpose(0, 2, 1, 3), np.repeat(k.transpose(0, 2, 1, 3), G, axis=1),
                    np.repeat(v.transpose(0, 2, 1, 3), G, axis=1)).transpose(0, 2, 1, 3)
                store_kv_prefill(cache, layer, k, v)
            else:  # model.py:118-131
                store_kv_decode(cache, layer, k, v, token_count)
                assert cache.num_tokens == int(g[key + "num_tokens"])
                out = paged_attention_blockwise(q, cache.k[layer], cache.v[layer],
                                                cache.block_table, 64,
                                                num_tokens=cache.num_tokens)
            assert np.array_equal(out, g[key + "o"]), key
        assert np.array_equal(cache.block_table, g[f"f{i}_block_table"]), i
        assert cache.free_blocks == g[f"f{i}_free_blocks"].tolist(), i
        assert cache.num_tokens == int(g[f"f{i}_num_tokens"]), i
        assert _sha(cache.k) == str(g[f"f{i}_k_sha"]) and _sha(cache.v) == str(g[f"f{i}_v_sha"]), i
