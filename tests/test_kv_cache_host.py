"""Host-side KVCache logic (allocation order, block tables, batch growth) against
the reference's golden block tables — runs on CPU tensors, no kernels."""

from pathlib import Path

import numpy as np
import pytest
import torch

from fast_infer_b200.kv_cache import KVCache
from tests.golden.inputs import KV_WRITE

GOLDEN = Path(__file__).resolve().parent / "golden"


def _replay_allocations(cache, c):
    bs = cache.block_size
    cache._grow_batch(c["batch"])
    need = (c["prefill"] + bs - 1) // bs
    for b in range(c["batch"]):
        cache._ensure_blocks(b, need)
    after_prefill = cache._bt.copy()
    tc = c["prefill"]
    for _ in range(c["decode_steps"]):
        tc += 1
        blk = (tc - 1) // bs
        for b in range(c["batch"]):
            cache._ensure_blocks(b, blk + 1)
    return after_prefill


def test_allocation_order_matches_reference_block_tables():
    c = KV_WRITE
    g = np.load(GOLDEN / "kv_write.npz")
    cache = KVCache(c["layers"], c["heads"], c["head_dim"], c["max_seq_len"], c["block"],
                    torch.device("cpu"))
    after_prefill = _replay_allocations(cache, c)
    assert np.array_equal(after_prefill, g["bt_after_prefill"])
    assert np.array_equal(cache._bt, g["bt_final"])
    assert cache.free_blocks == list(g["free_blocks"])
    cache.sync_block_table()
    assert np.array_equal(cache.block_table.numpy(), g["bt_final"])


def test_alloc_errors_reset_and_grow():
    cache = KVCache(1, 2, 128, 128, 64, torch.device("cpu"))
    assert cache.alloc_block(0) == 0 and cache.alloc_block(0) == 1
    with pytest.raises(RuntimeError, match="out of memory"):
        cache.alloc_block(0)
    cache.reset()
    assert cache.free_blocks == [0, 1] and (cache.block_table == -1).all()
    cache._grow_batch(3)
    assert tuple(cache.block_table.shape) == (3, 2)
    cache2 = KVCache(1, 2, 128, 128, 64, torch.device("cpu"), num_blocks=4)
    cache2.alloc_block(0)
    cache2.alloc_block(0)
    with pytest.raises(RuntimeError, match="table full"):
        cache2.alloc_block(0)
    assert cache2.allocated_tokens() == 128


def test_permute_rope_rows_layout():
    """permute_rope_rows (the fused decode QKV weight layout): within each 128-row head,
    16-row tile c holds dims 8c..8c+7 then 64+8c..64+8c+7, so each tile carries its
    rotary pairs (d, d + 64); whole heads only; a pure row permutation."""
    from fast_infer_b200.kv_cache import permute_rope_rows
    heads, k = 5, 64
    w = torch.arange(heads * 128, dtype=torch.float32)[:, None].repeat(1, k).half()
    p = permute_rope_rows(w)
    src = p[:, 0].float().long()
    for h in range(heads):
        for c in range(8):
            for r in range(8):
                assert src[128 * h + 16 * c + r] == 128 * h + 8 * c + r
                assert src[128 * h + 16 * c + 8 + r] == 128 * h + 64 + 8 * c + r
    assert sorted(src.tolist()) == list(range(heads * 128))
    assert p.is_contiguous() and torch.equal(p[:, 1:], p[:, :1].expand(-1, k - 1))
    with pytest.raises(ValueError):
        permute_rope_rows(w[:100])
    with pytest.raises(ValueError):
        permute_rope_rows(w, head_dim=64)
