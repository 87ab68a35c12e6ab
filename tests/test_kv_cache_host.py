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
