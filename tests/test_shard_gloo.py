"""Multi-rank host logic on CPU (gloo, world_size 2): KV-head and sequence
partitioning reproduce the unsharded attention exactly, and the head all-gather
reassembles outputs in head order."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from fast_infer_b200.shard import head_shard, seq_range


def test_head_shard_ranges():
    shards = [head_shard(r, 4, 24, 8) for r in range(4)]
    assert [(s.kv_start, s.kv_end) for s in shards] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert [(s.q_start, s.q_end) for s in shards] == [(0, 6), (6, 12), (12, 18), (18, 24)]
    s8 = head_shard(7, 8, 24, 8)
    assert (s8.kv_start, s8.q_start, s8.q_end) == (7, 21, 24)
    with pytest.raises(ValueError):
        head_shard(0, 3, 24, 8)
    # every query head's KV head is on the same rank
    for r in range(8):
        s = head_shard(r, 8, 24, 8)
        assert all(s.kv_start <= h // 3 < s.kv_end for h in range(s.q_start, s.q_end))


def test_seq_range_covers_batch():
    for world in (1, 2, 3, 8):
        spans = [seq_range(r, world, 13) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 13
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, k, v, result_q):
    import torch.distributed as dist
    from fast_infer_b200.shard import gather_heads, head_shard, shard_heads
    from oracle.attention_oracle import attention_fp32
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = head_shard(rank, world, q.shape[1], k.shape[1])
        ql = shard_heads(torch.from_numpy(q), s, kv=False).numpy()
        kl = shard_heads(torch.from_numpy(k), s, kv=True).numpy()
        vl = shard_heads(torch.from_numpy(v), s, kv=True).numpy()
        ol = attention_fp32(ql, kl, vl)                       # [B, Hq_r, S, D]
        B, Hr, S, D = ol.shape
        flat = torch.from_numpy(ol).permute(0, 2, 1, 3).reshape(B, S, Hr * D)
        full = gather_heads(flat)                             # [B, S, Hq*D]
        if rank == 0:
            result_q.put(full.numpy())
    finally:
        dist.destroy_process_group()


def test_kv_head_partition_allgather_matches_unsharded():
    rng = np.random.default_rng(0)
    B, Hq, Hkv, S, D = 2, 24, 8, 40, 128
    q = rng.standard_normal((B, Hq, S, D), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((B, Hkv, S, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((B, Hkv, S, D), dtype=np.float32).astype(np.float16)
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    full = result_q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle.attention_oracle import attention_fp32
    ref = attention_fp32(q, k, v).transpose(0, 2, 1, 3).reshape(B, S, Hq * D)
    assert np.array_equal(full, ref)


def _peer_nbuf_worker(rank, world, port, result_q):
    import torch.distributed as dist
    from fast_infer_b200.shard import PeerGather
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        try:
            PeerGather(16, 768, nbuf=1, device="cpu")
            result_q.put((rank, "accepted"))
        except ValueError as e:
            result_q.put((rank, str(e)))
    finally:
        dist.destroy_process_group()


def test_peer_gather_rejects_one_buffer_over_two_ranks():
    """Two ranks with one gather buffer: the constructor refuses before it allocates
    or maps anything (a rank one call ahead would overwrite the words a slower rank
    is still reading)."""
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_nbuf_worker, args=(r, 2, port, result_q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = dict(result_q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        assert "nbuf >= 2" in got[r], got[r]


def _token_split_worker(rank, world, port, full, result_q):
    import torch.distributed as dist
    from fast_infer_b200.shard import gather_rows, heads_to_tokens, token_block
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = torch.from_numpy(full)                        # [T, heads * D], every rank
        cols = x.shape[1] // world
        mine = x[:, rank * cols:(rank + 1) * cols]        # this rank's heads, every token
        t0, t1 = token_block(rank, world, x.shape[0])
        rows = heads_to_tokens(mine)                      # every head, this rank's tokens
        back = gather_rows(rows)                          # every head, every token
        result_q.put((rank, torch.equal(rows, x[t0:t1]), torch.equal(back, x)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_heads_to_tokens_and_row_gather(world):
    """The token-split prefill's two collectives: the all-to-all hands each rank every
    head of its own token block (head order kept), and the row all-gather puts the
    blocks back in token order, bit for bit."""
    rng = np.random.default_rng(world)
    full = rng.standard_normal((6 * world, 4 * world * 8), dtype=np.float32).astype(np.float16)
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_token_split_worker, args=(r, world, port, full, result_q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = [result_q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, rows_ok, back_ok in got:
        assert rows_ok and back_ok, (rank, rows_ok, back_ok)


def test_token_block_rejects_uneven_split():
    from fast_infer_b200.shard import token_block
    assert token_block(2, 4, 16) == (8, 12)
    with pytest.raises(ValueError):
        token_block(0, 3, 16)
