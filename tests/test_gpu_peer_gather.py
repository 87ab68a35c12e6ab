"""Decode-step head gather over NVLink peer memory (fi_peer_gather), one rank per GPU
on every GPU of the box (2 to 8): the gathered rows equal an NCCL all-gather bit for bit over many calls with
rotating buffers and ragged row counts, and when replayed from a CUDA graph; the
KV-head-sharded stack (decode_exchange="gather") decodes the same bits with the peer
gather as with NCCL, on every rank; no gather reports a time-out. Skipped on a box with fewer than two GPUs."""

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_gather(x, world):
    import torch.distributed as dist
    out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous())
    return out.movedim(0, -2).reshape(*x.shape[:-1], world * x.shape[-1])


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    checks = {}
    try:
        from fast_infer_b200.shard import PeerGather
        from fast_infer_b200.stack import AttentionStack
        rows, elems, nbuf = 16, 3072 // world, 3
        pg = PeerGather(rows, elems, nbuf, device=dev)
        g = torch.Generator(device=dev)
        g.manual_seed(100 + rank)
        ok = True
        for call in range(12):
            x = torch.randn(rows - (call % 3), elems, generator=g, device=dev).half()
            got = pg.gather(x, call % nbuf).clone()
            ok = ok and torch.equal(got, _nccl_gather(x, world))
        checks["eager"] = ok

        xs = [torch.randn(rows, elems, generator=g, device=dev).half() for _ in range(nbuf)]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                outs = [pg.gather(xs[b], b) for b in range(nbuf)]
        torch.cuda.current_stream(dev).wait_stream(side)
        refs = [_nccl_gather(x, world) for x in xs]
        ok = True
        for _ in range(5):
            graph.replay()
            torch.cuda.synchronize(dev)
            ok = ok and all(torch.equal(o, r) for o, r in zip(outs, refs))
        checks["graph"] = ok
        del graph
        checks["no_timeout"] = pg.errors() == 0
        pg.close()

        results = {}
        for mode in ("gather", "nccl"):
            st = AttentionStack(num_layers=3, batch=4, max_seq_len=256, rank=rank, world=world,
                                device=dev, seed=7, decode_exchange=mode)
            gp = torch.Generator(device=dev)
            gp.manual_seed(8)
            prompt = (torch.randn(4, 64, 3072, generator=gp, device=dev) * 0.5).half()
            results[mode] = st.generate(prompt, steps=6, use_graph=True).cpu()
            checks[f"peer_used_{mode}"] = st._peer is not None
            st.close()
        checks["stack_same_bits"] = torch.equal(results["gather"], results["nccl"])
        torch.save({"checks": checks, "out": results["gather"]}, Path(out_dir) / f"r{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_wait_runs_out_and_reports_timeout(cuda_device):
    """One GPU, one kernel: rank 0 of a two-rank gather whose rank 1 never calls (both
    regions are plain memory of this GPU; nothing writes rank 1's words). The wait
    gives up after its 2 s bound, the host reads FI_DEVERR_TIMEOUT, rank 0's own rows
    arrived, a second call with the same error word returns at once without waiting,
    and the context still runs kernels (a one-rank gather gives its input back)."""
    import ctypes
    import time
    from fast_infer_b200 import _lib
    lib = _lib.load()
    world, rows, elems, nbuf = 2, 4, 256, 2
    row_bytes = elems * 2
    nbytes = lib.fi_peer_gather_bytes(nbuf, rows, world * row_bytes)
    regions = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device) for _ in range(world)]
    bases = (ctypes.c_void_p * world)(*[r.data_ptr() for r in regions])
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    x = torch.randn(rows, elems, device=cuda_device).half()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream

    def gather(b, bs, w, e):
        st = lib.fi_peer_gather(x.data_ptr(), rows, row_bytes, row_bytes,
                                ctypes.cast(bs, ctypes.POINTER(ctypes.c_void_p)), w, 0, b,
                                nbuf, rows, e.data_ptr(), stream)
        _lib.check(st, "peer gather")

    torch.cuda.synchronize()
    t0 = time.monotonic()
    gather(0, bases, world, err)
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(err.item()) == _lib.FI_DEVERR_TIMEOUT
    assert 1.5 < waited < 30.0, waited
    out = regions[0][:rows * world * row_bytes].view(torch.float16).view(rows, world * elems)
    assert torch.equal(out[:, :elems], x)  # its own rows landed; rank 1's never came

    t0 = time.monotonic()
    gather(1, bases, world, err)  # the sticky error word: no second wait
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 1.0
    assert int(err.item()) == _lib.FI_DEVERR_TIMEOUT

    one = torch.zeros(lib.fi_peer_gather_bytes(nbuf, rows, row_bytes), dtype=torch.uint8,
                      device=cuda_device)
    err1 = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    gather(0, (ctypes.c_void_p * 1)(one.data_ptr()), 1, err1)
    torch.cuda.synchronize()
    assert int(err1.item()) == 0
    assert torch.equal(one[:rows * row_bytes].view(torch.float16).view(rows, elems), x)


def test_peer_gather_all_gpus(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    for r in res:
        assert r["checks"] == {"eager": True, "graph": True, "no_timeout": True,
                               "peer_used_gather": True, "peer_used_nccl": False,
                               "stack_same_bits": True}, r["checks"]
    for r in res[1:]:
        assert torch.equal(res[0]["out"], r["out"])
