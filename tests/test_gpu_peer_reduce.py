"""O projection sharded by head with the cross-rank sum inside the GEMM
(fi_small_gemm_peer_reduce / PeerReduce).

One GPU: with one rank the result is fp16(x @ w^T) + residual, within one fp16 ulp of
the unsharded decode GEMM; a two-rank call whose second rank never calls gives up
after its 2 s bound and reports FI_DEVERR_TIMEOUT (both regions plain memory of this
GPU, nothing writes rank 1's partials). Every GPU of the box (2 to 8 ranks): the
result equals an NCCL all-reduce of the ranks' partials within tolerance, eagerly and
replayed from a CUDA graph, with the same bits on every rank; the KV-head-sharded
stack decodes within tolerance of the NCCL-gather stack."""

import ctypes
import datetime
import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _call(lib, x, w, out, res, bases, world, rank, buffer, nbuf, err):
    from fast_infer_b200 import _lib
    return lib.fi_small_gemm_peer_reduce(
        x.data_ptr(), w.data_ptr(), out.data_ptr(), res.data_ptr() if res is not None else None,
        x.shape[0], w.shape[0], x.shape[1], _lib.strides(*x.stride()), _lib.strides(*w.stride()),
        _lib.strides(*out.stride()), _lib.strides(*res.stride()) if res is not None else None,
        ctypes.cast(bases, ctypes.POINTER(ctypes.c_void_p)), world, rank, buffer, nbuf, 0,
        err.data_ptr() if err is not None else None, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m", [1, 5, 16])
def test_one_rank_matches_the_decode_gemm(cuda_device, m):
    from fast_infer_b200 import _lib
    from fast_infer_b200.kernels.matmul import fp16_linear
    lib = _lib.load()
    g = torch.Generator(device=cuda_device)
    g.manual_seed(m)
    n, k, nbuf = 3072, 384, 2
    region = torch.zeros(lib.fi_peer_reduce_bytes(nbuf, 1, n), dtype=torch.uint8,
                         device=cuda_device)
    bases = (ctypes.c_void_p * 1)(region.data_ptr())
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for call in range(4):  # buffers rotate; the call counter advances on the device
        x = torch.randn(m, k, generator=g, device=cuda_device).half()
        w = (torch.randn(n, k, generator=g, device=cuda_device) * 0.05).half()
        res = torch.randn(m, n, generator=g, device=cuda_device).half()
        out = torch.empty_like(res)
        assert _call(lib, x, w, out, res, bases, 1, 0, call % nbuf, nbuf, err) == _lib.FI_OK
        ref = fp16_linear(x, w, residual=res)
        part = (x.float() @ w.float().t()).half().float()
        exact = (part + res.float()).half()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        # the partial is rounded to fp16 before the residual is added: within one
        # ulp of the output of the unsharded GEMM, and equal to that formula up to
        # one ulp of the partial (fp32 summation order)
        ulp = torch.finfo(torch.float16).eps * out.float().abs().clamp_min(1.0)
        assert ((out.float() - ref.float()).abs() <= 1.01 * ulp).all()
        ulp_p = torch.finfo(torch.float16).eps * part.abs().clamp_min(2 ** -14)
        assert ((out.float() - exact.float()).abs() <= ulp + ulp_p).all()
    # in place (out is the residual), as the stack calls it
    x = torch.randn(m, k, generator=g, device=cuda_device).half()
    h = torch.randn(m, n, generator=g, device=cuda_device).half()
    expect = torch.empty_like(h)
    assert _call(lib, x, w, expect, h, bases, 1, 0, 0, nbuf, err) == _lib.FI_OK
    assert _call(lib, x, w, h, h, bases, 1, 0, 1, nbuf, err) == _lib.FI_OK
    torch.cuda.synchronize()
    assert torch.equal(h, expect)


def test_wait_runs_out_and_reports_timeout(cuda_device):
    """Rank 0 of two on one GPU, rank 1 never calls: its partials never land, the wait
    gives up after 2 s, FI_DEVERR_TIMEOUT is reported, a second call with the same
    error word does not wait, and the context still runs kernels."""
    from fast_infer_b200 import _lib
    lib = _lib.load()
    n, k, m, nbuf = 256, 128, 4, 2
    nbytes = lib.fi_peer_reduce_bytes(nbuf, 2, n)
    regions = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device) for _ in range(2)]
    bases = (ctypes.c_void_p * 2)(regions[0].data_ptr(), regions[1].data_ptr())
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    x = torch.randn(m, k, device=cuda_device).half()
    w = torch.randn(n, k, device=cuda_device).half()
    out = torch.zeros(m, n, dtype=torch.float16, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    assert _call(lib, x, w, out, None, bases, 2, 0, 0, nbuf, err) == _lib.FI_OK
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(err.item()) == _lib.FI_DEVERR_TIMEOUT
    assert 1.5 < waited < 30.0, waited
    t0 = time.monotonic()
    assert _call(lib, x, w, out, None, bases, 2, 0, 1, nbuf, err) == _lib.FI_OK
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 1.0
    one = torch.zeros(lib.fi_peer_reduce_bytes(nbuf, 1, n), dtype=torch.uint8, device=cuda_device)
    err1 = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    assert _call(lib, x, w, out, None, (ctypes.c_void_p * 1)(one.data_ptr()), 1, 0, 0, nbuf,
                 err1) == _lib.FI_OK
    torch.cuda.synchronize()
    assert int(err1.item()) == 0
    ref = (x.float() @ w.float().t()).half()
    ulp = torch.finfo(torch.float16).eps * ref.float().abs().clamp_min(2 ** -14)
    assert ((out.float() - ref.float()).abs() <= ulp).all()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


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
        from fast_infer_b200.shard import PeerReduce
        from fast_infer_b200.stack import AttentionStack
        n, k, m, nbuf = 3072, 3072 // world, 16, 3
        pr = PeerReduce(n, nbuf, device=dev)
        g = torch.Generator(device=dev)
        g.manual_seed(200 + rank)
        gs = torch.Generator(device=dev)
        gs.manual_seed(300)  # the residual is the same on every rank
        worst = 0.0
        outs = []
        for call in range(9):
            x = torch.randn(m - (call % 3), k, generator=g, device=dev).half()
            w = (torch.randn(n, k, generator=g, device=dev) * 0.02).half()
            res = torch.randn(x.shape[0], n, generator=gs, device=dev).half()
            out = torch.empty_like(res)
            pr.linear(x, w, res, out, call % nbuf)
            ref = (x.float() @ w.float().t())
            dist.all_reduce(ref)
            ref = ref + res.float()
            worst = max(worst, _rel(out, ref))
            outs.append(out)
        checks["eager_rel"] = worst < 1e-3
        same = True
        for o in outs:
            r0 = o.clone()
            dist.broadcast(r0, 0)
            same = same and torch.equal(r0, o)
        checks["same_on_every_rank"] = same

        xs = [torch.randn(m, k, generator=g, device=dev).half() for _ in range(nbuf)]
        w = (torch.randn(n, k, generator=g, device=dev) * 0.02).half()
        res = torch.randn(m, n, generator=gs, device=dev).half()
        gouts = [torch.empty_like(res) for _ in range(nbuf)]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for b in range(nbuf):
                    pr.linear(xs[b], w, res, gouts[b], b)
        torch.cuda.current_stream(dev).wait_stream(side)
        refs = []
        for b in range(nbuf):
            r = xs[b].float() @ w.float().t()
            dist.all_reduce(r)
            refs.append(r + res.float())
        ok = True
        first = None
        for _ in range(4):
            graph.replay()
            torch.cuda.synchronize(dev)
            ok = ok and all(_rel(o, r) < 1e-3 for o, r in zip(gouts, refs))
            snap = [o.clone() for o in gouts]
            if first is None:
                first = snap
            ok = ok and all(torch.equal(a, b) for a, b in zip(snap, first))
        checks["graph"] = ok
        del graph
        checks["no_timeout"] = pr.errors() == 0
        pr.close()

        results = {}
        for mode in ("reduce", "nccl"):
            st = AttentionStack(num_layers=3, batch=4, max_seq_len=256, rank=rank, world=world,
                                device=dev, seed=7, decode_exchange=mode)
            gp = torch.Generator(device=dev)
            gp.manual_seed(8)
            prompt = (torch.randn(4, 64, 3072, generator=gp, device=dev) * 0.5).half()
            results[mode] = st.generate(prompt, steps=6, use_graph=True).cpu()
            checks[f"reduce_used_{mode}"] = st._reduce is not None
            checks[f"stack_errors_{mode}"] = st._reduce.errors() if st._reduce else 0
            st.close()
        checks["stack_close_to_nccl"] = _rel(results["reduce"], results["nccl"]) < 1e-3
        # prefill with the residual stream split by token (all-to-all of head outputs)
        # against the head all-gather with the whole O projection on every rank
        pf = {}
        for pmode in ("tokens", "gather"):
            st = AttentionStack(num_layers=3, batch=4, max_seq_len=256, rank=rank, world=world,
                                device=dev, seed=7, prefill_exchange=pmode)
            pf[pmode] = st.prefill(prompt).cpu()
            st.close()
        checks["prefill_tokens_close_to_gather"] = _rel(pf["tokens"], pf["gather"]) < 1e-3
        torch.save({"checks": checks, "out": results["reduce"]}, Path(out_dir) / f"r{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_peer_reduce_all_gpus(tmp_path):
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
        assert r["checks"] == {"eager_rel": True, "same_on_every_rank": True, "graph": True,
                               "no_timeout": True, "reduce_used_reduce": True,
                               "stack_errors_reduce": 0, "reduce_used_nccl": False,
                               "stack_errors_nccl": 0, "stack_close_to_nccl": True,
                               "prefill_tokens_close_to_gather": True}, r["checks"]
    for r in res[1:]:
        assert torch.equal(res[0]["out"], r["out"])
