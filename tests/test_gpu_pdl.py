"""Programmatic dependent launch: the library's kernels may start while the previous
kernel on the stream finishes, and read its output only after their dependency wait.
Chains of dependent calls (each input the previous call's output, intermediates freed
at once so the caching allocator recycles them) must give bit-identical results with
a synchronisation after every call, replayed from a CUDA graph, and with the overlap
switched off (FI_PDL=0, in a child process)."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

# (N, K) of the projections in the chain: each K is the previous N.
CHAIN = ((3072, 3072), (8192, 3072), (3072, 8192), (5120, 3072), (3072, 5120))


def _chain_weights(device, seed=11):
    from fast_infer_b200.loader import quantize_int4_groupwise
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    ws = []
    for n, k in CHAIN:
        w = (torch.randn(n, k, device=device, generator=g) * 0.02).half()
        ws.append(quantize_int4_groupwise(w, 128))
    norm_w = (1 + 0.1 * torch.randn(3072, device=device, generator=g)).half()
    return ws, norm_w


def _run_chain(x, ws, norm_w, sync_each=False):
    from fast_infer_b200.kernels.matmul import int4_matmul
    from fast_infer_b200.kernels.rms_norm import rms_norm
    h = x
    for w in ws:
        h = int4_matmul(h, w, groupsize=128)
        if sync_each:
            torch.cuda.synchronize()
        if h.shape[-1] == 3072:
            h = rms_norm(h, norm_w, 1e-5)
            if sync_each:
                torch.cuda.synchronize()
    return h


@pytest.mark.parametrize("m", [1, 16])
def test_int4_rmsnorm_chain_matches_synchronised_and_graph(cuda_device, m):
    ws, norm_w = _chain_weights(cuda_device)
    g = torch.Generator(device=cuda_device)
    g.manual_seed(5)
    x = torch.randn(m, 3072, device=cuda_device, generator=g).half()
    ref = _run_chain(x, ws, norm_w, sync_each=True)
    assert torch.isfinite(ref.float()).all()
    for _ in range(3):  # back-to-back repeats: every launch overlaps its predecessor
        out = _run_chain(x, ws, norm_w)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)

    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        _run_chain(x, ws, norm_w)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            gout = _run_chain(x, ws, norm_w)
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, ref)
    del graph


def test_weights_written_by_the_previous_kernel(cuda_device):
    """fi_int4_quantize writes the weights and fi_int4_gemm reads them in the very next
    launch: the GEMM's early start may only pull them into L2 before its wait."""
    from fast_infer_b200.kernels.matmul import int4_matmul
    from fast_infer_b200.loader import quantize_int4_groupwise
    g = torch.Generator(device=cuda_device)
    g.manual_seed(9)
    x = torch.randn(4, 3072, device=cuda_device, generator=g).half()
    w = (torch.randn(4096, 3072, device=cuda_device, generator=g) * 0.02).half()
    outs = []
    for rep in range(4):
        packed, scales = quantize_int4_groupwise(w * (1 + rep), 128)
        outs.append(int4_matmul(x, (packed, scales), groupsize=128))
    torch.cuda.synchronize()
    for rep in range(4):
        packed, scales = quantize_int4_groupwise(w * (1 + rep), 128)
        torch.cuda.synchronize()
        ref = int4_matmul(x, (packed, scales), groupsize=128)
        torch.cuda.synchronize()
        assert torch.equal(outs[rep], ref), rep


_CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from tests.test_gpu_pdl import _chain_weights, _run_chain
dev = torch.device("cuda:0")
ws, norm_w = _chain_weights(dev)
g = torch.Generator(device=dev); g.manual_seed(5)
x = torch.randn(16, 3072, device=dev, generator=g).half()
out = _run_chain(x, ws, norm_w)
torch.cuda.synchronize()
torch.save(out.cpu(), sys.argv[2])
"""


def test_pdl_off_gives_the_same_bits(cuda_device, tmp_path):
    ws, norm_w = _chain_weights(cuda_device)
    g = torch.Generator(device=cuda_device)
    g.manual_seed(5)
    x = torch.randn(16, 3072, device=cuda_device, generator=g).half()
    out = _run_chain(x, ws, norm_w).cpu()
    path = tmp_path / "off.pt"
    env = dict(os.environ, FI_PDL="0")
    r = subprocess.run([sys.executable, "-c", _CHILD, str(ROOT), str(path)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert torch.equal(torch.load(path), out)
