"""Decode-sized fp16 GEMM (fi_small_gemm via kernels.matmul.fp16_linear): against an
fp32 reference within one fp16 ulp of the output plus 1e-3 (rel-L2 <= 1e-3); the
fused RMSNorm prologue gives the same bits as fi_rms_norm followed by the plain GEMM;
residual in place; ragged N and K; deterministic; more than 16 rows fall back to the
dense library path with the same semantics."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _kernel_up_to_16_rows(monkeypatch):
    """Route every size the kernel supports (up to 16 rows) through fi_small_gemm."""
    import fast_infer_b200.kernels.matmul as mm
    monkeypatch.setattr(mm, "SMALL_GEMM_MAX_M", 16)
    monkeypatch.setattr(mm, "STREAM_GEMM_MAX_M", 16)


def _close(out, ref, abs_tol=1e-3, rel_tol=2.0 ** -10):
    out, ref = out.float(), ref.float()
    err = (out - ref).abs()
    ok = bool((err <= abs_tol + ref.abs() * rel_tol).all())
    rel = float((out - ref).norm() / ref.norm().clamp_min(1e-30))
    return ok and rel <= 1e-3, float(err.max()), rel


def _data(m, n, k, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(m, k, device=dev, generator=g).half()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).half()
    res = torch.randn(m, n, device=dev, generator=g).half()
    nw = (1 + 0.1 * torch.randn(k, device=dev, generator=g)).half()
    return x, w, res, nw


@pytest.mark.parametrize("m", [1, 5, 8, 9, 16])
@pytest.mark.parametrize("n,k", [(2560, 3072), (3072, 3072), (100, 192), (17, 64), (5120, 3072)])
def test_against_fp32(cuda_device, m, n, k):
    from fast_infer_b200.kernels.matmul import fp16_linear
    from fast_infer_b200.kernels.rms_norm import rms_norm
    x, w, res, nw = _data(m, n, k, cuda_device, m * 131 + n + k)
    plain = fp16_linear(x, w)
    ok = _close(plain, x.float() @ w.float().t())
    assert ok[0], ("plain", ok)
    xn = rms_norm(x, nw, 1e-5)
    full = fp16_linear(x, w, residual=res, norm_weight=nw)
    ok = _close(full, res.float() + xn.float() @ w.float().t())
    assert ok[0], ("norm+residual", ok)
    # the fused norm reproduces fi_rms_norm bit for bit
    assert torch.equal(fp16_linear(x, w, norm_weight=nw), fp16_linear(xn, w))


def test_residual_in_place_and_determinism(cuda_device):
    from fast_infer_b200.kernels.matmul import fp16_linear
    x, w, res, nw = _data(16, 3072, 3072, cuda_device, 7)
    expect = fp16_linear(x, w, residual=res, norm_weight=nw)
    h = res.clone()
    fp16_linear(x, w, residual=h, norm_weight=nw, out=h)
    assert torch.equal(h, expect)
    for _ in range(3):
        assert torch.equal(fp16_linear(x, w, residual=res, norm_weight=nw), expect)


def test_leading_dims_strides_and_fallback(cuda_device):
    from fast_infer_b200.kernels.matmul import fp16_linear
    from fast_infer_b200.kernels.rms_norm import rms_norm
    x, w, res, nw = _data(12, 768, 1024, cuda_device, 9)
    wide = torch.zeros(12, 1024 + 64, dtype=torch.float16, device=cuda_device)
    wide[:, 32:32 + 1024] = x
    a = fp16_linear(wide[:, 32:32 + 1024], w, residual=res, norm_weight=nw)
    b = fp16_linear(x.reshape(3, 4, 1024), w, residual=res.reshape(3, 4, 768), norm_weight=nw)
    assert b.shape == (3, 4, 768)
    assert torch.equal(a, b.reshape(12, 768))
    # 40 rows: the dense path, same semantics
    x4, w4, r4, n4 = _data(40, 768, 1024, cuda_device, 10)
    big = fp16_linear(x4, w4, residual=r4, norm_weight=n4)
    ref = r4.float() + rms_norm(x4, n4).float() @ w4.float().t()
    assert _close(big, ref)[0]


@pytest.mark.parametrize("m", [1, 7, 16])
@pytest.mark.parametrize("n,k", [(2560, 3072), (5120, 3072), (100, 192)])
def test_folded_norm(cuda_device, m, n, k):
    """RMSNorm weight folded into the weights, per-row factor in the epilogue, against
    rms_norm(x) @ w.T (+ residual) in fp32. Folding rounds every w * g to fp16 (where
    the reference rounds the normalised x): one more fp16 rounding per product, so the
    bound is max-abs 2e-3 + two fp16 ulps of the output, rel-L2 <= 1e-3."""
    from fast_infer_b200.kernels.matmul import fold_rms_weight, fp16_linear_folded
    x, w, res, nw = _data(m, n, k, cuda_device, m * 7 + n + k)
    wf = fold_rms_weight(w, nw)
    xf = x.float()
    xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.float()
    ok = _close(fp16_linear_folded(x, wf), xn @ w.float().t(), 2e-3, 2.0 ** -9)
    assert ok[0], ok
    ok = _close(fp16_linear_folded(x, wf, residual=res), res.float() + xn @ w.float().t(),
                2e-3, 2.0 ** -9)
    assert ok[0], ok
    h = res.clone()
    fp16_linear_folded(x, wf, residual=h, out=h)
    assert torch.equal(h, fp16_linear_folded(x, wf, residual=res))


@pytest.mark.parametrize("m", [1, 8, 16])
def test_static_weights_same_bits(cuda_device, m):
    """FI_STATIC_WEIGHTS (weight tiles loaded before the dependency wait) changes no
    bit: staged (norm) and streamed paths, folded, and a back-to-back chain in which
    every x is the previous kernel's output, eagerly and from a CUDA graph."""
    from fast_infer_b200.kernels.matmul import fold_rms_weight, fp16_linear, fp16_linear_folded
    x, w, res, nw = _data(m, 3072, 3072, cuda_device, 40 + m)
    for kw in ({}, {"norm_weight": nw}, {"residual": res}):
        assert torch.equal(fp16_linear(x, w, static_weight=True, **kw), fp16_linear(x, w, **kw))
    wf = fold_rms_weight(w, nw)
    assert torch.equal(fp16_linear_folded(x, wf, residual=res, static_weight=True),
                       fp16_linear_folded(x, wf, residual=res))

    g = torch.Generator(device=cuda_device)
    g.manual_seed(3)
    ws = [(torch.randn(3072, 3072, device=cuda_device, generator=g) * 0.02).half()
          for _ in range(4)]

    def chain(static, sync):
        h = x
        for i, wi in enumerate(ws):
            h = (fp16_linear_folded(h, wi, static_weight=static) if i % 2 else
                 fp16_linear(h, wi, residual=h, static_weight=static))
            if sync:
                torch.cuda.synchronize()
        return h

    ref = chain(False, True)
    for _ in range(3):
        out = chain(True, False)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        chain(True, False)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            gout = chain(True, False)
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, ref)
    del graph
