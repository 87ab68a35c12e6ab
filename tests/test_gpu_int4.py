"""GPU parity of the INT4 weight path: the CUDA quantizer and dequantizer reproduce
the reference's bytes exactly; the fused dequant-matmul matches the reference
kernel's outputs (golden) and the numpy oracle within the INT4 tolerance (one fp16
ulp of the output plus 1e-3, relative L2 <= 1e-3)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.int4_oracle import dequantize_int4, int4_matmul, quantize_int4_groupwise
from tests.golden.inputs import INT4_CASES, int4_inputs
from tests.test_int4_oracle import int4_close

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"

# Llama-3.2-3B projections: (name, N, K) — qkv, o, gate_up, down.
LLAMA_SHAPES = (("qkv", 5120, 3072), ("o", 3072, 3072), ("gate_up", 16384, 3072),
                ("down", 3072, 8192))


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _weights(n, k, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(size=(n, k), dtype=np.float32) * scale).astype(np.float16)


def _x(m, k, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(size=(m, k), dtype=np.float32).astype(np.float16)


@pytest.mark.parametrize("case", [c[0] for c in INT4_CASES])
def test_quantize_and_dequant_bit_identical_to_reference(cuda_device, case):
    from fast_infer_b200.loader import dequantize_int4 as gpu_dequant
    from fast_infer_b200.loader import quantize_int4_groupwise as gpu_quant
    g = np.load(GOLDEN / "int4.npz")
    w, _, gs = int4_inputs(case)
    packed, scales = gpu_quant(_dev(w, cuda_device), groupsize=gs)
    assert np.array_equal(packed.cpu().numpy(), g[f"{case}_packed"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint16), g[f"{case}_scales"].view(np.uint16))
    d = gpu_dequant(packed, scales, groupsize=gs)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), g[f"{case}_dequant"].view(np.uint16))


def test_quantize_dequant_large_and_subnormal_scales(cuda_device):
    from fast_infer_b200.loader import dequantize_int4 as gpu_dequant
    from fast_infer_b200.loader import quantize_int4_groupwise as gpu_quant
    w = _weights(512, 3072, 5)
    w[3] *= np.float16(1e-3)   # scales below fp16's normal range (subnormal products)
    w[4, :128] = 0             # clamped all-zero group
    w[5, 7] = np.float16(-9.0)  # outlier: rest of the group rounds to 0
    packed, scales = gpu_quant(_dev(w, cuda_device))
    p_ref, s_ref = quantize_int4_groupwise(w)
    assert np.array_equal(packed.cpu().numpy(), p_ref)
    assert np.array_equal(scales.cpu().numpy().view(np.uint16), s_ref.view(np.uint16))
    d = gpu_dequant(packed, scales).cpu().numpy()
    assert np.array_equal(d.view(np.uint16), dequantize_int4(p_ref, s_ref).view(np.uint16))


@pytest.mark.parametrize("case", [c[0] for c in INT4_CASES])
def test_matmul_matches_reference_kernel_outputs(cuda_device, case):
    from fast_infer_b200.kernels.matmul import int4_matmul as gpu_mm
    g = np.load(GOLDEN / "int4.npz")
    _, xs, gs = int4_inputs(case)
    packed = _dev(g[f"{case}_packed"], cuda_device)
    scales = _dev(g[f"{case}_scales"], cuda_device)
    for m, x in xs.items():
        c = gpu_mm(_dev(x, cuda_device), (packed, scales), groupsize=gs).cpu().numpy()
        ok, max_abs, rel = int4_close(c, g[f"{case}_c_m{m}"])
        assert ok, (case, m, max_abs, rel)


_LLAMA_CACHE = {}


def _llama_weights(n, k, device):
    """Oracle-quantized weights of one shape, their oracle dequant (fp64) and device
    copies, built once per shape (numpy's fp16 arithmetic is slow at 50M elements)."""
    if (n, k) not in _LLAMA_CACHE:
        packed, scales = quantize_int4_groupwise(_weights(n, k, n + k))
        wd = dequantize_int4(packed, scales).astype(np.float64)
        _LLAMA_CACHE[(n, k)] = (wd, _dev(packed, device), _dev(scales, device))
    return _LLAMA_CACHE[(n, k)]


@pytest.mark.parametrize("name,n,k", LLAMA_SHAPES)
@pytest.mark.parametrize("m", [1, 16, 40, 64, 80])
def test_llama_projection_shapes_vs_oracle(cuda_device, name, n, k, m):
    from fast_infer_b200.kernels.matmul import int4_matmul as gpu_mm
    wd, packed, scales = _llama_weights(n, k, cuda_device)
    x = _x(m, k, m + n)
    # oracle int4_matmul: fp64 product of x and the oracle's fp16 dequant, rounded to fp16
    ref = (x.astype(np.float64) @ wd.T).astype(np.float32).astype(np.float16)
    c = gpu_mm(_dev(x, cuda_device), (packed, scales))
    ok, max_abs, rel = int4_close(c.cpu().numpy(), ref)
    assert ok, (name, m, max_abs, rel)


@pytest.mark.parametrize("n,k,gs,m", [(100, 256, 128, 3), (1000, 96, 32, 7), (130, 160, 32, 17),
                                      (8, 128, 128, 1), (257, 640, 64, 33), (4096, 4096, 128, 2),
                                      (8, 128, 128, 12), (100, 256, 128, 10), (130, 160, 32, 16),
                                      (4112, 3072, 128, 9),
                                      # x too large for shared memory at 9-16 tokens: staged
                                      # round by round (group size 128), or read from
                                      # global memory (group size 64)
                                      (3000, 8192, 128, 11), (1000, 8192, 64, 16)])
def test_ragged_shapes_and_group_sizes(cuda_device, n, k, gs, m):
    from fast_infer_b200.kernels.matmul import int4_matmul as gpu_mm
    w = _weights(n, k, 7 * n + k)
    packed, scales = quantize_int4_groupwise(w, gs)
    x = _x(m, k, 3 * m + k)
    ref = int4_matmul(x, packed, scales, gs)
    c = gpu_mm(_dev(x, cuda_device), (_dev(packed, cuda_device), _dev(scales, cuda_device)),
               groupsize=gs)
    ok, max_abs, rel = int4_close(c.cpu().numpy(), ref)
    assert ok, (n, k, gs, m, max_abs, rel)


def test_strided_operands_and_batched_input(cuda_device):
    from fast_infer_b200 import _lib
    from fast_infer_b200.kernels.matmul import int4_matmul as gpu_mm
    n, k, m = 768, 1024, 12
    w = _weights(n, k, 99)
    packed, scales = quantize_int4_groupwise(w)
    x = _x(m, k, 98)
    ref = int4_matmul(x, packed, scales)
    # x as a column slice of a wider buffer, scales transposed in memory, 3-D input
    xb = torch.zeros(m, k + 64, dtype=torch.float16, device=cuda_device)
    xb[:, 32:32 + k] = _dev(x, cuda_device)
    sc_t = _dev(scales, cuda_device).t().contiguous().t()
    c = gpu_mm(xb[:, 32:32 + k], (_dev(packed, cuda_device), sc_t))
    assert int4_close(c.cpu().numpy(), ref)[0]
    c3 = gpu_mm(_dev(x, cuda_device).reshape(3, 4, k), (_dev(packed, cuda_device), sc_t))
    assert c3.shape == (3, 4, n)
    assert int4_close(c3.reshape(m, n).cpu().numpy(), ref)[0]
    # output into a transposed view through the C ABI (any output strides)
    lib = _lib.load()
    xd, pd, sd = _dev(x, cuda_device), _dev(packed, cuda_device), _dev(scales, cuda_device)
    ct = torch.empty(n, m, dtype=torch.float16, device=cuda_device).t()
    st = lib.fi_int4_gemm(xd.data_ptr(), pd.data_ptr(), sd.data_ptr(), ct.data_ptr(), m, n, k,
                          128, _lib.strides(*xd.stride()), _lib.strides(*pd.stride()),
                          _lib.strides(*sd.stride()), _lib.strides(*ct.stride()), None,
                          torch.cuda.current_stream().cuda_stream)
    assert st == _lib.FI_OK
    assert int4_close(ct.cpu().numpy(), ref)[0]


def test_deterministic_across_calls_and_shapes(cuda_device):
    from fast_infer_b200.kernels.matmul import int4_matmul as gpu_mm
    shapes = [(3072, 8192, 16), (5120, 3072, 1), (3072, 8192, 16), (16384, 3072, 64)]
    first = {}
    from fast_infer_b200.loader import quantize_int4_groupwise as gpu_quant
    for n, k, m in shapes:
        wt = gpu_quant(_dev(_weights(n, k, n ^ k), cuda_device))
        x = _dev(_x(m, k, m), cuda_device)
        outs = [gpu_mm(x, wt) for _ in range(3)]
        for o in outs[1:]:
            assert torch.equal(o, outs[0])
        key = (n, k, m)
        if key in first:
            assert torch.equal(first[key], outs[0])
        first[key] = outs[0]


def test_dense_speed_mode_and_weight_preparation(cuda_device):
    from fast_infer_b200.kernels.matmul import (_dequant_storage, dequantize_all,
                                                fuse_qkv_inplace, int4_matmul as gpu_mm)
    n, k, m = 256, 512, 5
    w = _weights(n, k, 17)
    packed, scales = quantize_int4_groupwise(w)
    x = _x(m, k, 18)
    wd = _dequant_storage(_dev(packed, cuda_device), _dev(scales, cuda_device))
    assert np.array_equal(wd.cpu().numpy().view(np.uint16),
                          dequantize_int4(packed, scales).view(np.uint16))
    c = gpu_mm(_dev(x, cuda_device), wd)
    assert int4_close(c.cpu().numpy(), int4_matmul(x, packed, scales))[0]
    t = lambda: (_dev(packed, cuda_device), _dev(scales, cuda_device))
    layer = {"self_attn": {p: t() for p in ("q_proj", "k_proj", "v_proj", "o_proj")},
             "mlp": {p: t() for p in ("gate_proj", "up_proj", "down_proj")}}
    fused = {"layers": [{"self_attn": dict(layer["self_attn"]), "mlp": dict(layer["mlp"])}]}
    fuse_qkv_inplace(fused)
    sa = fused["layers"][0]["self_attn"]
    assert set(sa) == {"qkv_proj", "o_proj"} and sa["qkv_proj"][0].shape == (3 * n, k // 2)
    qkv = gpu_mm(_dev(x, cuda_device), sa["qkv_proj"])
    assert int4_close(qkv[:, :n].cpu().numpy(), int4_matmul(x, packed, scales))[0]
    dense = dequantize_all({"layers": [layer]})
    sa = dense["layers"][0]["self_attn"]
    assert sa["qkv_proj"].dtype == torch.float16 and sa["qkv_proj"].shape == (3 * n, k)
    assert dense["layers"][0]["mlp"]["gate_up_proj"].shape == (2 * n, k)


def test_reference_error_behaviour(cuda_device):
    from fast_infer_b200.kernels.matmul import int4_matmul as gpu_mm
    packed = torch.zeros(8, 64, dtype=torch.int8, device=cuda_device)
    scales = torch.ones(8, 1, dtype=torch.float16, device=cuda_device)
    with pytest.raises(AssertionError):
        gpu_mm(torch.zeros(2, 100, dtype=torch.float16, device=cuda_device), (packed, scales))
    with pytest.raises(AssertionError):
        gpu_mm(torch.zeros(2, 256, dtype=torch.float16, device=cuda_device), (packed, scales))
    with pytest.raises(ValueError):
        gpu_mm(torch.zeros(2, 128), (packed.cpu(), scales.cpu()))
