"""GPU parity of fi_rms_norm against the reference's outputs (golden) and the oracle:
within one fp16 rounding step (the sum order and the reciprocal square root differ
between implementations)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.norm_oracle import rms_norm as rms_oracle
from tests.golden.inputs import RMS_CASES, rms_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _close(out, ref):
    o, r = out.astype(np.float32), ref.astype(np.float32)
    return bool(np.all(np.abs(o - r) <= 2.0 ** -10 * np.abs(r) + 1e-4)), float(np.abs(o - r).max())


def test_matches_reference_kernel(cuda_device):
    from fast_infer_b200.kernels.rms_norm import rms_norm
    g = np.load(GOLDEN / "rms_norm.npz")
    for rows, hidden in RMS_CASES:
        x, w = rms_inputs(rows, hidden)
        out = rms_norm(torch.from_numpy(x).to(cuda_device), torch.from_numpy(w).to(cuda_device))
        ok, err = _close(out.cpu().numpy(), g[f"out_{rows}x{hidden}"])
        assert ok, (rows, hidden, err)


@pytest.mark.parametrize("shape", [(16, 1, 3072), (3, 77, 3072), (16384, 3072), (5, 8), (2, 4096)])
def test_shapes_vs_oracle(cuda_device, shape):
    from fast_infer_b200.kernels.rms_norm import rms_norm
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal(size=shape, dtype=np.float32).astype(np.float16)
    w = (1.0 + 0.1 * rng.standard_normal(size=(shape[-1],), dtype=np.float32)).astype(np.float16)
    out = rms_norm(torch.from_numpy(x).to(cuda_device), torch.from_numpy(w).to(cuda_device))
    assert out.shape == shape
    ok, err = _close(out.cpu().numpy(), rms_oracle(x, w))
    assert ok, (shape, err)


def test_strided_rows_and_empty(cuda_device):
    from fast_infer_b200.kernels.rms_norm import rms_norm
    rng = np.random.default_rng(5)
    big = torch.from_numpy(rng.standard_normal(size=(6, 3072 + 64), dtype=np.float32)
                           .astype(np.float16)).to(cuda_device)
    x = big[:, 32:32 + 3072]
    w = torch.ones(3072, dtype=torch.float16, device=cuda_device)
    out = rms_norm(x, w)
    ok, err = _close(out.cpu().numpy(), rms_oracle(x.cpu().numpy(), w.cpu().numpy()))
    assert ok, err
    assert rms_norm(torch.empty(0, 3072, dtype=torch.float16, device=cuda_device), w).shape == (0, 3072)
