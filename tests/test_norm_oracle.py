"""The RMSNorm oracle reproduces the reference's Triton kernel (golden vectors made by
running kernels/rms_norm.py under TRITON_INTERPRET=1; see tests/golden/make_golden.py)."""

from pathlib import Path

import numpy as np

from oracle.norm_oracle import rms_norm
from tests.golden.inputs import RMS_CASES, rms_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_rms_norm_matches_reference_kernel():
    g = np.load(GOLDEN / "rms_norm.npz")
    for rows, hidden in RMS_CASES:
        x, w = rms_inputs(rows, hidden)
        out = rms_norm(x, w)
        assert np.array_equal(out.view(np.uint16), g[f"out_{rows}x{hidden}"].view(np.uint16))
