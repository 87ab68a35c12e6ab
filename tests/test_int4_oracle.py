"""The INT4 oracle reproduces the reference's own weight format and dequant-matmul
(golden vectors from the reference's loader.py quantizer/dequantizer and its fused
Triton kernel under TRITON_INTERPRET=1; see tests/golden/make_golden.py)."""

from pathlib import Path

import numpy as np
import pytest

from oracle.int4_oracle import (dequantize_int4, int4_matmul, int4_weight_bytes,
                                quantize_int4_groupwise, unpack_int4)
from tests.golden.inputs import INT4_CASES, int4_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"

# Output tolerance of every INT4 matmul comparison: one fp16 ulp of the output
# magnitude plus 1e-3 absolute (accumulation order differs between implementations),
# and relative L2 <= 1e-3.
INT4_REL_ULP = 2.0 ** -10
INT4_ABS = 1e-3
INT4_REL_L2 = 1e-3


def int4_close(out: np.ndarray, ref: np.ndarray) -> tuple[bool, float, float]:
    o = out.astype(np.float32)
    r = ref.astype(np.float32)
    err = np.abs(o - r)
    ok_elem = bool(np.all(err <= INT4_ABS + INT4_REL_ULP * np.abs(r)))
    rel = float(np.linalg.norm(o - r) / max(np.linalg.norm(r), 1e-30))
    return ok_elem and rel <= INT4_REL_L2, float(err.max(initial=0.0)), rel


@pytest.mark.parametrize("case", [c[0] for c in INT4_CASES])
def test_quantizer_bit_identical_to_reference(case):
    g = np.load(GOLDEN / "int4.npz")
    w, _, gs = int4_inputs(case)
    packed, scales = quantize_int4_groupwise(w, gs)
    assert packed.dtype == np.int8 and scales.dtype == np.float16
    assert np.array_equal(packed, g[f"{case}_packed"])
    assert np.array_equal(scales.view(np.uint16), g[f"{case}_scales"].view(np.uint16))


@pytest.mark.parametrize("case", [c[0] for c in INT4_CASES])
def test_dequant_bit_identical_to_reference(case):
    g = np.load(GOLDEN / "int4.npz")
    gs = {c[0]: c[3] for c in INT4_CASES}[case]
    d = dequantize_int4(g[f"{case}_packed"], g[f"{case}_scales"], gs)
    assert np.array_equal(d.view(np.uint16), g[f"{case}_dequant"].view(np.uint16))
    assert np.array_equal(d.view(np.uint16), g[f"{case}_dequant_storage"].view(np.uint16))


@pytest.mark.parametrize("case", [c[0] for c in INT4_CASES])
def test_matmul_matches_reference_kernel(case):
    g = np.load(GOLDEN / "int4.npz")
    _, xs, gs = int4_inputs(case)
    for m, x in xs.items():
        c = int4_matmul(x, g[f"{case}_packed"], g[f"{case}_scales"], gs)
        ok, max_abs, rel = int4_close(c, g[f"{case}_c_m{m}"])
        assert ok, (case, m, max_abs, rel)


def test_format_edges():
    # All 16 nibble values round-trip through pack/unpack; the clamp keeps a zero
    # group finite; an outlier saturates at +7 / -8 of its group's scale.
    q = np.arange(-8, 8, dtype=np.int8)
    packed = ((q[0::2] & 0xF) | ((q[1::2] & 0xF) << 4)).astype(np.uint8).view(np.int8)
    assert np.array_equal(unpack_int4(packed[None, :])[0], q)
    w, _, gs = int4_inputs("a")
    packed, scales = quantize_int4_groupwise(w, gs)
    assert np.all(np.isfinite(scales.astype(np.float32))) and scales[0, 0] > 0
    assert np.all(unpack_int4(packed)[0, :gs] == 0)
    assert unpack_int4(packed)[1, 3] == 7
    assert int4_weight_bytes(3072, 3072) == 3072 * 1536 + 3072 * 24 * 2
