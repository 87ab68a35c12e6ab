"""CPU oracle for the reference's RMSNorm (TEST INFRASTRUCTURE ONLY).

Restates reference kernels/rms_norm.py:8-43 in numpy: x upcast to fp32,
mean of squares over the row, rsqrt(mean + eps), (x * rms) * weight in fp32, rounded
to fp16. Only ``tests/`` may import this file; the CUDA library never calls it.
Pinned against ``tests/golden/rms_norm.npz`` (the reference's Triton kernel run under
TRITON_INTERPRET=1 by ``tests/golden/make_golden.py``) within fp16 rounding: the sum
order and the reciprocal square root differ between implementations.
"""

from __future__ import annotations

import numpy as np


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    xf = np.asarray(x, np.float16).astype(np.float32)
    ms = (xf * xf).sum(axis=-1, keepdims=True, dtype=np.float32) / np.float32(xf.shape[-1])
    rms = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    w = np.asarray(weight, np.float16).astype(np.float32)
    return ((xf * rms) * w).astype(np.float16)
