"""CPU oracle for the reference's INT4 weight path (TEST INFRASTRUCTURE ONLY).

Restates in numpy the reference's group-wise INT4 weight format and its fused
dequant-matmul:

* ``quantize_int4_groupwise``  reference loader.py:9-41 (symmetric, per-group
  scale = max|w| / 7, round half-to-even, clamp to [-8, 7], two nibbles per byte:
  element 2j in the low nibble, 2j+1 in the high nibble, two's complement)
* ``dequantize_int4``          reference loader.py:157-190 and
                               kernels/matmul.py:309-326 (``_dequant_storage``):
  w = fp16(fp32(q) * fp32(scale))
* ``int4_matmul``              reference kernels/matmul.py:14-132: C = x @ dequant(W)^T
  with fp16 inputs, fp32 accumulation, fp16 output.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import
this file; the CUDA library never calls it. Pinned against the reference's own
functions by ``tests/golden/int4.npz`` (``tests/golden/make_golden.py``): the
quantizer and dequantizer bit for bit, the matmul within its floating-point
tolerance (the reference's interpreter run and this restatement sum in different
orders).
"""

from __future__ import annotations

import numpy as np

GROUPSIZE_DEFAULT = 128


def quantize_int4_groupwise(w: np.ndarray, groupsize: int = GROUPSIZE_DEFAULT):
    """fp16 [N, K] -> (packed int8 [N, K/2], scales fp16 [N, K/groupsize]).

    Every step is an fp16 tensor op in the reference (max, clamp, divide by 7,
    divide, round); numpy's float16 arithmetic rounds each result to fp16 the same
    way (loader.py:19-41).
    """
    w = np.asarray(w, np.float16)
    n, k = w.shape
    assert k % groupsize == 0 and groupsize % 2 == 0
    g = w.reshape(n, k // groupsize, groupsize)
    w_max = np.abs(g).max(axis=-1, keepdims=True)
    w_max = np.maximum(w_max, np.float16(1e-6))
    scale = (w_max / np.float16(7.0)).astype(np.float16)
    q = np.round(g / scale).astype(np.float16)          # half-to-even, like torch.round
    q = np.clip(q, -8, 7).astype(np.int8)
    q = q.reshape(n, k // 2, 2)
    packed = ((q[..., 0] & 0xF) | ((q[..., 1] & 0xF) << 4)).astype(np.uint8).view(np.int8)
    return packed.reshape(n, k // 2), scale.reshape(n, k // groupsize).astype(np.float16)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """int8 [N, K/2] -> int8 [N, K] signed values in [-8, 7] (low nibble first)."""
    p = np.asarray(packed).view(np.uint8).astype(np.int16)
    lo = p & 0xF
    hi = (p >> 4) & 0xF
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    n, kh = p.shape
    return np.stack([lo, hi], axis=-1).reshape(n, 2 * kh).astype(np.int8)


def dequantize_int4(packed: np.ndarray, scales: np.ndarray,
                    groupsize: int = GROUPSIZE_DEFAULT) -> np.ndarray:
    """fp16 [N, K] = fp16(fp32(q) * fp32(scale)), the reference's storage dequant."""
    q = unpack_int4(packed).astype(np.float32)
    n, k = q.shape
    s = np.asarray(scales, np.float16).astype(np.float32)
    w = q.reshape(n, k // groupsize, groupsize) * s[:, :, None]
    return w.reshape(n, k).astype(np.float16)


def int4_matmul(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
                groupsize: int = GROUPSIZE_DEFAULT) -> np.ndarray:
    """[..., K] fp16 x (packed, scales) -> [..., N] fp16, fp32 accumulation.

    The reference kernel dequantizes each weight to fp16 (``(w * scale).to(fp16)``,
    kernels/matmul.py:87-88), multiplies fp16 x fp16 and accumulates in fp32.
    """
    w = dequantize_int4(packed, scales, groupsize).astype(np.float64)
    xs = np.asarray(x, np.float16)
    x2 = xs.reshape(-1, xs.shape[-1]).astype(np.float64)
    c = (x2 @ w.T).astype(np.float32)
    return c.astype(np.float16).reshape(*xs.shape[:-1], w.shape[0])


def int4_weight_bytes(n: int, k: int, groupsize: int = GROUPSIZE_DEFAULT) -> int:
    """Bytes one dequant-matmul must read for its weight: nibbles plus fp16 scales."""
    return n * k // 2 + n * (k // groupsize) * 2
