"""RMSNorm on B200 — drop-in for the reference ``kernels/rms_norm.py`` (``rms_norm`` at
:29-43): same name, arguments and result, one launch of ``fi_rms_norm`` (one warp per
row, fp32 sum of squares, ``x * rsqrt(mean(x^2) + eps) * weight`` in the reference's
order, fp16 out). CPU tensors are rejected: there is no CPU path.
"""

from __future__ import annotations

import torch

from fast_infer_b200 import _lib
from fast_infer_b200._runtime import stream_of, with_device


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """x: [..., hidden] fp16, weight: [hidden] fp16 -> [..., hidden] fp16."""
    if not x.is_cuda or not weight.is_cuda:
        raise ValueError("x and weight must be CUDA tensors (fast_infer_b200 has no CPU path)")
    if x.dtype != torch.float16 or weight.dtype != torch.float16:
        raise TypeError("rms_norm expects float16 x and weight")
    hidden = x.shape[-1]
    if weight.shape != (hidden,):
        raise ValueError(f"weight must be [{hidden}]")
    x2 = x.reshape(-1, hidden)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    w = weight if weight.is_contiguous() and weight.data_ptr() % 16 == 0 else weight.contiguous()
    out = torch.empty(x2.shape, dtype=torch.float16, device=x.device)
    if x2.shape[0] == 0:
        return out.reshape(x.shape)
    lib = _lib.load()
    with with_device(x.device):
        st = lib.fi_rms_norm(x2.data_ptr(), w.data_ptr(), out.data_ptr(), x2.shape[0], hidden,
                             x2.stride(0), out.stride(0), float(eps), stream_of(x.device))
        _lib.check(st, "rms_norm")
    return out.reshape(x.shape)
