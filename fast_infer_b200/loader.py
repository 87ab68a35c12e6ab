"""INT4 weight format on B200 — the quantize / dequantize half of the reference
``loader.py`` (``quantize_int4_groupwise`` at :9-41, ``dequantize_int4`` at :157-190),
with the same names, arguments and results.

Both run as sm_100a kernels through the C ABI (``fi_int4_quantize``,
``fi_int4_dequant``) and are bit-identical to the reference's fp16 tensor ops.
Reading checkpoints (safetensors) is outside this library's scope.
"""

from __future__ import annotations

import torch

from fast_infer_b200 import _lib
from fast_infer_b200._runtime import stream_of, with_device
from fast_infer_b200.kernels.matmul import _dequant_storage


def quantize_int4_groupwise(w: torch.Tensor, groupsize: int = 128):
    """fp16 [out_features, in_features] on the GPU -> (packed int8 [out, in/2],
    scales fp16 [out, in/groupsize]), symmetric per group (max|w| / 7)."""
    if not isinstance(w, torch.Tensor) or not w.is_cuda:
        raise ValueError("w must be a CUDA tensor (fast_infer_b200 has no CPU path)")
    if w.dim() != 2:
        raise ValueError("w must be 2-D [out_features, in_features]")
    if w.dtype != torch.float16:
        w = w.to(torch.float16)
    n, k = w.shape
    if k % groupsize != 0 or groupsize % 2 != 0:
        raise ValueError(f"in_features ({k}) must be a multiple of an even groupsize ({groupsize})")
    packed = torch.empty(n, k // 2, dtype=torch.int8, device=w.device)
    scales = torch.empty(n, k // groupsize, dtype=torch.float16, device=w.device)
    if n == 0:
        return packed, scales
    lib = _lib.load()
    with with_device(w.device):
        st = lib.fi_int4_quantize(w.data_ptr(), packed.data_ptr(), scales.data_ptr(), n, k,
                                  int(groupsize), _lib.strides(*w.stride()),
                                  _lib.strides(*packed.stride()), _lib.strides(*scales.stride()),
                                  stream_of(w.device))
        _lib.check(st, "quantize_int4_groupwise")
    return packed, scales


def dequantize_int4(packed: torch.Tensor, scales: torch.Tensor,
                    groupsize: int = 128) -> torch.Tensor:
    """INT4 weights -> fp16 [out_features, in_features] (fp16(q * scale))."""
    return _dequant_storage(packed, scales, groupsize)
