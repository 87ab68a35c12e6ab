"""INT4 / FP16 projections on B200 — drop-in for the reference ``kernels/matmul.py``.

Same public functions, argument meaning and return conventions as the reference
(``int4_matmul`` at :217-231, ``dequantize_all`` at :236-266, ``fuse_qkv_inplace`` at
:269-306, ``_dequant_storage`` at :309-326), so ``model.py`` and ``kernels/mlp.py``
call this module unchanged.

* ``int4_matmul(x, (packed, scales), groupsize)`` — the reference's memory mode
  (its default, model.py:15-21): for up to 64 rows of ``x`` (decode) one launch of
  the fused sm_100a dequant-matmul ``fi_int4_gemm``, which streams the 4-bit weights
  once from HBM; for more rows (prefill) the weights are dequantized bit-exactly by
  ``fi_int4_dequant`` and multiplied by the dense library GEMM.
* ``int4_matmul(x, w_fp16)`` — the reference's speed mode: the dense library GEMM.
* ``_dequant_storage`` / ``dequantize_all`` — the speed-mode weight preparation,
  dequantized on the GPU by ``fi_int4_dequant`` (bit-identical to the reference).

CPU tensors are rejected: there is no CPU path.
"""

from __future__ import annotations

import torch

from fast_infer_b200 import _lib
from fast_infer_b200._runtime import device_errors, error_word, stream_of, with_device

FUSED_MAX_M = 64


def _check_int4(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, groupsize: int):
    for name, t in (("x", x), ("packed", packed), ("scales", scales)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (fast_infer_b200 has no CPU path)")
    if packed.dtype not in (torch.int8, torch.uint8):
        raise TypeError(f"packed must be int8, got {packed.dtype}")
    if scales.dtype != torch.float16:
        raise TypeError(f"scales must be float16, got {scales.dtype}")
    if packed.dim() != 2 or scales.dim() != 2 or scales.shape[0] != packed.shape[0]:
        raise ValueError("expected packed [N, K/2] and scales [N, K/groupsize]")
    if x.device != packed.device or scales.device != packed.device:
        raise ValueError("all tensors must be on the same device")
    K = x.shape[-1]
    # The reference asserts these two (kernels/matmul.py:107-108).
    assert K % groupsize == 0, f"K ({K}) must be multiple of groupsize ({groupsize})"
    assert packed.shape[1] == K // 2, f"Weight packed dim mismatch: {packed.shape[1]} != {K // 2}"
    if scales.shape[1] != K // groupsize:
        raise ValueError(f"scales must have K/groupsize = {K // groupsize} columns")


def _fused_int4_matmul(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                       groupsize: int = 128) -> torch.Tensor:
    """C = x @ dequant(packed, scales).T, fp16 [..., N] (reference kernels/matmul.py:99-132)."""
    _check_int4(x, packed, scales, groupsize)
    orig_shape = x.shape
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float16:
        x2 = x2.to(torch.float16)
    M, K = x2.shape
    N = packed.shape[0]
    if M > FUSED_MAX_M:
        w = _dequant_storage(packed, scales, groupsize)
        return torch.matmul(x2, w.t()).reshape(*orig_shape[:-1], N)
    if x2.stride(1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    if packed.stride(1) != 1 or packed.stride(0) % 16 != 0 or packed.data_ptr() % 16 != 0:
        packed = packed.contiguous()
    c = torch.empty(M, N, dtype=torch.float16, device=x.device)
    if M == 0 or N == 0:
        return c.reshape(*orig_shape[:-1], N)
    lib = _lib.load()
    with with_device(x.device):
        err = error_word(x.device)
        st = lib.fi_int4_gemm(
            x2.data_ptr(), packed.data_ptr(), scales.data_ptr(), c.data_ptr(), M, N, K,
            int(groupsize), _lib.strides(*x2.stride()), _lib.strides(*packed.stride()),
            _lib.strides(*scales.stride()), _lib.strides(*c.stride()),
            err.data_ptr() if err is not None else None, stream_of(x.device))
        _lib.check(st, "int4_matmul")
        device_errors(err, "int4_matmul")
    return c.reshape(*orig_shape[:-1], N)


def _fp16_matmul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w.T with fp16 weights [N, K] (reference kernels/matmul.py:187-212)."""
    if not x.is_cuda or not w.is_cuda:
        raise ValueError("x and w must be CUDA tensors (fast_infer_b200 has no CPU path)")
    orig_shape = x.shape
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != w.dtype:
        x2 = x2.to(w.dtype)
    return torch.matmul(x2, w.t()).reshape(*orig_shape[:-1], w.shape[0])


def int4_matmul(x: torch.Tensor, w, scales=None, groupsize: int = 128) -> torch.Tensor:
    """fp16 input x weight -> fp16 [..., N].

    ``w`` is either an fp16 [N, K] tensor (speed mode, already dequantized) or a
    ``(packed_int8, scales)`` tuple (memory mode, fused dequant-matmul).
    """
    if isinstance(w, tuple):
        packed, sc = w
        return _fused_int4_matmul(x, packed, sc, groupsize)
    return _fp16_matmul(x, w)


def _dequant_storage(packed: torch.Tensor, scales: torch.Tensor,
                     groupsize: int = 128) -> torch.Tensor:
    """INT4 weights -> fp16 [N, K], bit-identical to the reference's storage dequant."""
    if not packed.is_cuda or not scales.is_cuda:
        raise ValueError("packed and scales must be CUDA tensors (fast_infer_b200 has no CPU path)")
    if scales.dtype != torch.float16:
        raise TypeError(f"scales must be float16, got {scales.dtype}")
    N, K_half = packed.shape
    K = K_half * 2
    if K % groupsize != 0 or scales.shape != (N, K // groupsize):
        raise ValueError("expected packed [N, K/2] and scales [N, K/groupsize]")
    if packed.stride(1) != 1 or packed.stride(0) % 4 != 0 or packed.data_ptr() % 4 != 0:
        packed = packed.contiguous()
    out = torch.empty(N, K, dtype=torch.float16, device=packed.device)
    if N == 0:
        return out
    lib = _lib.load()
    with with_device(packed.device):
        st = lib.fi_int4_dequant(packed.data_ptr(), scales.data_ptr(), out.data_ptr(), N, K,
                                 int(groupsize), _lib.strides(*packed.stride()),
                                 _lib.strides(*scales.stride()), _lib.strides(*out.stride()),
                                 stream_of(packed.device))
        _lib.check(st, "_dequant_storage")
    return out


def dequantize_all(weights: dict) -> dict:
    """Speed mode: dequantize every INT4 projection of every layer to fp16 and fuse
    q/k/v into ``qkv_proj`` and gate/up into ``gate_up_proj`` (same dict layout as the
    reference produces)."""
    for layer in weights["layers"]:
        sa, mlp = layer["self_attn"], layer["mlp"]
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            if isinstance(sa.get(name), tuple):
                sa[name] = _dequant_storage(*sa[name])
        for name in ("gate_proj", "up_proj", "down_proj"):
            if isinstance(mlp.get(name), tuple):
                mlp[name] = _dequant_storage(*mlp[name])
        sa["qkv_proj"] = torch.cat([sa.pop("q_proj"), sa.pop("k_proj"), sa.pop("v_proj")], dim=0)
        mlp["gate_up_proj"] = torch.cat([mlp.pop("gate_proj"), mlp.pop("up_proj")], dim=0)
    torch.cuda.empty_cache()
    return weights


def fuse_qkv_inplace(weights: dict):
    """Concatenate q/k/v and gate/up projections (INT4 tuples or fp16 tensors) so each
    layer runs one projection launch for each group."""
    def cat(parts):
        if isinstance(parts[0], tuple):
            return (torch.cat([p[0] for p in parts], dim=0), torch.cat([p[1] for p in parts], dim=0))
        return torch.cat(parts, dim=0)

    for layer in weights["layers"]:
        sa, mlp = layer["self_attn"], layer["mlp"]
        if "qkv_proj" not in sa:
            sa["qkv_proj"] = cat([sa.pop("q_proj"), sa.pop("k_proj"), sa.pop("v_proj")])
        if "gate_up_proj" not in mlp:
            mlp["gate_up_proj"] = cat([mlp.pop("gate_proj"), mlp.pop("up_proj")])
