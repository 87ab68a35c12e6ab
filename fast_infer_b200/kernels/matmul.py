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


# fi_small_gemm handles up to 16 rows. With the exact RMSNorm prologue (x staged and
# normalised by every CTA) it beats the library GEMM + RMSNorm launch up to 8 rows
# and loses at 16 (QKV: 14.6 vs 12.3 us); without a norm x streams in by TMA with the
# weight tiles (two CTAs per SM).
SMALL_GEMM_MAX_M = 8
STREAM_GEMM_MAX_M = 16


def fp16_linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor = None,
                norm_weight: torch.Tensor = None, eps: float = 1e-5,
                out: torch.Tensor = None, static_weight: bool = False) -> torch.Tensor:
    """``residual + rms_norm(x, norm_weight, eps) @ w.T`` in fp16 (fp32 accumulation).

    x [..., K], w [N, K] fp16 (the reference's linear layout, kernels/matmul.py:187-212);
    residual [..., N] or None; norm_weight [K] or None (no norm). Up to 16 rows of x
    take one ``fi_small_gemm`` launch (norm on load, residual in the epilogue, a single
    rounding) up to ``SMALL_GEMM_MAX_M`` rows; more rows use ``rms_norm`` and the dense
    library GEMM with the residual as its beta = 1 input. ``out`` (may be
    ``residual``) receives the result. ``static_weight``: ``w`` is constant (model
    weights, not written by kernels still running), so the kernel's first weight tiles
    load while the previous kernel finishes (``FI_STATIC_WEIGHTS``; same result bits).
    """
    if not x.is_cuda or not w.is_cuda:
        raise ValueError("x and w must be CUDA tensors (fast_infer_b200 has no CPU path)")
    if x.dtype != torch.float16 or w.dtype != torch.float16:
        raise TypeError("fp16_linear expects float16 x and w")
    K = x.shape[-1]
    if w.dim() != 2 or w.shape[1] != K:
        raise ValueError(f"w must be [N, {K}]")
    N = w.shape[0]
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    r2 = residual.reshape(-1, N) if residual is not None else None
    if r2 is not None and r2.shape[0] != M:
        raise ValueError("residual must be [..., N] with x's leading shape")
    if out is None:
        out = torch.empty(*lead, N, dtype=torch.float16, device=x.device)
    o2 = out.view(-1, N)
    limit = SMALL_GEMM_MAX_M if norm_weight is not None else STREAM_GEMM_MAX_M
    if M <= limit and K % 64 == 0 and M > 0 and N > 0:
        if x2.stride(1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
            x2 = x2.contiguous()
        flags = _lib.FI_STATIC_WEIGHTS if static_weight else 0
        if w.stride(1) != 1 or w.stride(0) % 8 != 0 or w.data_ptr() % 16 != 0:
            w, flags = w.contiguous(), 0  # a fresh copy is the previous kernel's output
        nw = norm_weight
        if nw is not None and (not nw.is_contiguous() or nw.data_ptr() % 16 != 0):
            nw = nw.contiguous()
        lib = _lib.load()
        with with_device(x.device):
            err = error_word(x.device)
            st = lib.fi_small_gemm(
                x2.data_ptr(), w.data_ptr(), o2.data_ptr(),
                r2.data_ptr() if r2 is not None else None,
                nw.data_ptr() if nw is not None else None, float(eps), M, N, K,
                _lib.strides(*x2.stride()), _lib.strides(*w.stride()),
                _lib.strides(*o2.stride()),
                _lib.strides(*r2.stride()) if r2 is not None else None, flags,
                err.data_ptr() if err is not None else None, stream_of(x.device))
            _lib.check(st, "fp16_linear")
            device_errors(err, "fp16_linear")
        return out
    from fast_infer_b200.kernels.rms_norm import rms_norm
    h = rms_norm(x2, norm_weight, eps) if norm_weight is not None else x2
    if r2 is not None:
        torch.addmm(r2, h, w.t(), out=o2) if o2.data_ptr() != r2.data_ptr() else o2.addmm_(h, w.t())
    else:
        torch.matmul(h, w.t(), out=o2)
    return out


def fold_rms_weight(w: torch.Tensor, norm_weight: torch.Tensor) -> torch.Tensor:
    """w [N, K] with the RMSNorm weight folded in: fp16(w[n, k] * norm_weight[k]) (for
    ``fp16_linear_folded``; prepared once per weight)."""
    return (w.float() * norm_weight.float()[None, :]).half().contiguous()


def fp16_linear_folded(x: torch.Tensor, w_folded: torch.Tensor, eps: float = 1e-5,
                       residual: torch.Tensor = None, out: torch.Tensor = None,
                       static_weight: bool = False) -> torch.Tensor:
    """``residual + rsqrt(mean(x^2) + eps) * (x @ w_folded.T)`` = rms_norm(x) @ w.T with
    the norm weight folded into ``w_folded`` (``fold_rms_weight``). Up to 16 rows: one
    ``fi_small_gemm_folded`` launch (x streamed with the weight tiles, the per-row
    factor applied in the epilogue); the rounding differs from the reference's
    normalised-then-rounded x by fp16 noise. More rows: the same formula with library
    ops. ``static_weight`` as in ``fp16_linear``."""
    if not x.is_cuda or not w_folded.is_cuda:
        raise ValueError("x and w must be CUDA tensors (fast_infer_b200 has no CPU path)")
    if x.dtype != torch.float16 or w_folded.dtype != torch.float16:
        raise TypeError("fp16_linear_folded expects float16 x and w")
    K = x.shape[-1]
    if w_folded.dim() != 2 or w_folded.shape[1] != K:
        raise ValueError(f"w_folded must be [N, {K}]")
    N = w_folded.shape[0]
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    r2 = residual.reshape(-1, N) if residual is not None else None
    if out is None:
        out = torch.empty(*lead, N, dtype=torch.float16, device=x.device)
    o2 = out.view(-1, N)
    if 0 < M <= STREAM_GEMM_MAX_M and K % 64 == 0 and N > 0:
        if x2.stride(1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
            x2 = x2.contiguous()
        w = w_folded
        flags = _lib.FI_STATIC_WEIGHTS if static_weight else 0
        if w.stride(1) != 1 or w.stride(0) % 8 != 0 or w.data_ptr() % 16 != 0:
            w, flags = w.contiguous(), 0  # a fresh copy is the previous kernel's output
        lib = _lib.load()
        with with_device(x.device):
            err = error_word(x.device)
            st = lib.fi_small_gemm_folded(
                x2.data_ptr(), w.data_ptr(), o2.data_ptr(),
                r2.data_ptr() if r2 is not None else None, float(eps), M, N, K,
                _lib.strides(*x2.stride()), _lib.strides(*w.stride()),
                _lib.strides(*o2.stride()),
                _lib.strides(*r2.stride()) if r2 is not None else None, flags,
                err.data_ptr() if err is not None else None, stream_of(x.device))
            _lib.check(st, "fp16_linear_folded")
            device_errors(err, "fp16_linear_folded")
        return out
    xf = x2.float()
    y = (xf @ w_folded.float().t()) * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if r2 is not None:
        y = y + r2.float()
    o2.copy_(y.half())
    return out
