"""FlashAttention (prefill) and paged attention (decode) on B200 — drop-in module.

Same functions, argument meaning and return conventions as the reference
``kernels/attention.py`` (``flash_attention`` at :80-113, ``paged_attention`` at
:191-233), so ``model.py`` calls this module unchanged. The work runs in the
sm_100a CUDA library (``libfast_infer_b200.so``) reached through its C ABI; there
is no Triton and no CPU path — CPU tensors are rejected.

Backward-compatible extensions:
* ``flash_attention`` also accepts un-expanded GQA K/V (``k.shape[1]`` dividing
  ``q.shape[1]``), so callers can drop the ``repeat_interleave`` of model.py:110-111.
* ``paged_attention`` takes optional per-sequence ``context_lens`` (ragged
  batches) and ``pages_per_split`` (split-KV tuning).
"""

from __future__ import annotations

import torch

from fast_infer_b200 import _lib
from fast_infer_b200._runtime import (device_errors, error_word, stream_of, with_device)

HEAD_DIM = 128
BLOCK_SIZE = 64


def _check_cuda_f16(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (fast_infer_b200 has no CPU path)")
    if t.dtype != torch.float16:
        raise TypeError(f"{name} must be float16, got {t.dtype}")


def _tma_ready(t: torch.Tensor) -> bool:
    """True if the tensor can be addressed by a TMA map as is: 16-byte aligned base,
    unit innermost stride, every other stride a multiple of 8 elements."""
    if t.data_ptr() % 16 != 0 or t.stride(-1) != 1:
        return False
    return all(s % 8 == 0 or n == 1 for s, n in zip(t.stride()[:-1], t.shape[:-1]))


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    sm_scale: float = None) -> torch.Tensor:
    """Causal FlashAttention for the prefill phase.

    q: [batch, num_heads, seq_len, head_dim] fp16 (any strides, e.g. the BHSD view of
    BSHD memory that model.py passes); k, v: [batch, num_kv_heads, seq_len, head_dim]
    with num_kv_heads == num_heads (expanded, as the reference caller passes them) or
    dividing num_heads (GQA, no expansion needed).
    Returns a tensor shaped and strided like ``torch.empty_like(q)``
    (reference attention.py:99).
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda_f16(name, t)
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4-D [batch, heads, seq_len, head_dim]")
    batch, num_heads, seq_len, head_dim = q.shape
    if head_dim != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM}, got {head_dim}")
    if k.shape != v.shape or k.shape[0] != batch or k.shape[2] != seq_len or k.shape[3] != head_dim:
        raise ValueError(f"k/v shape {tuple(k.shape)}/{tuple(v.shape)} incompatible with q {tuple(q.shape)}")
    num_kv_heads = k.shape[1]
    if num_kv_heads == 0 or num_heads % num_kv_heads != 0:
        raise ValueError(f"num_heads {num_heads} not a multiple of k/v heads {num_kv_heads}")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on the same device")
    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    o = torch.empty_like(q)
    if q.numel() == 0:
        return o
    qx = q if _tma_ready(q) else q.contiguous()
    kx = k if _tma_ready(k) else k.contiguous()
    vx = v if _tma_ready(v) else v.contiguous()
    ox = o if _tma_ready(o) else torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lib = _lib.load()
    with with_device(q.device):
        err = error_word(q.device)
        st = lib.fi_prefill_fwd(
            qx.data_ptr(), kx.data_ptr(), vx.data_ptr(), ox.data_ptr(),
            batch, num_heads, num_kv_heads, seq_len, head_dim,
            _lib.strides(*qx.stride()), _lib.strides(*kx.stride()),
            _lib.strides(*vx.stride()), _lib.strides(*ox.stride()),
            float(sm_scale), err.data_ptr() if err is not None else None, stream_of(q.device))
        _lib.check(st, "flash_attention")
        device_errors(err, "flash_attention")
    if ox is not o:
        o.copy_(ox)
    return o


def flash_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           cu_seqlens: torch.Tensor, max_seqlen: int,
                           sm_scale: float = None) -> torch.Tensor:
    """Causal prefill over a ragged batch packed along the token axis (extension; the
    reference's ``flash_attention`` takes one shared sequence length).

    q: [total_tokens, num_heads, 128] fp16; k, v: [total_tokens, num_kv_heads, 128];
    sequence b owns tokens [cu_seqlens[b], cu_seqlens[b+1]) (int32 on the device);
    max_seqlen (host int) bounds the lengths. Returns o shaped like q.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda_f16(name, t)
        if t.dim() != 3 or t.shape[-1] != HEAD_DIM:
            raise ValueError(f"{name} must be [total_tokens, heads, {HEAD_DIM}]")
    total, num_heads, head_dim = q.shape
    if k.shape != v.shape or k.shape[0] != total:
        raise ValueError("k/v must be [total_tokens, num_kv_heads, head_dim] like q")
    num_kv_heads = k.shape[1]
    if num_heads % num_kv_heads != 0:
        raise ValueError(f"num_heads {num_heads} not a multiple of k/v heads {num_kv_heads}")
    if cu_seqlens.dim() != 1 or cu_seqlens.device != q.device:
        raise ValueError("cu_seqlens must be a 1-D int32 tensor on q's device")
    cu = cu_seqlens.to(torch.int32).contiguous()
    batch = cu.numel() - 1
    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    o = torch.empty_like(q)
    if batch <= 0 or total == 0:
        return o
    qx = q if _tma_ready(q) else q.contiguous()
    kx = k if _tma_ready(k) else k.contiguous()
    vx = v if _tma_ready(v) else v.contiguous()
    ox = o if _tma_ready(o) else torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lib = _lib.load()
    with with_device(q.device):
        err = error_word(q.device)
        st = lib.fi_prefill_fwd_varlen(
            qx.data_ptr(), kx.data_ptr(), vx.data_ptr(), ox.data_ptr(), cu.data_ptr(), batch,
            num_heads, num_kv_heads, int(max_seqlen), total, head_dim,
            _lib.strides(*qx.stride()), _lib.strides(*kx.stride()),
            _lib.strides(*vx.stride()), _lib.strides(*ox.stride()), float(sm_scale),
            err.data_ptr() if err is not None else None, stream_of(q.device))
        _lib.check(st, "flash_attention_varlen")
        device_errors(err, "flash_attention_varlen")
    if ox is not o:
        o.copy_(ox)
    return o


def paged_attention_workspace_bytes(batch: int, num_q_heads: int, num_kv_heads: int,
                                    max_context_len: int, pages_per_split: int = 0) -> int:
    """Split-KV workspace bytes ``paged_attention`` needs for these sizes."""
    return int(_lib.load().fi_paged_decode_workspace_size(
        batch, num_q_heads, num_kv_heads, HEAD_DIM, max_context_len, BLOCK_SIZE, pages_per_split))


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_table: torch.Tensor, block_size: int,
                    num_tokens: int,
                    sm_scale: float = None, *,
                    context_lens: torch.Tensor = None,
                    max_context_len: int = None,
                    pages_per_split: int = 0,
                    workspace: torch.Tensor = None) -> torch.Tensor:
    """PagedAttention for the decode phase (one query token per sequence).

    q: [batch, num_q_heads, head_dim] fp16; k_cache, v_cache: [num_blocks, block_size,
    num_kv_heads, head_dim] fp16 (one layer of ``KVCache.k`` / ``.v``); block_table:
    [>= batch, max_blocks_per_seq] int32 with -1 for unused slots; num_tokens: valid
    tokens of every sequence (reference semantics; 0 returns zeros). Pass
    ``context_lens`` ([batch] int32 on the device) for per-sequence lengths instead;
    ``max_context_len`` (host int) then bounds them (default: the block table's span,
    which needs no device sync). ``workspace`` optionally supplies the split-KV
    scratch (uint8, at least ``paged_attention_workspace_bytes`` bytes).
    Returns [batch, num_q_heads, head_dim] fp16 like ``torch.empty_like(q)``.
    """
    if context_lens is None and num_tokens == 0:
        return torch.zeros_like(q)
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check_cuda_f16(name, t)
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("expected q [B, Hq, D] and k_cache/v_cache [NB, block_size, Hkv, D]")
    batch, num_q_heads, head_dim = q.shape
    num_blocks, bs, num_kv_heads, d2 = k_cache.shape
    if head_dim != HEAD_DIM or d2 != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM}")
    if block_size != bs or bs != BLOCK_SIZE:
        raise ValueError(f"block_size must be {BLOCK_SIZE} and match k_cache.shape[1]")
    if block_table.dim() != 2 or block_table.shape[0] < batch:
        raise ValueError("block_table must be [>= batch, max_blocks_per_seq]")
    if block_table.device != q.device or k_cache.device != q.device:
        raise ValueError("all tensors must be on the same device")
    if block_table.dtype != torch.int32:
        block_table = block_table.to(torch.int32)
    max_blocks = block_table.shape[1]
    if context_lens is not None:
        if context_lens.dtype != torch.int32:
            context_lens = context_lens.to(torch.int32)
        if context_lens.device != q.device or context_lens.numel() < batch:
            raise ValueError("context_lens must be a [batch] int32 tensor on q's device")
        context_lens = context_lens.contiguous()
        if max_context_len is None:
            max_context_len = max_blocks * block_size
        ntok = 0
    else:
        if num_tokens < 0 or (num_tokens + block_size - 1) // block_size > max_blocks:
            raise ValueError(f"num_tokens {num_tokens} does not fit the block table")
        ntok = int(num_tokens)
        max_context_len = ntok
    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    o = torch.empty_like(q)
    if batch == 0:
        return o
    lib = _lib.load()
    need = int(lib.fi_paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                  max_context_len, block_size, pages_per_split))
    if need > 0:
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    with with_device(q.device):
        err = error_word(q.device)
        st = lib.fi_paged_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(),
            block_table.data_ptr(),
            context_lens.data_ptr() if context_lens is not None else None,
            ntok, int(max_context_len), batch, num_q_heads, num_kv_heads, head_dim,
            num_blocks, block_size, max_blocks,
            _lib.strides(*q.stride()), _lib.strides(*k_cache.stride()),
            _lib.strides(*v_cache.stride()), _lib.strides(*o.stride()),
            _lib.strides(*block_table.stride()), float(sm_scale), int(pages_per_split),
            workspace.data_ptr() if need > 0 else None, need,
            err.data_ptr() if err is not None else None, stream_of(q.device))
        _lib.check(st, "paged_attention")
        device_errors(err, "paged_attention")
    return o
