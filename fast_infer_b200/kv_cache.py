"""Block-based paged KV cache — drop-in for the reference ``kv_cache.py``.

Layout, allocation order and method semantics are those of the reference
(kv_cache.py:6-113): pools ``k``, ``v`` of shape [num_layers, num_blocks,
block_size, num_heads, head_dim] fp16, zero-initialised; ``block_table``
[batch, max_blocks_per_seq] int32 on the device with -1 for unallocated slots;
a FIFO free list; ``alloc_block`` fills the first -1 slot of the row.

What changes is how it runs:
* The block table is mirrored on the host (numpy), so allocation never reads the
  device (the reference's ``.item()`` / ``nonzero`` syncs, kv_cache.py:57-60,75,92);
  dirty rows are uploaded once per write call.
* Every slot write — ``store``, ``store_batch``, and the model-level
  ``store_kv_prefill`` / ``store_kv_decode`` (model.py:162-201) — is one launch of
  the CUDA slot-write kernel for all sequences, blocks, heads and both K and V,
  instead of one torch copy plus one host sync per (sequence, block).

Extension: ``num_blocks`` may be given explicitly to size the pool independently
of ``max_seq_len`` (the reference pool holds ceil(max_seq_len/block_size) blocks
shared by the whole batch).
"""

from __future__ import annotations

import numpy as np
import torch

from fast_infer_b200 import _lib
from fast_infer_b200._runtime import device_errors, error_word, stream_of, with_device


class KVCache:
    """Paged KV cache for a batch of sequences (reference kv_cache.py:6-113)."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int,
                 max_seq_len: int, block_size: int, device: torch.device,
                 num_blocks: int = None):
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.block_size = block_size
        self.device = torch.device(device)
        self.max_blocks_per_seq = (max_seq_len + block_size - 1) // block_size
        self.num_blocks = self.max_blocks_per_seq if num_blocks is None else int(num_blocks)
        self.k = torch.zeros(num_layers, self.num_blocks, block_size, num_heads, head_dim,
                             dtype=torch.float16, device=self.device)
        self.v = torch.zeros(num_layers, self.num_blocks, block_size, num_heads, head_dim,
                             dtype=torch.float16, device=self.device)
        self._bt = np.full((1, self.max_blocks_per_seq), -1, np.int32)
        self.block_table = torch.full((1, self.max_blocks_per_seq), -1, dtype=torch.int32,
                                      device=self.device)
        self._dirty = False
        self.free_blocks = list(range(self.num_blocks))
        self._allocated = 0
        self.num_tokens = 0
        # Extension: per-sequence stored-token counts (the reference keeps only the
        # batch-wide num_tokens, kv_cache.py:39 / model.py:59,67-72).
        self.seq_lens = np.zeros(1, np.int64)

    # ------------------------------------------------------------ allocation
    def _grow_batch(self, batch_size: int):
        """Expand the block table for a larger batch (reference kv_cache.py:41-48)."""
        if batch_size <= self._bt.shape[0]:
            return
        nt = np.full((batch_size, self.max_blocks_per_seq), -1, np.int32)
        nt[: self._bt.shape[0]] = self._bt
        self._bt = nt
        sl = np.zeros(batch_size, np.int64)
        sl[: self.seq_lens.shape[0]] = self.seq_lens
        self.seq_lens = sl
        self.block_table = torch.from_numpy(nt.copy()).to(self.device)
        self._dirty = False

    def alloc_block(self, batch_idx: int = 0) -> int:
        """Allocate a physical block for a sequence; returns its logical index
        (reference kv_cache.py:50-63: FIFO free list, first free logical slot)."""
        if not self.free_blocks:
            raise RuntimeError("KV cache out of memory")
        row = self._bt[batch_idx]
        empty = np.flatnonzero(row == -1)
        if len(empty) == 0:
            raise RuntimeError("Sequence block table full")
        phys = self.free_blocks.pop(0)
        logical = int(empty[0])
        row[logical] = phys
        self._allocated += 1
        self._dirty = True
        return logical

    def _ensure_blocks(self, batch_idx: int, count: int):
        while int((self._bt[batch_idx] >= 0).sum()) < count:
            self.alloc_block(batch_idx)

    def sync_block_table(self):
        """Upload host-side allocations to ``block_table`` (stream-ordered)."""
        if self._dirty:
            if self.device.type == "cuda":
                with with_device(self.device):
                    self.block_table.copy_(torch.from_numpy(self._bt))
            else:
                self.block_table.copy_(torch.from_numpy(self._bt))
            self._dirty = False

    def pull_block_table(self):
        """Adopt edits made directly to the device ``block_table`` (synchronises)."""
        self._bt = self.block_table.cpu().numpy().astype(np.int32).copy()
        self._dirty = False

    def get_physical_blocks(self, batch_idx: int = 0) -> torch.Tensor:
        """Row of the block table for a sequence (reference kv_cache.py:65-67)."""
        self.sync_block_table()
        return self.block_table[batch_idx]

    def allocated_tokens(self, batch_idx: int = 0) -> int:
        """Upper bound of stored tokens (reference kv_cache.py:104-106)."""
        return self._allocated * self.block_size

    def reset(self):
        """Free all blocks (reference kv_cache.py:108-113)."""
        self._bt.fill(-1)
        self.block_table.fill_(-1)
        self._dirty = False
        self.free_blocks = list(range(self.num_blocks))
        self._allocated = 0
        self.num_tokens = 0
        self.seq_lens[:] = 0

    def context_lens(self, batch: int = None) -> torch.Tensor:
        """Per-sequence token counts as a device int32 tensor (for paged_attention)."""
        n = self.seq_lens.shape[0] if batch is None else batch
        return torch.from_numpy(self.seq_lens[:n].astype(np.int32)).to(self.device)

    # ------------------------------------------------------------ slot writes
    def write_tokens(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor,
                     start_pos, n_new: torch.Tensor = None):
        """Write k, v [B, T, H, D] at logical positions start_pos[b] + t of each
        sequence (start_pos: int or [B] int32 device tensor) — one kernel launch."""
        self.sync_block_table()
        if k.shape != v.shape or k.dim() != 4:
            raise ValueError("k, v must both be [batch, tokens, heads, head_dim]")
        B, T, H, D = k.shape
        if H != self.num_heads or D != self.head_dim:
            raise ValueError(f"k/v heads/dim {H}/{D} != cache {self.num_heads}/{self.head_dim}")
        if B > self.block_table.shape[0]:
            raise ValueError("batch larger than the block table; call _grow_batch first")
        for name, t in (("k", k), ("v", v)):
            if not t.is_cuda or t.dtype != torch.float16 or t.device != self.device:
                raise ValueError(f"{name} must be float16 on {self.device}")
        if B == 0 or T == 0:
            return
        kc, vc = self.k[layer_idx], self.v[layer_idx]
        if isinstance(start_pos, torch.Tensor):
            sp_ptr, sp_scalar = start_pos.to(torch.int32).contiguous(), 0
        else:
            sp_ptr, sp_scalar = None, int(start_pos)
        nn = n_new.to(torch.int32).contiguous() if n_new is not None else None
        lib = _lib.load()
        with with_device(self.device):
            err = error_word(self.device)
            st = lib.fi_kv_write(
                k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                self.block_table.data_ptr(),
                sp_ptr.data_ptr() if sp_ptr is not None else None, sp_scalar,
                nn.data_ptr() if nn is not None else None,
                B, T, H, D, self.num_blocks, self.block_size, self.max_blocks_per_seq,
                _lib.strides(*k.stride()), _lib.strides(*v.stride()),
                _lib.strides(*kc.stride()), _lib.strides(*vc.stride()),
                _lib.strides(*self.block_table.stride()),
                err.data_ptr() if err is not None else None, stream_of(self.device))
            _lib.check(st, "KVCache.write_tokens")
            device_errors(err, "KVCache.write_tokens")

    def store(self, layer_idx: int, logical_block: int, token_offset: int,
              k: torch.Tensor, v: torch.Tensor):
        """Store one token's K, V ([num_heads, head_dim]) of sequence 0
        (reference kv_cache.py:69-77)."""
        self.write_tokens(layer_idx, k[None, None], v[None, None],
                          logical_block * self.block_size + token_offset)

    def store_batch(self, layer_idx: int, start_block: int, start_offset: int,
                    k: torch.Tensor, v: torch.Tensor):
        """Store consecutive tokens ([num_tokens, num_heads, head_dim]) of sequence 0
        starting at (start_block, start_offset) (reference kv_cache.py:79-102)."""
        self.write_tokens(layer_idx, k[None], v[None],
                          start_block * self.block_size + start_offset)


def store_kv_prefill(cache: KVCache, layer_idx: int, k: torch.Tensor, v: torch.Tensor):
    """Prefill slot write of reference model.py:162-183.

    k, v: [batch, seq_len, num_kv_heads, head_dim]. At layer 0 sets
    ``cache.num_tokens = seq_len``; for each sequence (in order) allocates blocks
    until ceil(seq_len / block_size) are held, then writes tokens 0..seq_len-1.
    """
    B, S = k.shape[0], k.shape[1]
    bs = cache.block_size
    num_needed = (S + bs - 1) // bs
    if layer_idx == 0:
        cache.num_tokens = S
    cache._grow_batch(B)
    for b in range(B):
        cache._ensure_blocks(b, num_needed)
    cache.write_tokens(layer_idx, k, v, 0)


def store_kv_decode(cache: KVCache, layer_idx: int, k: torch.Tensor, v: torch.Tensor,
                    token_count: int):
    """Decode slot write of reference model.py:185-201.

    k, v: [batch, num_kv_heads, head_dim]; ``token_count`` is the model's position
    counter after the increment (the token is stored at position token_count - 1).
    At layer 0 increments ``cache.num_tokens``; allocates a block on crossing.
    """
    B = k.shape[0]
    pos = token_count - 1
    blk = pos // cache.block_size
    if layer_idx == 0:
        cache.num_tokens += 1
    cache._grow_batch(B)
    for b in range(B):
        cache._ensure_blocks(b, blk + 1)
    cache.write_tokens(layer_idx, k[:, None], v[:, None], pos)


def store_kv_ragged(cache: KVCache, layer_idx: int, k: torch.Tensor, v: torch.Tensor,
                    start_pos, n_new):
    """Per-sequence slot write (extension for ragged batches).

    k, v: [B, T, H, D] (rows past n_new[b] are padding); token t of sequence b is
    stored at position start_pos[b] + t for t < n_new[b]. Blocks are allocated on
    demand per sequence in batch order (the reference's first-free-slot / FIFO rule),
    and at layer 0 ``cache.seq_lens`` grows to cover the written positions.
    """
    start = np.asarray(start_pos, np.int64).reshape(-1)
    nn = np.asarray(n_new, np.int64).reshape(-1)
    B = k.shape[0]
    if start.shape[0] != B or nn.shape[0] != B:
        raise ValueError("start_pos and n_new need one entry per sequence")
    cache._grow_batch(B)
    bs = cache.block_size
    for b in range(B):
        if nn[b] > 0:
            cache._ensure_blocks(b, int((start[b] + nn[b] + bs - 1) // bs))
    if layer_idx == 0:
        cache.seq_lens[:B] = np.maximum(cache.seq_lens[:B], start + nn)
    dev = cache.device
    cache.write_tokens(layer_idx, k, v, torch.from_numpy(start.astype(np.int32)).to(dev),
                       torch.from_numpy(nn.astype(np.int32)).to(dev))


def rope_and_store(cache: KVCache, layer_idx: int, qkv: torch.Tensor, num_q_heads: int,
                   cos_table: torch.Tensor, sin_table: torch.Tensor, start_pos,
                   q_out: torch.Tensor = None, k_out: torch.Tensor = None) -> torch.Tensor:
    """Fused RoPE of q and k plus the KV slot write (one launch).

    Equivalent to the reference's ``apply_rope`` (kernels/rope.py:26-44, cos/sin rows
    cast to fp16 as model.py:74-75 does) followed by storing the rotated k and v at
    positions start_pos[b] + t (model.py:162-201), bit for bit.

    qkv: [B, S, (nq + 2*nkv) * D] fp16 projection output (q | k | v heads);
    cos_table / sin_table: fp32 [max_pos, D]; start_pos: int or [B] int32 device tensor.
    Returns rotated q [B, S, nq, D] (``q_out`` if given). If ``k_out`` ([B, S, nkv, D])
    is given, the rotated k is also written there.
    """
    cache.sync_block_table()
    if qkv.dim() != 3 or qkv.dtype != torch.float16 or qkv.device != cache.device:
        raise ValueError("qkv must be [batch, seq, heads*head_dim] float16 on the cache device")
    B, S, W = qkv.shape
    D, nkv = cache.head_dim, cache.num_heads
    if W != (num_q_heads + 2 * nkv) * D:
        raise ValueError(f"qkv width {W} != (nq + 2*nkv) * head_dim = {(num_q_heads + 2 * nkv) * D}")
    if B > cache.block_table.shape[0]:
        raise ValueError("batch larger than the block table; call _grow_batch first")
    for name, t in (("cos_table", cos_table), ("sin_table", sin_table)):
        if t.dtype != torch.float32 or t.device != cache.device or t.dim() != 2 or t.stride(1) != 1:
            raise ValueError(f"{name} must be a float32 [max_pos, head_dim] table on the device")
    if q_out is None:
        q_out = torch.empty(B, S, num_q_heads, D, dtype=torch.float16, device=cache.device)
    if isinstance(start_pos, torch.Tensor):
        sp, sp_scalar = start_pos.to(torch.int32).contiguous(), 0
    else:
        sp, sp_scalar = None, int(start_pos)
    kc, vc = cache.k[layer_idx], cache.v[layer_idx]
    lib = _lib.load()
    with with_device(cache.device):
        err = error_word(cache.device)
        st = lib.fi_rope_kv_write(
            qkv.data_ptr(), B, S, num_q_heads, nkv, D, _lib.strides(*qkv.stride()),
            cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], cos_table.stride(0),
            sp.data_ptr() if sp is not None else None, sp_scalar,
            q_out.data_ptr(), _lib.strides(*q_out.stride()),
            k_out.data_ptr() if k_out is not None else None,
            _lib.strides(*k_out.stride()) if k_out is not None else None,
            kc.data_ptr(), vc.data_ptr(), cache.block_table.data_ptr(), cache.num_blocks,
            cache.block_size, cache.max_blocks_per_seq, _lib.strides(*kc.stride()),
            _lib.strides(*vc.stride()), _lib.strides(*cache.block_table.stride()),
            err.data_ptr() if err is not None else None, stream_of(cache.device))
        _lib.check(st, "rope_and_store")
        device_errors(err, "rope_and_store")
    return q_out


def permute_rope_rows(w: torch.Tensor, head_dim: int = 128) -> torch.Tensor:
    """Rows of a QKV weight [heads * head_dim, K] reordered for ``qkv_rope_store``:
    within each head, 16-row tiles of dims (8c .. 8c+7, 64+8c .. 64+8c+7), c = 0..7,
    so every tile holds its rotary pairs (d, d + 64)."""
    if head_dim != 128 or w.shape[0] % head_dim != 0:
        raise ValueError("permute_rope_rows expects head_dim 128 and whole heads")
    heads = w.shape[0] // head_dim
    base = torch.arange(8).repeat_interleave(8) * 8 + torch.arange(8).repeat(8)  # 8c + r
    tile = torch.stack([base.view(8, 8), base.view(8, 8) + 64], dim=1).reshape(-1)
    idx = (torch.arange(heads)[:, None] * head_dim + tile[None, :]).reshape(-1)
    return w[idx.to(w.device)].contiguous()


def qkv_rope_store(cache: KVCache, layer_idx: int, x: torch.Tensor, w_rope: torch.Tensor,
                   num_q_heads: int, cos_table: torch.Tensor, sin_table: torch.Tensor,
                   start_pos: torch.Tensor, eps: float = 1e-5,
                   q_out: torch.Tensor = None, static_weight: bool = False) -> torch.Tensor:
    """Decode step, one launch: RMSNorm + QKV projection + RoPE + KV slot writes.

    x: [B, 1, K] or [B, K] fp16 (one new token per sequence, B <= 16); w_rope: the
    folded QKV weight (``kernels.matmul.fold_rms_weight``) with rows permuted by
    ``permute_rope_rows``; start_pos: [B] int32 device positions. The same bits as
    ``fp16_linear_folded`` followed by ``rope_and_store``. Returns rotated q
    [B, 1, nq, D] (``q_out`` if given). ``static_weight``: ``w_rope`` is constant, so
    its first tiles load while the previous kernel finishes (``FI_STATIC_WEIGHTS``).
    """
    cache.sync_block_table()
    D, nkv = cache.head_dim, cache.num_heads
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    if x2.dtype != torch.float16 or x2.device != cache.device:
        raise ValueError("x must be float16 on the cache device")
    if w_rope.shape != ((num_q_heads + 2 * nkv) * D, K):
        raise ValueError("w_rope must be [(nq + 2*nkv) * head_dim, K]")
    if B > cache.block_table.shape[0]:
        raise ValueError("batch larger than the block table; call _grow_batch first")
    if not isinstance(start_pos, torch.Tensor) or start_pos.numel() != B:
        raise ValueError("start_pos must be a [B] device tensor")
    if x2.stride(1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    sp = start_pos.to(torch.int32).contiguous()
    if q_out is None:
        q_out = torch.empty(B, 1, num_q_heads, D, dtype=torch.float16, device=cache.device)
    q2 = q_out[:, 0]
    kc, vc = cache.k[layer_idx], cache.v[layer_idx]
    lib = _lib.load()
    with with_device(cache.device):
        err = error_word(cache.device)
        st = lib.fi_qkv_rope_kv_write(
            x2.data_ptr(), w_rope.data_ptr(), float(eps), B, K, num_q_heads, nkv, D,
            _lib.strides(*x2.stride()), _lib.strides(*w_rope.stride()),
            cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], cos_table.stride(0),
            sp.data_ptr(), q2.data_ptr(), _lib.strides(*q2.stride()),
            kc.data_ptr(), vc.data_ptr(), cache.block_table.data_ptr(), cache.num_blocks,
            cache.block_size, cache.max_blocks_per_seq, _lib.strides(*kc.stride()),
            _lib.strides(*vc.stride()), _lib.strides(*cache.block_table.stride()),
            _lib.FI_STATIC_WEIGHTS if static_weight else 0,
            err.data_ptr() if err is not None else None, stream_of(cache.device))
        _lib.check(st, "qkv_rope_store")
        device_errors(err, "qkv_rope_store")
    return q_out
