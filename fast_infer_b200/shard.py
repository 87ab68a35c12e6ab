"""Partitioning of the attention path across the GPUs of one node.

Attention needs no exchange between GPUs: each query head reads exactly one KV
head (GQA, h -> h // (Hq/Hkv)) and each sequence its own pages. So the path shards
with no collective on the data path, one process per GPU:

* by KV head — rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and the query heads
  that read them (contiguous, since the group of KV head j is [j*G, (j+1)*G)); each
  rank keeps a KVCache with Hkv/N heads and the full (replicated) block table;
* by sequence — rank r owns a contiguous slice of the batch with all heads.

Collectives for callers that need more than attention (NCCL over NVLink on B200; gloo
in the CPU tests): ``gather_heads`` all-gathers the per-rank [tokens, heads_r*D]
outputs and reassembles them in head order; ``heads_to_tokens`` (an all-to-all) hands
each rank every head of its own block of tokens instead, and ``gather_rows``
all-gathers row blocks — the pair a token-split prefill uses. ``PeerGather`` does the
head gather for the decode step in one kernel of our own: each rank stores its rows
straight into every rank's buffer over NVLink (CUDA IPC mappings) and waits on
per-call flags; ``PeerReduce`` sums per-rank partial projections the same way.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_start: int
    kv_end: int
    q_start: int
    q_end: int

    @property
    def num_kv_heads(self) -> int:
        return self.kv_end - self.kv_start

    @property
    def num_q_heads(self) -> int:
        return self.q_end - self.q_start


def head_shard(rank: int, world: int, num_q_heads: int, num_kv_heads: int) -> HeadShard:
    """KV-head partition of rank ``rank`` of ``world`` (KV heads must divide evenly)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    if num_q_heads % num_kv_heads != 0:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")
    per = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    kv0 = rank * per
    return HeadShard(rank, world, kv0, kv0 + per, kv0 * g, (kv0 + per) * g)


def seq_range(rank: int, world: int, batch: int) -> tuple[int, int]:
    """Contiguous batch slice of a rank (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_heads(x, shard: HeadShard, kv: bool, dim: int = 1):
    """Slice a tensor's head dimension to this rank's query (kv=False) or KV heads."""
    lo, hi = (shard.kv_start, shard.kv_end) if kv else (shard.q_start, shard.q_end)
    return x.narrow(dim, lo, hi - lo)


def gather_heads(local, group=None, head_dim_axis: int = -1):
    """All-gather per-rank attention outputs along the flattened head axis.

    ``local``: [..., heads_r * D] of this rank (equal shapes on every rank). Returns
    [..., world * heads_r * D] with rank r's block at position r, i.e. the heads in
    their original order. Uses torch.distributed (NCCL on GPUs, gloo on CPU).
    """
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local
    local = local.contiguous()
    if dist.get_backend(group) == "nccl" and head_dim_axis in (-1, local.dim() - 1):
        # one collective into [world, ...], then one copy into head order
        out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local, group=group)
        return out.movedim(0, -2).reshape(*local.shape[:-1], world * local.shape[-1])
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local, group=group)
    return torch.cat(parts, dim=head_dim_axis)


def token_block(rank: int, world: int, tokens: int) -> tuple[int, int]:
    """Rows [start, end) of the token block a rank owns when a [tokens, ...] tensor is
    split evenly by rows (``tokens`` a multiple of ``world``)."""
    if tokens % world != 0:
        raise ValueError(f"{tokens} tokens do not split evenly over {world} ranks")
    per = tokens // world
    return rank * per, (rank + 1) * per


def gather_rows(local, group=None):
    """All-gather equal row blocks: [T / world, ...] of every rank -> [T, ...] with rank
    r's block at rows [r*T/world, (r+1)*T/world) (one collective)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local
    local = local.contiguous()
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), local, group=group)
    return out


def heads_to_tokens(local, group=None):
    """Switch a [T, heads_r * D] tensor (this rank's heads, every token) to
    [T / world, world * heads_r * D] (every head in head order, this rank's token block
    of ``token_block``): one all-to-all of equal blocks, then one copy into head order.
    Each rank sends and receives (world - 1) / world of its block — an all-gather of the
    same outputs moves world times more."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local
    T, cols = local.shape
    if T % world != 0:
        raise ValueError(f"{T} tokens do not split evenly over {world} ranks")
    local = local.contiguous()
    recv = torch.empty_like(local)  # block j = rank j's heads of this rank's tokens
    dist.all_to_all_single(recv, local, group=group)
    return recv.view(world, T // world, cols).transpose(0, 1).reshape(T // world, world * cols)


class _DeviceArray:
    """Zero-copy view of raw device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape, typestr: str = "<f2"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


def _map_regions(nbytes: int, world: int, rank: int, group, device):
    """Allocate this rank's peer region and map every other rank's (CUDA IPC handles
    exchanged with ``all_gather_object``; collective). Returns (own pointer, pointers
    opened here, a ctypes array of every rank's region as seen from this rank)."""
    import ctypes
    import torch
    import torch.distributed as dist
    from fast_infer_b200 import _lib
    lib = _lib.load()
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * 64)()
    with torch.cuda.device(device):
        _lib.check(lib.fi_peer_alloc(nbytes, ctypes.byref(own), handle), "fi_peer_alloc")
    handles = [None] * world
    dist.all_gather_object(handles, bytes(handle), group=group)
    opened, bases = [], []
    with torch.cuda.device(device):
        for p, hb in enumerate(handles):
            if p == rank:
                bases.append(own.value)
                continue
            ptr = ctypes.c_void_p()
            hbuf = (ctypes.c_uint8 * 64).from_buffer_copy(hb)
            _lib.check(lib.fi_peer_open(hbuf, ctypes.byref(ptr)), "fi_peer_open")
            opened.append(ptr.value)
            bases.append(ptr.value)
    return own.value, opened, (ctypes.c_void_p * 8)(*bases, *([None] * (8 - world)))


def _unmap_regions(lib, own, opened, device, group):
    """Unmap the peers' regions, then free this rank's once every rank has unmapped
    it (collective)."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize(device)
    with torch.cuda.device(device):
        for p in opened:
            lib.fi_peer_close(p)
        dist.barrier(group=group)
        lib.fi_peer_free(own)


class PeerGather:
    """``gather_heads`` for the decode step, over NVLink peer memory instead of NCCL.

    Every rank allocates one region of ``nbuf`` gather buffers [max_rows, world *
    row_elems] fp16 and maps every other rank's region (CUDA IPC handles exchanged
    with ``all_gather_object`` on ``group``). ``gather(local, buffer)`` is one kernel
    (``fi_peer_gather``) that stores this rank's rows into buffer ``buffer`` of every
    region and waits until every rank has delivered the same call; it returns this
    rank's buffer as [rows, world * row_elems], heads in their original order. Every
    rank must make the same sequence of calls, and two uses of one buffer need another
    gather between them, so more than one rank needs ``nbuf >= 2`` (the stack uses one
    buffer per layer and at least two layers). Construct it on every
    rank at the same point (it runs collectives); call ``close`` before the process
    group goes away.
    """

    def __init__(self, max_rows: int, row_elems: int, nbuf: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        from fast_infer_b200 import _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerGather supports up to 8 ranks")
        if self.world > 1 and nbuf < 2:
            # a rank one call ahead would overwrite words a slower rank has not read
            raise ValueError(f"PeerGather over {self.world} ranks needs nbuf >= 2, got {nbuf}")
        self.device = torch.device(device or "cuda")
        self.max_rows, self.row_elems, self.nbuf = max_rows, row_elems, nbuf
        self._lib = lib = _lib.load()
        nbytes = lib.fi_peer_gather_bytes(nbuf, max_rows, self.world * row_elems * 2)
        self._own, self._opened, self._bases = _map_regions(nbytes, self.world, self.rank, group,
                                                            self.device)
        self._buffers = torch.as_tensor(
            _DeviceArray(self._own, (nbuf, max_rows, self.world * row_elems)), device=self.device)
        # persistent device error word of every gather (FI_DEVERR_TIMEOUT once a wait ran
        # out; later gathers then skip their waits); read with ``errors()``
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def gather(self, local, buffer: int):
        import ctypes
        from fast_infer_b200 import _lib
        from fast_infer_b200._runtime import device_errors, error_word, stream_of
        rows = local.numel() // self.row_elems
        x = local.reshape(rows, self.row_elems)
        if x.stride(1) != 1 or (x.stride(0) * 2) % 16 != 0 or x.data_ptr() % 16 != 0:
            x = x.contiguous()
        st = self._lib.fi_peer_gather(
            x.data_ptr(), rows, self.row_elems * 2, x.stride(0) * 2,
            ctypes.cast(self._bases, ctypes.POINTER(ctypes.c_void_p)), self.world, self.rank,
            buffer, self.nbuf, self.max_rows, self._err.data_ptr(), stream_of(self.device))
        _lib.check(st, "peer gather")
        if error_word(self.device) is not None:  # device checks on: raise at once
            device_errors(self._err, "peer gather")
        return self._buffers[buffer, :rows].view(*local.shape[:-1], self.world * self.row_elems)

    def result(self, buffer: int, rows: int):
        """This rank's buffer ``buffer`` as [rows, world * row_elems]: what the last
        gather into it delivered (rank p's block at columns [p * row_elems, ...))."""
        return self._buffers[buffer, :rows]

    def errors(self) -> int:
        """FI_DEVERR_* bits raised by any gather so far (synchronises the stream)."""
        return int(self._err.item())

    def close(self, group=None):
        """Unmap the peers' regions and free this rank's once every rank has unmapped
        it (collective: every rank calls it)."""
        if self._own is None:
            return
        self._buffers = None
        _unmap_regions(self._lib, self._own, self._opened, self.device, group)
        self._own, self._opened = None, []


class PeerReduce:
    """The O projection of a KV-head-sharded decode step with its cross-rank sum over
    NVLink peer memory, in one kernel (``fi_small_gemm_peer_reduce``).

    ``linear(x, w_part, residual, out, buffer)`` computes, on every rank,
    out = residual + sum over ranks p (rank order) of fp16(x_p @ w_part_p^T): x_p
    [rows, k] is rank p's heads' attention output, w_part_p [n, k] the projection's
    input columns of those heads. Every rank ends with the same bits. Every rank must
    make the same sequence of calls, consecutive calls using different buffers (more
    than one rank needs ``nbuf >= 2``; the stack uses one buffer per layer). Construct
    it on every rank at the same point (it runs collectives); call ``close`` before the
    process group goes away.
    """

    def __init__(self, n: int, nbuf: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        from fast_infer_b200 import _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerReduce supports up to 8 ranks")
        if self.world > 1 and nbuf < 2:
            raise ValueError(f"PeerReduce over {self.world} ranks needs nbuf >= 2, got {nbuf}")
        self.device = torch.device(device or "cuda")
        self.n, self.nbuf = n, nbuf
        self._lib = lib = _lib.load()
        nbytes = lib.fi_peer_reduce_bytes(nbuf, self.world, n)
        self._own, self._opened, self._bases = _map_regions(nbytes, self.world, self.rank, group,
                                                            self.device)
        # persistent device error word (FI_DEVERR_TIMEOUT once a wait ran out; later
        # calls then skip their waits); read with ``errors()``
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def linear(self, x, w_part, residual, out, buffer: int, static_weight: bool = False):
        import ctypes
        from fast_infer_b200 import _lib
        from fast_infer_b200._runtime import device_errors, error_word, stream_of
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
            x2 = x2.contiguous()
        o2 = out.view(-1, out.shape[-1])
        r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
        st = self._lib.fi_small_gemm_peer_reduce(
            x2.data_ptr(), w_part.data_ptr(), o2.data_ptr(),
            r2.data_ptr() if r2 is not None else None, x2.shape[0], w_part.shape[0],
            x2.shape[1], _lib.strides(*x2.stride()), _lib.strides(*w_part.stride()),
            _lib.strides(*o2.stride()), _lib.strides(*r2.stride()) if r2 is not None else None,
            ctypes.cast(self._bases, ctypes.POINTER(ctypes.c_void_p)), self.world, self.rank,
            buffer, self.nbuf, _lib.FI_STATIC_WEIGHTS if static_weight else 0,
            self._err.data_ptr(), stream_of(self.device))
        _lib.check(st, "peer reduce")
        if error_word(self.device) is not None:  # device checks on: raise at once
            device_errors(self._err, "peer reduce")
        return out

    def errors(self) -> int:
        """FI_DEVERR_* bits raised by any call so far (synchronises the stream)."""
        return int(self._err.item())

    def close(self, group=None):
        """Unmap the peers' regions and free this rank's (collective)."""
        if self._own is None:
            return
        _unmap_regions(self._lib, self._own, self._opened, self.device, group)
        self._own, self._opened = None, []
