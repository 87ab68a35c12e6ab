"""Multi-layer attention stack on the B200 path (the config-4 harness).

A Llama-3.2-3B-shaped stack of attention blocks — per layer
RMSNorm -> QKV projection -> RoPE -> causal attention -> O projection -> residual —
run the way the reference model runs them (model.py:77-135): prefill of a whole
prompt through ``flash_attention`` plus the KV slot write, then one token per step
through the slot write plus ``paged_attention`` over the paged cache. The MLP half
of each decoder layer is not part of this harness (it is not on the attention path).

Sharding by KV head (``fast_infer_b200.shard``): rank r of N holds the QKV weight
columns of its KV heads and their query heads, and a KV cache with Hkv/N heads;
attention needs no exchange. Every rank carries the whole hidden state. In the
decode step each rank multiplies its heads' attention output [tokens, Hq/N * D] by
the matching input columns of the O projection, and the ranks' partial outputs are
summed over NVLink inside that GEMM (``PeerReduce``, one kernel per layer; every rank
gets the same bits). Prefill keeps the residual stream split by token: the normalised
rows are all-gathered for the QKV projection, and an all-to-all hands each rank every
head of its own rows for the O projection (NCCL; ``prefill``).

Decode is autoregressive in hidden space: the stack's output for token t is the
input of token t+1 (there is no embedding or sampler in an attention-only stack).
Weights are random N(0, 0.02) fp16 drawn on the device from a fixed seed, identical
on every rank (same GPU model), then sliced to the rank's heads.

The projections are cuBLAS GEMMs through PyTorch (the residual add rides in the O
projection's GEMM as beta = 1); RMSNorm is one launch of ``fi_rms_norm`` (reference
kernels/rms_norm.py:8-43, fp32 math, fp16 out). RoPE (reference kernels/rope.py:9-44)
and the KV slot write are one fused kernel (``rope_and_store`` / fi_rope_kv_write),
bit-identical to the reference's fp16 ops. ``apply_rope`` and ``rms_norm_torch``
below restate the reference's RoPE and RMSNorm in PyTorch for tests.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch

from fast_infer_b200._runtime import device_checks
from fast_infer_b200.kernels.attention import flash_attention, paged_attention
from fast_infer_b200.kernels.matmul import fold_rms_weight, fp16_linear
from fast_infer_b200.kernels.rms_norm import rms_norm
from fast_infer_b200.kv_cache import KVCache, permute_rope_rows, qkv_rope_store, rope_and_store
from fast_infer_b200.shard import (HeadShard, PeerGather, PeerReduce, gather_heads, gather_rows,
                                   head_shard, heads_to_tokens, token_block)


def precompute_freqs(head_dim: int, max_seq_len: int, theta: float, device) -> tuple:
    """cos/sin tables [max_seq_len, head_dim] (reference kernels/rope.py:9-16)."""
    freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    pos = torch.arange(max_seq_len, device=device).float()
    ang = torch.outer(pos, freq)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos(), ang.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x * cos + rotate_half(x) * sin for x [B, S, H, D], cos/sin [S, D] fp16
    (reference kernels/rope.py:19-44)."""
    d = x.shape[-1]
    rot = torch.cat([-x[..., d // 2:], x[..., : d // 2]], dim=-1)
    return x * cos.unsqueeze(1) + rot * sin.unsqueeze(1)


def rms_norm_torch(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w in fp32, fp16 out (reference kernels/rms_norm.py)."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class AttentionStack:
    """``num_layers`` attention blocks of the config-4 shape, sharded by KV head."""

    def __init__(self, num_layers: int = 28, hidden: int = 3072, num_q_heads: int = 24,
                 num_kv_heads: int = 8, head_dim: int = 128, rope_theta: float = 500000.0,
                 rms_eps: float = 1e-5, batch: int = 16, max_seq_len: int = 1280,
                 rank: int = 0, world: int = 1, device=None, seed: int = 0,
                 gather: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 decode_exchange: str = "reduce", prefill_exchange: str = "tokens"):
        """``decode_exchange`` (multi-rank decode): "reduce" = O projection sharded by
        head with the cross-rank sum in the GEMM (``PeerReduce``); "gather" = head
        outputs gathered over peer memory (``PeerGather``), whole O projection on every
        rank; "nccl" = the same with an NCCL all-gather. A custom ``gather`` callable
        or fewer than two layers use the gather path with that callable / NCCL.
        ``prefill_exchange`` (multi-rank prefill, see ``prefill``): "tokens" = residual
        stream split by token, heads switched to tokens by an all-to-all; "gather" =
        head outputs all-gathered, whole O projection on every rank (also used with a
        custom ``gather`` callable, or when B*S does not split evenly)."""
        if decode_exchange not in ("reduce", "gather", "nccl"):
            raise ValueError(f"decode_exchange must be reduce, gather or nccl: {decode_exchange}")
        if prefill_exchange not in ("tokens", "gather"):
            raise ValueError(f"prefill_exchange must be tokens or gather: {prefill_exchange}")
        self.device = torch.device(device or "cuda")
        self.L, self.hidden, self.D = num_layers, hidden, head_dim
        self.hq, self.hkv = num_q_heads, num_kv_heads
        self.eps = rms_eps
        self.batch = batch
        self.shard: HeadShard = head_shard(rank, world, num_q_heads, num_kv_heads)
        self.world = world
        self.gather = gather if gather is not None else gather_heads
        # decode-step exchange over NVLink peer memory, set up with the decode state on
        # multi-rank runs that use the default gather (one buffer per layer, so two
        # consecutive calls never share one: at least two layers)
        self._peer = None
        self._reduce = None
        peer_ok = gather is None and world > 1 and num_layers >= 2
        self._exchange = decode_exchange if peer_ok else "nccl"
        self._prefill_exchange = prefill_exchange if gather is None else "gather"
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        dev = self.device
        sh = self.shard
        self.layers = []
        for _ in range(num_layers):
            # full weights drawn identically on every rank, then sliced to the shard
            wq = torch.randn(hidden, num_q_heads * head_dim, generator=g, device=dev) * 0.02
            wk = torch.randn(hidden, num_kv_heads * head_dim, generator=g, device=dev) * 0.02
            wv = torch.randn(hidden, num_kv_heads * head_dim, generator=g, device=dev) * 0.02
            wo = torch.randn(num_q_heads * head_dim, hidden, generator=g, device=dev) * 0.02
            norm = 1.0 + 0.1 * torch.randn(hidden, generator=g, device=dev)
            q_cols = slice(sh.q_start * head_dim, sh.q_end * head_dim)
            kv_cols = slice(sh.kv_start * head_dim, sh.kv_end * head_dim)
            wqkv = torch.cat([wq[:, q_cols], wk[:, kv_cols], wv[:, kv_cols]], dim=1)
            # weights kept as [out, in] (the reference's linear layout): the decode GEMMs
            # stream them row by row, the prefill GEMMs read them transposed
            wqkv_t = wqkv.t().half().contiguous()
            # decode: norm weight folded in, rows permuted so each 16-row tile holds
            # its rotary pairs (one launch for norm + QKV + RoPE + slot writes)
            wo_t = wo.t().half().contiguous()
            self.layers.append(dict(norm=norm.half(), wqkv_t=wqkv_t,
                                    wqkv_rope=permute_rope_rows(
                                        fold_rms_weight(wqkv_t, norm.half())),
                                    wo_t=wo_t,
                                    # the O projection's input columns of this rank's heads
                                    wo_part=wo_t[:, q_cols].contiguous()
                                    if self._exchange == "reduce" else None))
        self.cos, self.sin = precompute_freqs(head_dim, max_seq_len, rope_theta, self.device)
        pages_per_seq = (max_seq_len + 63) // 64
        self.cache = KVCache(num_layers, sh.num_kv_heads, head_dim, max_seq_len, 64, self.device,
                             num_blocks=batch * pages_per_seq)
        self.cache._grow_batch(batch)
        self.token_count = 0

    def reset(self):
        self.cache.reset()
        self.cache._grow_batch(self.batch)
        self.token_count = 0

    def _gather(self, o: torch.Tensor, layer: Optional[int] = None) -> torch.Tensor:
        if self.world == 1:
            return o
        if layer is not None and self._peer is not None:
            return self._peer.gather(o, layer)  # one buffer per layer
        return self.gather(o)

    @staticmethod
    def _residual(h: torch.Tensor, o: torch.Tensor, wo_t: torch.Tensor) -> None:
        """h += o @ wo_t.T as one GEMM with beta = 1 (h contiguous, updated in place)."""
        h.view(-1, h.shape[-1]).addmm_(o.reshape(-1, o.shape[-1]), wo_t.t())

    # ------------------------------------------------------------------ prefill
    def _qkv(self, w, h):
        return rms_norm(h, w["norm"], self.eps) @ w["wqkv_t"].t()

    def prefill(self, h: torch.Tensor) -> torch.Tensor:
        """Prompt pass (reference model.py:67-69, 101-117): h [B, S, hidden] fp16.
        Per layer: projection, then one fused RoPE + KV slot-write launch, then the
        causal prefill kernel on rotated q / k and the v columns of the projection.

        Several ranks with ``prefill_exchange="tokens"`` (the default): the residual
        stream is kept split by token (rank r owns rows ``token_block(r)`` of the
        flattened [B*S] tokens). Each layer normalises its own rows, all-gathers them
        for the QKV projection of its heads, and after attention switches its heads'
        outputs to every head of its own rows (``heads_to_tokens``: an all-to-all of
        1/N of the outputs instead of an all-gather of all of them), so the O
        projection and the residual add run on 1/N of the tokens. The full hidden
        state is gathered once at the end. ``"gather"``: the head outputs are
        all-gathered and every rank runs the whole O projection."""
        B, S, _ = h.shape
        self.reset()
        D, nq, nkv = self.D, self.shard.num_q_heads, self.shard.num_kv_heads
        need = (S + 63) // 64
        for b in range(B):  # model.py:172-174 allocation order
            self.cache._ensure_blocks(b, need)
        self.cache.num_tokens = S
        k_rot = torch.empty(B, S, nkv, D, dtype=torch.float16, device=self.device)
        if self.world > 1 and self._prefill_exchange == "tokens" and (B * S) % self.world == 0:
            h = self._prefill_token_split(h, k_rot)
        else:
            h = h.contiguous().clone()  # the residual stream is updated in place below
            for li, w in enumerate(self.layers):
                qkv = self._qkv(w, h)
                q_rot = rope_and_store(self.cache, li, qkv, nq, self.cos, self.sin, 0,
                                       k_out=k_rot)
                v = qkv[..., (nq + nkv) * D:].view(B, S, nkv, D)
                o = flash_attention(q_rot.transpose(1, 2), k_rot.transpose(1, 2),
                                    v.transpose(1, 2))
                o = self._gather(o.transpose(1, 2).reshape(B, S, nq * D))
                self._residual(h, o, w["wo_t"])
        self.token_count = S
        return h

    def _prefill_token_split(self, h: torch.Tensor, k_rot: torch.Tensor) -> torch.Tensor:
        """Layers of ``prefill`` with the residual stream split by token over the ranks
        (see ``prefill``); returns the full [B, S, hidden] output on every rank."""
        B, S, hid = h.shape
        D, nq, nkv = self.D, self.shard.num_q_heads, self.shard.num_kv_heads
        T = B * S
        t0, t1 = token_block(self.shard.rank, self.world, T)
        # this rank's rows of the stream, a copy: it is updated in place below (a row
        # slice of a contiguous tensor is itself contiguous, so .contiguous() would alias
        # the caller's h)
        h_rows = h.reshape(T, hid)[t0:t1].clone()
        for li, w in enumerate(self.layers):
            x = gather_rows(rms_norm(h_rows, w["norm"], self.eps))  # [T, hidden]
            qkv = (x @ w["wqkv_t"].t()).view(B, S, -1)
            q_rot = rope_and_store(self.cache, li, qkv, nq, self.cos, self.sin, 0, k_out=k_rot)
            v = qkv[..., (nq + nkv) * D:].view(B, S, nkv, D)
            o = flash_attention(q_rot.transpose(1, 2), k_rot.transpose(1, 2), v.transpose(1, 2))
            o_rows = heads_to_tokens(o.transpose(1, 2).reshape(T, nq * D))  # [T/N, Hq*D]
            h_rows.addmm_(o_rows, w["wo_t"].t())  # h += o @ Wo on this rank's rows
        return gather_rows(h_rows).view(B, S, hid)

    # ------------------------------------------------------------------- decode
    def _decode_state(self):
        """Device-resident step state, so one decode step is a fixed sequence of
        launches (CUDA-graph capturable): per-sequence context lengths (including the
        new token) and the new token's write / rotary position."""
        if getattr(self, "_dev_ctx", None) is None:
            B = self.batch
            self._dev_ctx = torch.zeros(B, dtype=torch.int32, device=self.device)
            self._dev_start = torch.zeros(B, dtype=torch.int32, device=self.device)
            span = self.cache.max_blocks_per_seq * 64
            from fast_infer_b200.kernels.attention import paged_attention_workspace_bytes
            need = paged_attention_workspace_bytes(B, self.shard.num_q_heads,
                                                   self.shard.num_kv_heads, span)
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
            self._h_in = torch.zeros(B, 1, self.hidden, dtype=torch.float16, device=self.device)
            self._graph = None
            if self._exchange == "reduce" and self._reduce is None:
                self._reduce = PeerReduce(self.hidden, self.L, device=self.device)
            elif self._exchange == "gather" and self._peer is None:
                self._peer = PeerGather(B, self.shard.num_q_heads * self.D, self.L,
                                        device=self.device)

    def _decode_body(self):
        """One decode token through every layer, reading positions from device
        memory (reference model.py:70-72, 118-131); advances them at the end."""
        B = self.batch
        nq, D = self.shard.num_q_heads, self.D
        span = self.cache.max_blocks_per_seq * 64
        h = self._h_in.clone()  # the residual stream is updated in place below
        for li, w in enumerate(self.layers):
            # RMSNorm + QKV projection + RoPE + KV slot writes in one launch; the
            # weights are constant, so their first tiles load during the previous kernel
            q = qkv_rope_store(self.cache, li, h, w["wqkv_rope"], nq, self.cos, self.sin,
                               self._dev_start, eps=self.eps, static_weight=True)
            o = paged_attention(q[:, 0], self.cache.k[li], self.cache.v[li],
                                self.cache.block_table, 64, 0, context_lens=self._dev_ctx,
                                max_context_len=span, workspace=self._ws)
            if self._reduce is not None:  # h += sum over ranks of o_r @ Wo_r, one kernel
                hv = h.view(B, self.hidden)
                self._reduce.linear(o.view(B, nq * D), w["wo_part"], hv, hv, li,
                                    static_weight=True)
                continue
            o = self._gather(o.reshape(B, 1, nq * D), li)
            fp16_linear(o, w["wo_t"], residual=h, out=h, static_weight=True)  # h += o @ Wo
        self._dev_ctx.add_(1)
        self._dev_start.add_(1)
        self._h_in.copy_(h)
        return h

    def _host_step(self):
        """Host bookkeeping before a decode step: allocate a page for every sequence
        when the new token starts one (reference model.py:193-198)."""
        pos = self.token_count
        if pos >= self.cache.max_blocks_per_seq * 64:
            raise RuntimeError("sequence longer than the stack's max_seq_len")
        if pos % 64 == 0 or self.cache._dirty:
            for b in range(self.batch):
                self.cache._ensure_blocks(b, pos // 64 + 1)
            self.cache.sync_block_table()
        self.cache.num_tokens += 1
        self.token_count += 1

    def begin_decode(self, h_last: torch.Tensor):
        """Set the decode state after ``prefill``: h_last [B, 1, hidden] is the first
        decode input; positions continue from the prompt length."""
        self._decode_state()
        self._dev_ctx.fill_(self.token_count + 1)
        self._dev_start.fill_(self.token_count)
        self._h_in.copy_(h_last)

    def decode_step(self, use_graph: bool = True) -> torch.Tensor:
        """One decode token for the whole batch; returns the stack output
        [B, 1, hidden] (a buffer that the next step overwrites)."""
        self._host_step()
        if not use_graph:
            return self._decode_body().clone()
        if self._graph is None:
            self._capture()  # captures the step and runs it once
        else:
            self._graph.replay()
        return self._h_out

    def _capture(self):
        # Save the state, run the body once eagerly (first-call set-up of every
        # kernel), restore the state, then capture one step.
        saved = [t.clone() for t in (self._dev_ctx, self._dev_start, self._h_in)]
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._decode_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        for t, v in zip((self._dev_ctx, self._dev_start, self._h_in), saved):
            t.copy_(v)
        g = torch.cuda.CUDAGraph()
        # reading the device error word synchronises, which a capture forbids
        with device_checks(False), torch.cuda.graph(g):
            self._h_out = self._decode_body()
        self._graph = g
        # the capture recorded but did not run the step: run it now
        self._graph.replay()

    def release_graph(self):
        """Drop the captured decode graph (call before destroying a process group
        whose collectives it holds)."""
        self._graph = None

    def close(self):
        """Release the decode graph and the peer-memory buffers (collective on
        multi-rank runs: every rank calls it before the process group goes away)."""
        self.release_graph()
        if self._peer is not None:
            self._peer.close()
            self._peer = None
        if self._reduce is not None:
            self._reduce.close()
            self._reduce = None

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """Reference-style entry (model.py:50-160): S > 1 or the first call = prefill,
        otherwise one decode token (eager). h: [B, S, hidden] fp16."""
        if h.shape[1] > 1 or self.token_count == 0:
            return self.prefill(h)
        if getattr(self, "_dev_ctx", None) is None or self._graph is None:
            self.begin_decode(h)
        else:
            self._h_in.copy_(h)
        return self.decode_step(use_graph=False)

    def generate(self, prompt_hidden: torch.Tensor, steps: int,
                 use_graph: bool = True) -> torch.Tensor:
        """Prefill the prompt, then ``steps`` decode steps each fed with the previous
        step's output; returns the decode outputs [B, steps, hidden]."""
        h = self.prefill(prompt_hidden)[:, -1:]
        self.begin_decode(h)
        outs = []
        for _ in range(steps):
            outs.append(self.decode_step(use_graph=use_graph).clone())
        return torch.cat(outs, dim=1) if outs else h[:, :0]
