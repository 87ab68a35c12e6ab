"""The drop-in through the reference model's own call sequence (model.py:50-160).

``tests/golden/model_forward.npz`` holds a run of the reference's
``LlamaForCausalLM.forward`` (2 layers of the Llama-3.2-3B shape, INT4 memory mode,
its Triton kernels under TRITON_INTERPRET=1): a 62-token prefill of 2 sequences and
4 decode tokens, the last of which starts a new page. These tests replay that call
sequence with the patch of INTEGRATION.md applied — this library's
``flash_attention``, ``paged_attention``, ``KVCache``, ``store_kv_prefill`` and
``store_kv_decode`` at model.py:10,113,117,120,123-130:

* teacher-forced: every attention call gets the inputs the reference's own call got
  (q after RoPE, k / v as stored), in model.py's forms (a BHSD view of BSHD memory,
  K/V expanded with ``repeat_interleave`` for prefill, the scalar ``num_tokens``
  for decode); outputs within the north-star tolerance of the reference's, the
  block table, free list and ``num_tokens`` equal, and the whole pool bit-identical
  (SHA-256) after every forward;
* free-running: the whole forward restated with the library's drop-ins for every
  kernel it has (RMSNorm, INT4 projections, attention, slot writes; embedding,
  RoPE, SiLU and the LM head in torch as model.py has them) reproduces the
  reference's logits.
"""

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import MAX_ABS_TOL, REL_L2_TOL, error_stats
from tests.golden.inputs import MODEL, model_token_ids, model_weights

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "model_forward.npz"
# Logits after 2 layers of INT4 projections + attention + SwiGLU: each projection is
# within one fp16 ulp of the reference kernel's (different fp32 summation order), so
# the logits are compared by relative L2 and by max-abs relative to their magnitude.
LOGITS_REL_L2 = 2e-3
LOGITS_MAX_ABS_REL = 5e-3


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def _check_cache_state(cache, g, i):
    cache.sync_block_table()
    assert np.array_equal(cache.block_table.cpu().numpy(), g[f"f{i}_block_table"]), i
    assert cache.free_blocks == g[f"f{i}_free_blocks"].tolist(), i
    assert cache.num_tokens == int(g[f"f{i}_num_tokens"]), i
    torch.cuda.synchronize()
    assert _sha(cache.k) == str(g[f"f{i}_k_sha"]), f"k pool after forward {i}"
    assert _sha(cache.v) == str(g[f"f{i}_v_sha"]), f"v pool after forward {i}"


def test_model_call_sequence_teacher_forced(cuda_device, golden):
    from fast_infer_b200.kernels.attention import flash_attention, paged_attention
    from fast_infer_b200.kv_cache import KVCache, store_kv_decode, store_kv_prefill
    c, g, dev = MODEL, golden, cuda_device
    L, G = c["layers"], c["heads"] // c["kv_heads"]
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    # model.py:40-48
    cache = KVCache(L, c["kv_heads"], c["head_dim"], c["max_seq_len"], 64, dev)
    cache._grow_batch(c["batch"])
    token_count = 0
    for i in range(1 + c["decode_steps"]):
        prefill = i == 0
        token_count = c["prompt"] if prefill else token_count + 1  # model.py:67-72
        for layer in range(L):
            key = f"f{i}_l{layer}_"
            q, k, v = t(g[key + "q"]), t(g[key + "k"]), t(g[key + "v"])
            if prefill:  # model.py:104-117
                q_attn = q.transpose(1, 2)
                k_attn = k.transpose(1, 2).repeat_interleave(G, dim=1)
                v_attn = v.transpose(1, 2).repeat_interleave(G, dim=1)
                o = flash_attention(q_attn, k_attn, v_attn)
                assert o.stride() == q_attn.stride()  # empty_like(q), attention.py:99
                out = o.transpose(1, 2).contiguous()
                store_kv_prefill(cache, layer, k, v)
            else:  # model.py:118-131
                store_kv_decode(cache, layer, k, v, token_count)
                assert cache.num_tokens == int(g[key + "num_tokens"])
                cache.sync_block_table()
                out = paged_attention(q, cache.k[layer], cache.v[layer], cache.block_table,
                                      64, cache.num_tokens)
            max_abs, rel = error_stats(out.float().cpu().numpy(),
                                       g[key + "o"].astype(np.float32))
            assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (key, max_abs, rel)
        _check_cache_state(cache, g, i)


# ---------------------------------------------------------------- free-running
def _precompute_freqs(head_dim, max_seq_len, theta):
    """cos/sin [max_seq_len, head_dim] fp32 on the CPU (reference kernels/rope.py:9-16)."""
    freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    ang = torch.outer(torch.arange(max_seq_len).float(), freq)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos(), ang.sin()


def _apply_rope(x, cos, sin):
    """x * cos + rotate_half(x) * sin, fp16 ops (reference kernels/rope.py:19-44)."""
    d = x.shape[-1]
    rot = torch.cat([-x[..., d // 2:], x[..., : d // 2]], dim=-1)
    return x * cos.unsqueeze(1) + rot * sin.unsqueeze(1)


class _Model:
    """model.py:13-206 in memory mode with INTEGRATION.md's patch: the attention,
    KV cache and slot writes of this library, and its RMSNorm / INT4 drop-ins."""

    def __init__(self, dev):
        from fast_infer_b200.kernels.matmul import fuse_qkv_inplace
        from fast_infer_b200.loader import quantize_int4_groupwise
        c = MODEL
        w = model_weights()
        t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
        q4 = lambda a: quantize_int4_groupwise(t(a))  # noqa: E731
        layers = []
        for lw in w["layers"]:
            layers.append({
                "input_layernorm": t(lw["input_layernorm"]),
                "post_attention_layernorm": t(lw["post_attention_layernorm"]),
                "self_attn": {n: q4(lw[n]) for n in ("q_proj", "k_proj", "v_proj", "o_proj")},
                "mlp": {n: q4(lw[n]) for n in ("gate_proj", "up_proj", "down_proj")},
            })
        embed = t(w["embed"])
        self.weights = {"embed_tokens": embed, "layers": layers, "norm": t(w["norm"]),
                        "lm_head": embed}
        fuse_qkv_inplace(self.weights)
        self.dev = dev
        cos, sin = _precompute_freqs(c["head_dim"], c["max_seq_len"], 500000.0)
        self.cos, self.sin = cos.to(dev), sin.to(dev)
        self.kv_cache = None
        self._token_count = 0

    def forward(self, ids):
        from fast_infer_b200.kernels.attention import flash_attention, paged_attention
        from fast_infer_b200.kernels.matmul import int4_matmul
        from fast_infer_b200.kernels.rms_norm import rms_norm
        from fast_infer_b200.kv_cache import KVCache, store_kv_decode, store_kv_prefill
        c = MODEL
        B, S = ids.shape
        H, nq, nkv, D = c["hidden"], c["heads"], c["kv_heads"], c["head_dim"]
        if self.kv_cache is None:
            self.kv_cache = KVCache(c["layers"], nkv, D, c["max_seq_len"], 64, self.dev)
            self.kv_cache._grow_batch(B)
            self._token_count = 0
        is_prefill = S > 1 or self._token_count == 0
        h = self.weights["embed_tokens"][ids].to(torch.float16)
        if is_prefill:
            positions = torch.arange(S, device=self.dev)
            self._token_count = S
        else:
            positions = torch.tensor([self._token_count], device=self.dev)
            self._token_count += 1
        cos, sin = self.cos[positions].half(), self.sin[positions].half()
        for li, lw in enumerate(self.weights["layers"]):
            residual = h
            hn = rms_norm(h, lw["input_layernorm"], 1e-5)
            q, k, v = int4_matmul(hn, lw["self_attn"]["qkv_proj"]).split(
                [H, nkv * D, nkv * D], dim=-1)
            q = _apply_rope(q.view(B, S, nq, D), cos, sin)
            k = _apply_rope(k.view(B, S, nkv, D), cos, sin)
            v = v.view(B, S, nkv, D)
            q_attn = q.transpose(1, 2)
            if is_prefill:
                o = flash_attention(q_attn, k.transpose(1, 2).repeat_interleave(nq // nkv, 1),
                                    v.transpose(1, 2).repeat_interleave(nq // nkv, 1))
                attn = o.transpose(1, 2).contiguous().view(B, S, H)
                store_kv_prefill(self.kv_cache, li, k, v)
            else:
                store_kv_decode(self.kv_cache, li, k.squeeze(1), v.squeeze(1),
                                self._token_count)
                self.kv_cache.sync_block_table()
                attn = paged_attention(q_attn.squeeze(2), self.kv_cache.k[li],
                                       self.kv_cache.v[li], self.kv_cache.block_table, 64,
                                       self.kv_cache.num_tokens).view(B, H).unsqueeze(1)
            h = residual + int4_matmul(attn, lw["self_attn"]["o_proj"])
            residual = h
            hn = rms_norm(h, lw["post_attention_layernorm"], 1e-5)
            gate, up = int4_matmul(hn, lw["mlp"]["gate_up_proj"]).split(c["intermediate"], -1)
            gf = gate.float()
            act = (gf * torch.sigmoid(gf) * up.float()).to(torch.float16)  # kernels/mlp.py:9-24
            h = residual + int4_matmul(act, lw["mlp"]["down_proj"])
        hn = rms_norm(h, self.weights["norm"], 1e-5)
        return torch.matmul(hn, self.weights["lm_head"].T).float()


def test_model_forward_free_running(cuda_device, golden):
    c, g = MODEL, golden
    model = _Model(cuda_device)
    prompt, steps = model_token_ids()
    inputs = [prompt] + [steps[s] for s in range(c["decode_steps"])]
    for i, ids in enumerate(inputs):
        logits = model.forward(torch.from_numpy(ids).to(cuda_device))
        ref = g[f"f{i}_logits"]
        max_abs, rel = error_stats(logits.cpu().numpy(), ref)
        scale = float(np.abs(ref).max())
        assert rel <= LOGITS_REL_L2 and max_abs <= LOGITS_MAX_ABS_REL * scale, \
            (i, max_abs, scale, rel)
        cache = model.kv_cache
        cache.sync_block_table()
        assert np.array_equal(cache.block_table.cpu().numpy(), g[f"f{i}_block_table"]), i
        assert cache.free_blocks == g[f"f{i}_free_blocks"].tolist(), i
        assert cache.num_tokens == int(g[f"f{i}_num_tokens"]), i
