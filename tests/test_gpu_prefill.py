"""GPU parity of the tcgen05 causal prefill kernel against the reference (golden
vectors), the fp32 oracle, and — at full size — an fp32 PyTorch attention:
max-abs <= 2e-3 and relative-L2 <= 1e-3 (north_star tolerances)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import MAX_ABS_TOL, REL_L2_TOL, attention_fp32, error_stats
from tests.golden.inputs import PREFILL_SMALL_S, c1_inputs, prefill_small_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _ok(out, ref, what=""):
    max_abs, rel = error_stats(out, ref)
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, f"{what} max_abs={max_abs} rel={rel}"


def _to(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def torch_causal_fp32(q, k, v, scale=None):
    """Plain fp32 PyTorch causal attention on the GPU (TF32 off), GQA by head index."""
    assert not torch.backends.cuda.matmul.allow_tf32
    B, Hq, S, D = q.shape
    G = Hq // k.shape[1]
    scale = D ** -0.5 if scale is None else scale
    out = torch.empty(B, Hq, S, D, dtype=torch.float32, device=q.device)
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).tril()
    for b in range(B):
        for h in range(Hq):
            s = (q[b, h].float() @ k[b, h // G].float().T) * scale
            s = s.masked_fill(~mask, float("-inf"))
            out[b, h] = torch.softmax(s, dim=-1) @ v[b, h // G].float()
    return out


def test_c1_prefill_vs_reference_and_fp32(cuda_device, device_checks):
    from fast_infer_b200.kernels.attention import flash_attention
    c1 = c1_inputs()
    g = np.load(GOLDEN / "c1.npz")
    q, k, v = (_to(c1[n], cuda_device) for n in ("q", "k", "v"))
    ref32 = attention_fp32(c1["q"], c1["k"], c1["v"])
    # the reference caller's form: K/V expanded with repeat_interleave (model.py:110-111)
    o_exp = flash_attention(q, k.repeat_interleave(3, dim=1), v.repeat_interleave(3, dim=1))
    # GQA without expansion
    o_gqa = flash_attention(q, k, v)
    for o, what in ((o_exp, "expanded"), (o_gqa, "gqa")):
        out = o.cpu().numpy()
        _ok(out, ref32, f"{what} vs fp32")
        _ok(out, g["o_prefill"].astype(np.float32), f"{what} vs reference")
    assert torch.equal(o_exp, o_gqa)


@pytest.mark.parametrize("S", PREFILL_SMALL_S)
def test_small_prefill_vs_reference(cuda_device, device_checks, S):
    from fast_infer_b200.kernels.attention import flash_attention
    q, k, v = prefill_small_inputs(S)
    g = np.load(GOLDEN / "prefill_small.npz")
    out = flash_attention(_to(q, cuda_device), _to(k, cuda_device), _to(v, cuda_device))
    out = out.cpu().numpy()
    _ok(out, g[f"o_S{S}"].astype(np.float32), "vs reference")
    _ok(out, attention_fp32(q, k, v), "vs fp32")


@pytest.mark.parametrize("S", [2, 16, 127, 128, 129, 255, 256, 257, 384, 1000])
def test_ragged_seq_lens_vs_fp32(cuda_device, device_checks, S):
    from fast_infer_b200.kernels.attention import flash_attention
    torch.manual_seed(S)
    q = torch.randn(2, 6, S, 128, device=cuda_device).half()
    k = torch.randn(2, 2, S, 128, device=cuda_device).half()
    v = torch.randn(2, 2, S, 128, device=cuda_device).half()
    out = flash_attention(q, k, v)
    _ok(out.float().cpu().numpy(), torch_causal_fp32(q, k, v).cpu().numpy())


def test_model_layout_strides_preserved(cuda_device, device_checks):
    """model.py passes q as a BHSD view of BSHD memory (strides (S*3072, 128, 3072, 1))
    and K/V expanded; the output must keep q's strides (empty_like, attention.py:99)."""
    from fast_infer_b200.kernels.attention import flash_attention
    torch.manual_seed(0)
    B, S = 2, 300
    q_bshd = torch.randn(B, S, 24, 128, device=cuda_device).half()
    k_bshd = torch.randn(B, S, 8, 128, device=cuda_device).half()
    v_bshd = torch.randn(B, S, 8, 128, device=cuda_device).half()
    q = q_bshd.transpose(1, 2)
    k = k_bshd.transpose(1, 2).repeat_interleave(3, dim=1)
    v = v_bshd.transpose(1, 2).repeat_interleave(3, dim=1)
    out = flash_attention(q, k, v)
    assert out.stride() == q.stride()
    ref = torch_causal_fp32(q, k, v)
    _ok(out.float().cpu().numpy(), ref.cpu().numpy())
    # un-expanded strided K/V views give identical bytes
    out2 = flash_attention(q, k_bshd.transpose(1, 2), v_bshd.transpose(1, 2))
    assert torch.equal(out, out2)


def test_custom_scale(cuda_device, device_checks):
    from fast_infer_b200.kernels.attention import flash_attention
    torch.manual_seed(3)
    q = torch.randn(1, 4, 200, 128, device=cuda_device).half()
    k = torch.randn(1, 4, 200, 128, device=cuda_device).half()
    v = torch.randn(1, 4, 200, 128, device=cuda_device).half()
    out = flash_attention(q, k, v, sm_scale=0.05)
    _ok(out.float().cpu().numpy(), torch_causal_fp32(q, k, v, 0.05).cpu().numpy())


def test_config2_full_size(cuda_device):
    """Config 2: B4 x S2048, GQA 24/8, N(0,1) fp16 (seed 1), checked against fp32
    PyTorch on every head; plus a checksum of the output over repeated runs."""
    from fast_infer_b200.kernels.attention import flash_attention
    from oracle.attention_oracle import randn_f16
    rng = np.random.default_rng(1)
    q = _to(randn_f16(rng, (4, 24, 2048, 128)), cuda_device)
    k = _to(randn_f16(rng, (4, 8, 2048, 128)), cuda_device)
    v = _to(randn_f16(rng, (4, 8, 2048, 128)), cuda_device)
    out = flash_attention(q, k, v)
    ref = torch_causal_fp32(q, k, v)
    d = (out.float() - ref)
    max_abs = d.abs().max().item()
    rel = (d.norm() / ref.norm()).item()
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (max_abs, rel)
    for _ in range(3):  # deterministic: identical bytes run to run
        assert torch.equal(flash_attention(q, k, v), out)


@pytest.mark.parametrize("lens", [(1, 77, 128, 129, 300, 512, 0, 1000), (2048, 5, 700)])
def test_varlen_ragged_batch_vs_fp32(cuda_device, device_checks, lens):
    """Packed ragged batch (extension): every sequence equals its own causal attention."""
    from fast_infer_b200.kernels.attention import flash_attention_varlen
    torch.manual_seed(len(lens))
    T = sum(lens)
    q = torch.randn(T, 24, 128, device=cuda_device).half()
    k = torch.randn(T, 8, 128, device=cuda_device).half()
    v = torch.randn(T, 8, 128, device=cuda_device).half()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=cuda_device)
    out = flash_attention_varlen(q, k, v, cu, max(lens))
    for b, n in enumerate(lens):
        if n == 0:
            continue
        s0 = int(cu[b])
        qs = q[s0:s0 + n].transpose(0, 1)[None]
        ks = k[s0:s0 + n].transpose(0, 1)[None]
        vs = v[s0:s0 + n].transpose(0, 1)[None]
        ref = torch_causal_fp32(qs, ks, vs)[0].transpose(0, 1)
        _ok(out[s0:s0 + n].float().cpu().numpy(), ref.cpu().numpy(), f"seq {b} len {n}")


def test_varlen_equal_lengths_match_uniform_kernel(cuda_device, device_checks):
    from fast_infer_b200.kernels.attention import flash_attention, flash_attention_varlen
    torch.manual_seed(5)
    B, S = 3, 333
    q = torch.randn(B, S, 24, 128, device=cuda_device).half()
    k = torch.randn(B, S, 8, 128, device=cuda_device).half()
    v = torch.randn(B, S, 8, 128, device=cuda_device).half()
    cu = torch.arange(0, (B + 1) * S, S, dtype=torch.int32, device=cuda_device)
    o_var = flash_attention_varlen(q.reshape(B * S, 24, 128), k.reshape(B * S, 8, 128),
                                   v.reshape(B * S, 8, 128), cu, S)
    o_uni = flash_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    assert torch.equal(o_var.reshape(B, S, 24, 128), o_uni.transpose(1, 2))


@pytest.mark.parametrize("scale", [6.0, 0.05])
def test_extreme_magnitudes_vs_fp32(cuda_device, device_checks, scale):
    """Peaky softmax (large scores: many lazy-rescale events, one dominant key) and
    nearly uniform softmax (tiny scores) both stay within tolerance."""
    from fast_infer_b200.kernels.attention import flash_attention
    torch.manual_seed(11)
    q = (torch.randn(2, 6, 700, 128, device=cuda_device) * scale).half()
    k = (torch.randn(2, 2, 700, 128, device=cuda_device) * scale).half()
    v = torch.randn(2, 2, 700, 128, device=cuda_device).half()
    out = flash_attention(q, k, v)
    assert torch.isfinite(out).all()
    # The north_star bound (2e-3 / 1e-3) is specified for N(0,1) inputs. With scores
    # 36x larger the softmax is nearly one-hot over V values up to ~4, and rounding P
    # to fp16 (as every FlashAttention PV product does) alone reaches ~2e-3 absolute;
    # the bound here is 4e-3 absolute and the north_star relative-L2.
    max_abs, rel = error_stats(out.float().cpu().numpy(), torch_causal_fp32(q, k, v).cpu().numpy())
    assert max_abs <= 4e-3 and rel <= REL_L2_TOL, (scale, max_abs, rel)


def test_increasing_scores_force_rescales(cuda_device, device_checks):
    """Keys whose scores grow along the sequence make the running max rise at every
    KV tile, so the O/l rescale path runs on every step."""
    from fast_infer_b200.kernels.attention import flash_attention
    torch.manual_seed(12)
    S = 1024
    q = torch.ones(1, 2, S, 128, device=cuda_device).half() * 0.5
    ramp = torch.linspace(0, 4, S, device=cuda_device)[:, None]
    k = (torch.randn(1, 2, S, 128, device=cuda_device) * 0.1 + ramp).half()
    v = torch.randn(1, 2, S, 128, device=cuda_device).half()
    out = flash_attention(q, k, v)
    _ok(out.float().cpu().numpy(), torch_causal_fp32(q, k, v).cpu().numpy())
