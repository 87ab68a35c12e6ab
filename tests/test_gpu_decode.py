"""GPU parity of paged decode attention against the reference (golden vectors) and
the fp32 oracle: max-abs <= 2e-3 and relative-L2 <= 1e-3 (north_star tolerances)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import (MAX_ABS_TOL, REL_L2_TOL, error_stats,
                                     paged_attention_fp32, slot_write)
from tests.golden.inputs import c1_inputs, decode_ragged_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _ok(out, ref, what=""):
    max_abs, rel = error_stats(out, ref)
    assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, f"{what} max_abs={max_abs} rel={rel}"


def _to(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_c1_decode_steps(cuda_device, device_checks):
    from fast_infer_b200.kernels.attention import paged_attention
    c1 = c1_inputs()
    g = np.load(GOLDEN / "c1.npz")
    NB = int(c1["num_blocks"])
    kc = np.zeros((NB, 64, 8, 128), np.float16)
    vc = np.zeros_like(kc)
    bt = c1["block_table"]
    slot_write(kc, vc, c1["k"][0].transpose(1, 0, 2)[None], c1["v"][0].transpose(1, 0, 2)[None],
               bt, np.array([0]), np.array([128]), 64)
    for t in range(c1["dq"].shape[0]):
        pos = 128 + t
        slot_write(kc, vc, c1["dk"][t][:, None], c1["dv"][t][:, None], bt, np.array([pos]),
                   np.array([1]), 64)
        out = paged_attention(_to(c1["dq"][t], cuda_device), _to(kc, cuda_device),
                              _to(vc, cuda_device), _to(bt, cuda_device), 64, pos + 1)
        out = out.cpu().numpy()
        ref32 = paged_attention_fp32(c1["dq"][t], kc, vc, bt, np.array([pos + 1]))
        _ok(out, ref32, f"step {t} vs fp32")
        _ok(out, g["o_decode"][t].astype(np.float32), f"step {t} vs reference")


@pytest.mark.parametrize("pps", [0, 1, 2, 32])
def test_ragged_lengths_vs_reference(cuda_device, device_checks, pps):
    from fast_infer_b200.kernels.attention import paged_attention
    d = decode_ragged_inputs()
    g = np.load(GOLDEN / "decode_ragged.npz")
    out = paged_attention(_to(d["q"], cuda_device), _to(d["k_cache"], cuda_device),
                          _to(d["v_cache"], cuda_device), _to(d["block_table"], cuda_device),
                          64, 0, context_lens=_to(d["context_lens"], cuda_device),
                          pages_per_split=pps).cpu().numpy()
    _ok(out, g["o"].astype(np.float32), "vs reference")
    ref32 = paged_attention_fp32(d["q"], d["k_cache"], d["v_cache"], d["block_table"],
                                 d["context_lens"])
    _ok(out, ref32, "vs fp32")
    assert not out[d["context_lens"] == 0].any()
    o64 = paged_attention(_to(d["q"][2:5], cuda_device), _to(d["k_cache"], cuda_device),
                          _to(d["v_cache"], cuda_device), _to(d["block_table"][2:5], cuda_device),
                          64, 64, pages_per_split=pps).cpu().numpy()
    _ok(o64, g["o_batch64"].astype(np.float32), "scalar num_tokens")


def _random_paged(rng, lens, hq, hkv, spare=3):
    nblk = [(int(n) + 63) // 64 for n in lens]
    NB = sum(nblk) + spare
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.full((len(lens), max(nblk) + 1), -1, np.int32)
    p = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[p:p + n]
        p += n
    q = rng.standard_normal((len(lens), hq, 128), dtype=np.float32).astype(np.float16)
    kc = rng.standard_normal((NB, 64, hkv, 128), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((NB, 64, hkv, 128), dtype=np.float32).astype(np.float16)
    return q, kc, vc, bt


def test_config3_shape_vs_fp32(cuda_device, device_checks):
    """Config 3: 64 sequences, ctx ~ U[512, 4096] (seed 2), GQA 24/8, shuffled pages."""
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(2)
    lens = rng.integers(512, 4097, size=64).astype(np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, 24, 8)
    out = paged_attention(_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
                          _to(bt, cuda_device), 64, 0, context_lens=_to(lens, cuda_device),
                          max_context_len=int(lens.max())).cpu().numpy()
    _ok(out, paged_attention_fp32(q, kc, vc, bt, lens))


@pytest.mark.parametrize("batch,hq,hkv,lo,hi,pps", [(16, 24, 8, 1024, 1280, 32),
                                                    (16, 12, 4, 1024, 1280, 0),
                                                    (16, 12, 4, 1024, 1280, 5),
                                                    (3, 24, 8, 1, 2048, 32),
                                                    (2, 6, 2, 4000, 4096, 0)])
def test_small_grids_two_page_groups(cuda_device, device_checks, batch, hq, hkv, lo, hi, pps):
    """Grids of at most one CTA per SM run two page groups per CTA, each with its own
    ring: long unsplit sequences (up to 64 pages a CTA), repeated back to back."""
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(batch * 1000 + hkv * 10 + pps)
    lens = rng.integers(lo, hi + 1, size=batch).astype(np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, hq, hkv)
    args = (_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
            _to(bt, cuda_device), 64, 0)
    outs = [paged_attention(*args, context_lens=_to(lens, cuda_device), pages_per_split=pps,
                            max_context_len=int(lens.max())) for _ in range(5)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    _ok(outs[0].cpu().numpy(), paged_attention_fp32(q, kc, vc, bt, lens))


@pytest.mark.parametrize("hq,hkv", [(8, 8), (32, 4), (24, 8), (4, 2), (3, 1), (6, 2), (12, 4)])
def test_gqa_group_sizes(cuda_device, device_checks, hq, hkv):
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(hq * 10 + hkv)
    lens = np.array([1, 64, 65, 777, 2048], np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, hq, hkv)
    out = paged_attention(_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
                          _to(bt, cuda_device), 64, 0,
                          context_lens=_to(lens, cuda_device)).cpu().numpy()
    _ok(out, paged_attention_fp32(q, kc, vc, bt, lens))


def test_stale_nonfinite_slots_do_not_leak(cuda_device, device_checks):
    """Rows past the context in the last page may hold inf/nan; the reference masks
    them on load (attention.py:164-165,180-181) and so must we."""
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(9)
    lens = np.array([70, 130, 5], np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, 24, 8)
    for b, n in enumerate(lens):
        last = bt[b, (n - 1) // 64]
        kc[last, n % 64:] = np.float16(np.inf)
        vc[last, n % 64:] = np.float16(np.nan)
    out = paged_attention(_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
                          _to(bt, cuda_device), 64, 0,
                          context_lens=_to(lens, cuda_device)).cpu().numpy()
    assert np.isfinite(out).all()
    _ok(out, paged_attention_fp32(q, kc, vc, bt, lens))


def test_strided_q_and_bad_block_table(cuda_device, device_checks):
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(4)
    lens = np.array([300, 100], np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, 24, 8)
    qbig = torch.zeros(2, 24, 256, dtype=torch.float16, device=cuda_device)
    qbig[:, :, 64:192] = _to(q, cuda_device)
    out = paged_attention(qbig[:, :, 64:192], _to(kc, cuda_device), _to(vc, cuda_device),
                          _to(bt, cuda_device), 64, 0,
                          context_lens=_to(lens, cuda_device)).cpu().numpy()
    _ok(out, paged_attention_fp32(q, kc, vc, bt, lens))
    bad = bt.copy()
    bad[0, 1] = kc.shape[0] + 5
    with pytest.raises(RuntimeError, match="outside the page pool"):
        paged_attention(_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
                        _to(bad, cuda_device), 64, 0, context_lens=_to(lens, cuda_device))


def test_config5_full_size_subsample(cuda_device):
    """Config 5 at full size (256 sequences, ctx ~ U[1024, 4096], seed 3); the fp32
    check runs on a 16-sequence subsample, the rest is checked for finiteness."""
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(3)
    lens = rng.integers(1024, 4097, size=256).astype(np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, 24, 8)
    out = paged_attention(_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
                          _to(bt, cuda_device), 64, 0, context_lens=_to(lens, cuda_device),
                          max_context_len=4096).cpu().numpy()
    assert np.isfinite(out).all()
    idx = np.arange(0, 256, 16)
    _ok(out[idx], paged_attention_fp32(q[idx], kc, vc, bt[idx], lens[idx]))


@pytest.mark.parametrize("scale", [6.0, 0.05])
def test_extreme_magnitudes(cuda_device, device_checks, scale):
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(31)
    lens = np.array([100, 1000, 3000], np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, 24, 8)
    q = (q.astype(np.float32) * scale).astype(np.float16)
    kc = (kc.astype(np.float32) * scale).astype(np.float16)
    out = paged_attention(_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
                          _to(bt, cuda_device), 64, 0, context_lens=_to(lens, cuda_device),
                          pages_per_split=4).cpu().numpy()
    assert np.isfinite(out).all()
    _ok(out, paged_attention_fp32(q, kc, vc, bt, lens))


@pytest.mark.parametrize("batch,hq,hkv,lo,hi,zeros", [
    (256, 3, 1, 1024, 4096, 0),    # config 5 with one KV head per rank (8-GPU partition)
    (16, 24, 8, 1025, 1025, 0),    # the stack's decode step
    (1, 24, 8, 8000, 8000, 0),     # one long sequence in many splits
    (2, 6, 2, 1, 70, 0),           # a few short sequences
    (40, 24, 8, 0, 300, 7),        # empty sequences among short ones
    (1280, 24, 8, 1, 200, 0),      # a wide batch of short sequences
    (33, 32, 4, 100, 2000, 3),     # GQA group of 8
])
def test_automatic_split_shapes(cuda_device, device_checks, batch, hq, hkv, lo, hi, zeros):
    """The automatic split over grids from a handful of CTAs to many waves, with empty
    sequences, one long sequence, the largest GQA group: against fp32, run twice for
    identical bits, and against a fixed 32-page split within tolerance."""
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(batch * 7 + hq + hi)
    lens = rng.integers(lo, hi + 1, size=batch).astype(np.int32)
    if zeros:
        lens[rng.choice(batch, zeros, replace=False)] = 0
    q, kc, vc, bt = _random_paged(rng, np.maximum(lens, 1), hq, hkv)
    args = (_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
            _to(bt, cuda_device), 64, 0)
    kw = dict(context_lens=_to(lens, cuda_device), max_context_len=int(lens.max()))
    out = paged_attention(*args, **kw)
    again = paged_attention(*args, **kw)
    assert torch.equal(out, again)
    o = out.cpu().numpy()
    assert not o[lens == 0].any()
    idx = np.arange(batch) if batch <= 64 else np.arange(0, batch, batch // 32)
    _ok(o[idx], paged_attention_fp32(q[idx], kc, vc, bt[idx], lens[idx]), "vs fp32")
    fixed = paged_attention(*args, pages_per_split=32, **kw).cpu().numpy()
    _ok(o.astype(np.float32), fixed.astype(np.float32), "vs fixed split")


def test_context_beyond_launch_bound(cuda_device):
    """A context longer than max_context_len is truncated to the bound's pages and
    reported as FI_DEVERR_CONTEXT_LEN."""
    from fast_infer_b200._runtime import device_checks
    from fast_infer_b200.kernels.attention import paged_attention
    rng = np.random.default_rng(5)
    lens = np.array([500, 200, 64], np.int32)
    q, kc, vc, bt = _random_paged(rng, lens, 24, 8)
    args = (_to(q, cuda_device), _to(kc, cuda_device), _to(vc, cuda_device),
            _to(bt, cuda_device), 64, 0)
    with device_checks(True):
        with pytest.raises(RuntimeError, match="context"):
            paged_attention(*args, context_lens=_to(lens, cuda_device), max_context_len=256)
    out = paged_attention(*args, context_lens=_to(lens, cuda_device),
                          max_context_len=256).cpu().numpy()
    cut = np.minimum(lens, 256)
    _ok(out, paged_attention_fp32(q, kc, vc, bt, cut))
