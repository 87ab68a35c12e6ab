"""The allocation-free decode entry point (fi_paged_decode_noalloc) against the
regular one (fi_paged_decode with a caller workspace), through the C ABI.

fi_paged_decode_noalloc exists for callers that cannot allocate device memory
themselves (a host that links only the C library, or a runtime that forbids
allocation after start-up): its split-KV scratch is a static device array of
FI_NOALLOC_SCRATCH_BYTES shared by every call on the device. This file is named
to run last, so a failure here cannot hide results of the other tests; it also
passes when run alone in a fresh process.
"""

import numpy as np
import pytest
import torch

from oracle.attention_oracle import MAX_ABS_TOL, REL_L2_TOL, error_stats

pytestmark = pytest.mark.gpu

NOALLOC_BYTES = 16 * 1024 * 1024  # FI_NOALLOC_SCRATCH_BYTES in include/fast_infer_b200.h


def _case(dev, seed, n_seqs, lo, hi):
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n_seqs).astype(np.int32)
    nblk = [(int(n) + 63) // 64 for n in lens]
    nb = sum(nblk) + 2
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((n_seqs, max(nblk) + 1), -1, np.int32)
    p = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[p:p + n]
        p += n
    t = lambda a: torch.from_numpy(a).to(dev)
    q = torch.randn(n_seqs, 24, 128, device=dev, dtype=torch.float32).half()
    kc = torch.randn(nb, 64, 8, 128, device=dev, dtype=torch.float32).half()
    vc = torch.randn(nb, 64, 8, 128, device=dev, dtype=torch.float32).half()
    return q, kc, vc, t(bt), t(lens), int(lens.max())


def _noalloc(lib, q, kc, vc, bt, lens, max_ctx, pps, o):
    from fast_infer_b200 import _lib
    s = _lib.strides
    return lib.fi_paged_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), bt.data_ptr(), lens.data_ptr(),
        0, max_ctx, q.shape[0], q.shape[1], kc.shape[2], q.shape[2], kc.shape[0], kc.shape[1],
        bt.shape[1], s(*q.stride()), s(*kc.stride()), s(*vc.stride()), s(*o.stride()),
        s(*bt.stride()), q.shape[2] ** -0.5, pps, None, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point(cuda_device):
    """Bit-identical to fi_paged_decode with a caller workspace (same kernels, same
    split), and within the north-star tolerance of the fp32 oracle. The cases run
    large, small, then large again in one process: every call shares the static
    scratch, so the second and third calls start from what a call of another size
    left there, and must still give the same bits."""
    from fast_infer_b200 import _lib
    from fast_infer_b200.kernels.attention import (paged_attention,
                                                   paged_attention_workspace_bytes)
    from oracle.attention_oracle import paged_attention_fp32
    lib = _lib.load()
    torch.manual_seed(0)
    # Small pages_per_split forces split-KV, so the scratch is really used (need > 0).
    cases = {"large": (21, 64, 512, 4096, 4), "small": (22, 40, 100, 2000, 2)}
    first = {}
    for name in ("large", "small", "large"):
        seed, n_seqs, lo, hi, pps = cases[name]
        torch.manual_seed(seed)
        q, kc, vc, bt, lens, max_ctx = _case(cuda_device, seed, n_seqs, lo, hi)
        need = paged_attention_workspace_bytes(n_seqs, 24, 8, max_ctx, pps)
        assert 0 < need <= NOALLOC_BYTES
        ref = paged_attention(q, kc, vc, bt, 64, 0, context_lens=lens, max_context_len=max_ctx,
                              pages_per_split=pps)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, q, kc, vc, bt, lens, max_ctx, pps, out)
        assert rc == _lib.FI_OK, lib.fi_last_error()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (name, (out.float() - ref.float()).abs().max().item())
        if name in first:  # the repeat of a case gives the bits of its first run
            assert torch.equal(out, first[name]), name
            continue
        first[name] = out.clone()
        fp32 = paged_attention_fp32(q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy(),
                                    bt.cpu().numpy(), lens.cpu().numpy())
        max_abs, rel = error_stats(out.float().cpu().numpy(), fp32)
        assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (name, max_abs, rel)


def test_noalloc_rejects_sizes_beyond_static_scratch(cuda_device):
    from fast_infer_b200 import _lib
    lib = _lib.load()
    q, kc, vc, bt, lens, _ = _case(cuda_device, 23, 4, 64, 200)
    big_batch = torch.zeros(512, 24, 128, dtype=torch.float16, device=cuda_device)
    big_bt = torch.zeros(512, 64, dtype=torch.int32, device=cuda_device)
    big_lens = torch.full((512,), 4096, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(big_batch)
    # 512 sequences x 24 heads x 64 splits of partials far exceed 16 MiB
    rc = _noalloc(lib, big_batch, kc, vc, big_bt, big_lens, 4096, 1, out)
    assert rc == _lib.FI_ERR_WORKSPACE
    assert b"static scratch" in lib.fi_last_error()
