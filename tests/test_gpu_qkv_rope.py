"""Decode-step QKV projection with RMSNorm, RoPE and KV-cache slot writes in one
launch (fi_qkv_rope_kv_write via kv_cache.qkv_rope_store): the same bits as the two
launches it replaces — the folded-norm projection (fp16_linear_folded) followed by
rope_and_store — for the rotated q and for every K/V page of the pool, at ragged
positions that cross page boundaries, 1 to 16 sequences, 24/8 heads and the per-rank
head counts of a stack sharded over 2, 4 and 8 GPUs (12/4, 6/2, 3/1); with
FI_STATIC_WEIGHTS too."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(dev, batch, nq, nkv, seed):
    from fast_infer_b200.kernels.matmul import fold_rms_weight
    from fast_infer_b200.stack import precompute_freqs
    from fast_infer_b200.kv_cache import KVCache, permute_rope_rows
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    hidden, D = 3072, 128
    x = torch.randn(batch, 1, hidden, device=dev, generator=g).half()
    w = (torch.randn((nq + 2 * nkv) * D, hidden, device=dev, generator=g) * 0.02).half()
    nw = (1 + 0.1 * torch.randn(hidden, device=dev, generator=g)).half()
    wf = fold_rms_weight(w, nw)
    cos, sin = precompute_freqs(D, 1024, 500000.0, dev)
    caches = []
    pos = torch.randint(0, 700, (batch,), generator=g, device=dev).to(torch.int32)
    pos[0] = 63  # last row of a page
    for _ in range(2):
        c = KVCache(2, nkv, D, 1024, 64, dev, num_blocks=batch * 16 + 3)
        c._grow_batch(batch)
        for b in range(batch):
            c._ensure_blocks(b, int(pos[b]) // 64 + 1)
        c.k.normal_(generator=g)  # stale contents must be overwritten identically
        c.v.copy_(c.k)
        caches.append(c)
    caches[1].k.copy_(caches[0].k)
    caches[1].v.copy_(caches[0].v)
    return x, wf, permute_rope_rows(wf), cos, sin, pos, caches


@pytest.mark.parametrize("batch,nq,nkv", [(1, 24, 8), (5, 24, 8), (16, 24, 8), (16, 12, 4),
                                            (16, 6, 2), (16, 3, 1), (7, 3, 1)])
def test_fused_equals_projection_then_rope_store(cuda_device, batch, nq, nkv):
    from fast_infer_b200.kernels.matmul import fp16_linear_folded
    from fast_infer_b200.kv_cache import qkv_rope_store, rope_and_store
    x, wf, wr, cos, sin, pos, (ca, cb) = _setup(cuda_device, batch, nq, nkv, 100 + batch + nq)
    qkv = fp16_linear_folded(x, wf, eps=1e-5)
    qa = rope_and_store(ca, 1, qkv, nq, cos, sin, pos)
    qb = qkv_rope_store(cb, 1, x, wr, nq, cos, sin, pos, eps=1e-5)
    torch.cuda.synchronize()
    assert qb.shape == qa.shape
    assert torch.equal(qa, qb)
    assert torch.equal(ca.k, cb.k) and torch.equal(ca.v, cb.v)
    # constant weights (first tiles loaded before the dependency wait): the same bits
    qs = qkv_rope_store(cb, 1, x, wr, nq, cos, sin, pos, eps=1e-5, static_weight=True)
    torch.cuda.synchronize()
    assert torch.equal(qs, qa)
    assert torch.equal(ca.k, cb.k) and torch.equal(ca.v, cb.v)
    # the new token really landed: row pos % 64 of page block_table[b, pos // 64]
    bt = ca.block_table.cpu()
    for b in range(batch):
        p = int(pos[b])
        page = int(bt[b, p // 64])
        assert torch.equal(cb.v[1, page, p % 64], qkv[b, 0, (nq + nkv) * 128:].view(nkv, 128))
