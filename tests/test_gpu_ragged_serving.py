"""Ragged serving end to end (per-sequence state): prompts of different lengths
prefilled as one packed batch, K/V stored per sequence, then decode steps where
each sequence appends at its own position and attends over its own length —
checked against each sequence's own fp32 attention."""

import numpy as np
import pytest
import torch

from oracle.attention_oracle import (MAX_ABS_TOL, REL_L2_TOL, attention_fp32, error_stats,
                                     paged_attention_fp32)

pytestmark = pytest.mark.gpu


def test_packed_prefill_then_ragged_decode(cuda_device, device_checks):
    from fast_infer_b200.kernels.attention import flash_attention_varlen, paged_attention
    from fast_infer_b200.kv_cache import KVCache, store_kv_ragged
    rng = np.random.default_rng(12)
    lens = np.array([5, 64, 100, 200], np.int64)
    B, Hq, Hkv, D = len(lens), 24, 8, 128
    T = int(lens.sum())
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q = rng.standard_normal((T, Hq, D), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((T, Hkv, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((T, Hkv, D), dtype=np.float32).astype(np.float16)
    dev = cuda_device
    o = flash_attention_varlen(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                               torch.from_numpy(v).to(dev), torch.from_numpy(cu).to(dev),
                               int(lens.max())).cpu().numpy()
    for b in range(B):
        sl = slice(cu[b], cu[b + 1])
        ref = attention_fp32(q[sl].transpose(1, 0, 2)[None], k[sl].transpose(1, 0, 2)[None],
                             v[sl].transpose(1, 0, 2)[None])[0].transpose(1, 0, 2)
        max_abs, rel = error_stats(o[sl], ref)
        assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (b, max_abs, rel)

    cache = KVCache(1, Hkv, D, 512, 64, dev, num_blocks=24)
    kp = np.zeros((B, int(lens.max()), Hkv, D), np.float16)
    vp = np.zeros_like(kp)
    for b in range(B):
        kp[b, : lens[b]] = k[cu[b]:cu[b + 1]]
        vp[b, : lens[b]] = v[cu[b]:cu[b + 1]]
    store_kv_ragged(cache, 0, torch.from_numpy(kp).to(dev), torch.from_numpy(vp).to(dev),
                    np.zeros(B), lens)
    assert list(cache.seq_lens) == list(lens)
    hist_k = [kp[b, : lens[b]].copy() for b in range(B)]
    hist_v = [vp[b, : lens[b]].copy() for b in range(B)]
    for step in range(3):
        dq = rng.standard_normal((B, Hq, D), dtype=np.float32).astype(np.float16)
        dk = rng.standard_normal((B, 1, Hkv, D), dtype=np.float32).astype(np.float16)
        dv = rng.standard_normal((B, 1, Hkv, D), dtype=np.float32).astype(np.float16)
        store_kv_ragged(cache, 0, torch.from_numpy(dk).to(dev), torch.from_numpy(dv).to(dev),
                        cache.seq_lens.copy(), np.ones(B))
        out = paged_attention(torch.from_numpy(dq).to(dev), cache.k[0], cache.v[0],
                              cache.block_table, 64, 0, context_lens=cache.context_lens(B),
                              max_context_len=int(cache.seq_lens.max())).cpu().numpy()
        for b in range(B):
            hist_k[b] = np.concatenate([hist_k[b], dk[b]])
            hist_v[b] = np.concatenate([hist_v[b], dv[b]])
            n = hist_k[b].shape[0]
            pages = (n + 63) // 64
            kc = np.zeros((pages, 64, Hkv, D), np.float16)
            vc = np.zeros_like(kc)
            kc.reshape(-1, Hkv, D)[:n] = hist_k[b]
            vc.reshape(-1, Hkv, D)[:n] = hist_v[b]
            ref = paged_attention_fp32(dq[b:b + 1], kc, vc, np.arange(pages)[None],
                                       np.array([n]))
            max_abs, rel = error_stats(out[b:b + 1], ref)
            assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, (step, b, max_abs, rel)
    assert list(cache.seq_lens) == list(lens + 3)
