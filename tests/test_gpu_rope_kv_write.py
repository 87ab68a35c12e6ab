"""GPU parity of the fused RoPE + KV slot-write kernel: bit-identical to the
reference's apply_rope (golden vectors) followed by its slot writes."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import apply_rope_fp16, slot_write
from tests.golden.inputs import ROPE_DECODE_POS, rope_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _tables(dev, rows):
    """fp32 tables whose rows are exactly the fp16 values the reference used, so the
    kernel's fp16 cast reproduces them (row index = position)."""
    cos = torch.zeros(ROPE_DECODE_POS + 8, 128, dtype=torch.float32)
    sin = torch.zeros_like(cos)
    for pos, c, s in rows:
        cos[pos] = torch.from_numpy(c.astype(np.float32))
        sin[pos] = torch.from_numpy(s.astype(np.float32))
    return cos.to(dev), sin.to(dev)


def test_prefill_and_decode_bit_identical(cuda_device, device_checks):
    from fast_infer_b200.kv_cache import KVCache, rope_and_store
    g = np.load(GOLDEN / "rope.npz")
    r = rope_inputs()
    rows = [(p, g["cos16"][i], g["sin16"][i]) for i, p in enumerate(range(6))]
    rows.append((ROPE_DECODE_POS, g["dcos16"][0], g["dsin16"][0]))
    cos, sin = _tables(cuda_device, rows)
    B = 2
    rng = np.random.default_rng(32)
    v = rng.standard_normal((B, 6, 8, 128), dtype=np.float32).astype(np.float16)
    dv = rng.standard_normal((B, 1, 8, 128), dtype=np.float32).astype(np.float16)
    cache = KVCache(1, 8, 128, 512, 64, cuda_device, num_blocks=20)
    cache._grow_batch(B)
    for b in range(B):
        cache._ensure_blocks(b, ROPE_DECODE_POS // 64 + 1)
    qkv = np.concatenate([r["q"].reshape(B, 6, -1), r["k"].reshape(B, 6, -1),
                          v.reshape(B, 6, -1)], axis=-1)
    k_out = torch.empty(B, 6, 8, 128, dtype=torch.float16, device=cuda_device)
    q_rot = rope_and_store(cache, 0, torch.from_numpy(qkv).to(cuda_device), 24, cos, sin, 0,
                           k_out=k_out)
    assert np.array_equal(q_rot.cpu().numpy(), g["q_rot"])
    assert np.array_equal(k_out.cpu().numpy(), g["k_rot"])
    # decode token at position 300 via device start positions
    dqkv = np.concatenate([r["dq"].reshape(B, 1, -1), r["dk"].reshape(B, 1, -1),
                           dv.reshape(B, 1, -1)], axis=-1)
    start = torch.full((B,), ROPE_DECODE_POS, dtype=torch.int32, device=cuda_device)
    dq_rot = rope_and_store(cache, 0, torch.from_numpy(dqkv).to(cuda_device), 24, cos, sin, start)
    assert np.array_equal(dq_rot.cpu().numpy(), g["dq_rot"])
    # pool bytes: the rotated k and raw v at their slots, nothing else touched
    kc = np.zeros((20, 64, 8, 128), np.float16)
    vc = np.zeros_like(kc)
    bt = cache._bt
    slot_write(kc, vc, g["k_rot"], v, bt, np.zeros(B, np.int64), np.full(B, 6), 64)
    slot_write(kc, vc, g["dk_rot"], dv, bt, np.full(B, ROPE_DECODE_POS), np.ones(B), 64)
    torch.cuda.synchronize()
    assert np.array_equal(cache.k[0].cpu().numpy(), kc)
    assert np.array_equal(cache.v[0].cpu().numpy(), vc)


def test_random_matches_oracle_with_torch_tables(cuda_device, device_checks):
    """Longer prompt, ragged start positions, tables built like the model builds them."""
    from fast_infer_b200.kv_cache import KVCache, rope_and_store
    from fast_infer_b200.stack import precompute_freqs
    B, S, nq, nkv = 3, 70, 24, 8
    cos, sin = precompute_freqs(128, 512, 500000.0, cuda_device)
    cache = KVCache(1, nkv, 128, 512, 64, cuda_device, num_blocks=30)
    cache._grow_batch(B)
    start = np.array([0, 17, 130], np.int32)
    for b in range(B):
        cache._ensure_blocks(b, (start[b] + S + 63) // 64)
    torch.manual_seed(7)
    qkv = torch.randn(B, S, (nq + 2 * nkv) * 128, device=cuda_device).half()
    q_rot = rope_and_store(cache, 0, qkv, nq, cos, sin, torch.from_numpy(start).to(cuda_device))
    x = qkv.cpu().numpy().reshape(B, S, nq + 2 * nkv, 128)
    c16, s16 = cos.half().cpu().numpy(), sin.half().cpu().numpy()
    for b in range(B):
        pos = np.arange(start[b], start[b] + S)
        qr = apply_rope_fp16(x[b:b + 1, :, :nq], c16[pos], s16[pos])
        assert np.array_equal(q_rot[b:b + 1].cpu().numpy(), qr)
    kc = np.zeros((30, 64, nkv, 128), np.float16)
    vc = np.zeros_like(kc)
    for b in range(B):
        pos = np.arange(start[b], start[b] + S)
        kr = apply_rope_fp16(x[b:b + 1, :, nq:nq + nkv], c16[pos], s16[pos])
        slot_write(kc, vc, kr, x[b:b + 1, :, nq + nkv:], cache._bt[b:b + 1],
                   start[b:b + 1], np.array([S]), 64)
    torch.cuda.synchronize()
    assert np.array_equal(cache.k[0].cpu().numpy(), kc)
    assert np.array_equal(cache.v[0].cpu().numpy(), vc)
