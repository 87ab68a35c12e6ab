"""GPU parity: the CUDA slot-write kernel reproduces the reference's KV-cache bytes
and block tables exactly."""

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import slot_write
from tests.golden.inputs import KV_WRITE, c1_inputs, kv_write_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _sha(t):
    return hashlib.sha256(np.ascontiguousarray(t.cpu().numpy()).tobytes()).hexdigest()


def test_model_level_writes_match_reference(cuda_device, device_checks):
    from fast_infer_b200.kv_cache import KVCache, store_kv_decode, store_kv_prefill
    c = KV_WRITE
    w = kv_write_inputs()
    g = np.load(GOLDEN / "kv_write.npz")
    cache = KVCache(c["layers"], c["heads"], c["head_dim"], c["max_seq_len"], c["block"],
                    cuda_device)
    cache._grow_batch(c["batch"])
    dev = lambda a: torch.from_numpy(a).to(cuda_device)
    for layer in range(c["layers"]):
        store_kv_prefill(cache, layer, dev(w["pk"][layer]), dev(w["pv"][layer]))
    assert np.array_equal(cache.block_table.cpu().numpy(), g["bt_after_prefill"])
    tc = c["prefill"]
    for t in range(c["decode_steps"]):
        tc += 1
        for layer in range(c["layers"]):
            store_kv_decode(cache, layer, dev(w["dk"][t, layer]), dev(w["dv"][t, layer]), tc)
    torch.cuda.synchronize()
    assert np.array_equal(cache.block_table.cpu().numpy(), g["bt_final"])
    assert cache.num_tokens == int(g["num_tokens"])
    assert cache.free_blocks == list(g["free_blocks"])
    assert _sha(cache.k) == str(g["k_sha"]) and _sha(cache.v) == str(g["v_sha"])


def test_store_batch_and_store_match_reference_pool(cuda_device, device_checks):
    from fast_infer_b200.kv_cache import KVCache
    c1 = c1_inputs()
    g = np.load(GOLDEN / "c1.npz")
    cache = KVCache(1, 8, 128, 64 * 64, 64, cuda_device)
    cache.block_table[0] = torch.from_numpy(c1["block_table"][0]).to(cuda_device)
    cache.pull_block_table()
    cache.free_blocks = []
    k = torch.from_numpy(c1["k"][0]).to(cuda_device).transpose(0, 1)  # [S, H, D] view
    v = torch.from_numpy(c1["v"][0]).to(cuda_device).transpose(0, 1)
    cache.store_batch(0, 0, 0, k, v)
    for t in range(c1["dk"].shape[0]):
        pos = 128 + t
        cache.store(0, pos // 64, pos % 64, torch.from_numpy(c1["dk"][t][0]).to(cuda_device),
                    torch.from_numpy(c1["dv"][t][0]).to(cuda_device))
    torch.cuda.synchronize()
    assert _sha(cache.k[0]) == str(g["k_pool_sha"])
    assert _sha(cache.v[0]) == str(g["v_pool_sha"])


@pytest.mark.parametrize("contiguous", [True, False])
def test_ragged_positions_bit_exact_vs_oracle(cuda_device, device_checks, contiguous):
    from fast_infer_b200.kv_cache import KVCache
    rng = np.random.default_rng(5)
    B, T, H, D, NB = 5, 70, 8, 128, 40
    cache = KVCache(2, H, D, 64 * 12, 64, cuda_device, num_blocks=NB)
    cache._grow_batch(B)
    perm = rng.permutation(NB)
    start = np.array([0, 5, 63, 64, 200], np.int32)
    n_new = np.array([70, 1, 2, 65, 0], np.int32)
    p = 0
    for b in range(B):
        nblk = (start[b] + max(n_new[b], 1) + 63) // 64
        cache._bt[b, :nblk] = perm[p:p + nblk]
        p += nblk
    cache._dirty = True
    if contiguous:
        k = torch.randn(B, T, H, D, device=cuda_device).half()
        v = torch.randn(B, T, H, D, device=cuda_device).half()
    else:  # odd strides force the element-wise path
        k = torch.randn(B, T, H, D + 1, device=cuda_device).half()[..., :D]
        v = torch.randn(B, T, H + 1, D, device=cuda_device).half()[:, :, 1:]
    cache.write_tokens(1, k, v, torch.from_numpy(start).to(cuda_device),
                       torch.from_numpy(n_new).to(cuda_device))
    kc = np.zeros((NB, 64, H, D), np.float16)
    vc = np.zeros_like(kc)
    slot_write(kc, vc, k.cpu().numpy(), v.cpu().numpy(), cache._bt, start, n_new, 64)
    assert np.array_equal(cache.k[1].cpu().numpy(), kc)
    assert np.array_equal(cache.v[1].cpu().numpy(), vc)
    assert not cache.k[0].any()


def test_invalid_block_entry_sets_device_error(cuda_device, device_checks):
    from fast_infer_b200.kv_cache import KVCache
    cache = KVCache(1, 8, 128, 256, 64, cuda_device)
    k = torch.randn(1, 3, 8, 128, device=cuda_device).half()
    with pytest.raises(RuntimeError, match="outside the page pool"):
        cache.write_tokens(0, k, k, 0)  # no block allocated: entry is -1
    assert not cache.k.any()
