"""Generate golden vectors by running the reference implementation itself.

Run once in a container that has the reference checkout (it is read, never
modified); the outputs are small ``.npz`` fixtures committed next to this script:

    python tests/golden/make_golden.py --reference <path-to-Fast_Infer-checkout>

The reference's Triton kernels run on CPU under ``TRITON_INTERPRET=1``; its
KV-cache methods run unchanged on CPU tensors. Inputs come from numpy's seeded
``default_rng`` so any machine regenerates them bit-identically (the tests do).

Fixtures:
* ``c1.npz``            config 1: causal prefill B1 x S128 (24/8 heads, D128,
                        seed 0) then 16 decode steps over a 64-block pool whose
                        block table is a seeded permutation.
* ``prefill_small.npz`` causal prefill, GQA 6/2 heads, D128, B2, S in {1, 77, 200}.
* ``decode_ragged.npz`` paged decode, 24/8 heads, ragged lengths incl. 0 and
                        block-boundary cases, one reference call per sequence.
* ``kv_write.npz``      block tables + pool digests after the reference model's
                        own ``_store_kv_prefill`` / ``_store_kv_decode``.
* ``rope.npz``          the reference's ``apply_rope`` (kernels/rope.py) on a 6-token
                        prefill and a decode token at position 300, with the fp16
                        cos/sin rows model.py:74-75 feeds it.
* ``rms_norm.npz``      the reference's ``rms_norm`` Triton kernel (kernels/rms_norm.py)
                        on the ``RMS_CASES`` shapes.
* ``model_forward.npz`` the reference's whole ``LlamaForCausalLM.forward`` (model.py:50-160,
                        INT4 memory mode, 2 layers of the Llama-3.2-3B shape, vocabulary
                        512): a 62-token prefill of 2 sequences and 4 decode tokens (the
                        last starts a new page). Per forward and layer it records the
                        attention inputs model.py passes (q after RoPE, k/v as stored), the
                        attention outputs, the ``num_tokens`` given to paged attention, and
                        after each forward the block table, free list, pool digests and
                        logits.
* ``int4.npz``          the reference's ``quantize_int4_groupwise`` and
                        ``dequantize_int4`` (loader.py), ``_dequant_storage`` and the
                        fused ``int4_matmul`` Triton kernel (kernels/matmul.py) on the
                        ``INT4_CASES`` shapes (ragged N, groupsize 64, a clamped group).
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.inputs import (  # noqa: E402
    DECODE_RAGGED_LENS, INT4_CASES, KV_WRITE, PREFILL_SMALL_S, RMS_CASES, ROPE_DECODE_POS,
    ROPE_PREFILL_POS, c1_inputs, decode_ragged_inputs, int4_inputs, kv_write_inputs,
    prefill_small_inputs, rms_inputs, rope_inputs)


def _import_reference(ref_path: str):
    os.environ["TRITON_INTERPRET"] = "1"
    tmp = tempfile.mkdtemp(prefix="fi_ref_")
    os.symlink(os.path.abspath(ref_path), os.path.join(tmp, "fast_infer"))
    sys.path.insert(0, tmp)
    import torch  # noqa: F401
    from fast_infer.kernels import attention as ref_attn  # type: ignore
    from fast_infer.kernels import rope as ref_rope  # type: ignore
    from fast_infer import kv_cache as ref_kv  # type: ignore
    from fast_infer import model as ref_model  # type: ignore
    return ref_attn, ref_kv, ref_model, ref_rope


def _import_reference_int4():
    from fast_infer import loader as ref_loader  # type: ignore
    from fast_infer.kernels import matmul as ref_matmul  # type: ignore
    return ref_loader, ref_matmul


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", choices=["attention", "int4", "rms_norm", "model"], default=None,
                    help="regenerate one group of fixtures (default: all)")
    args = ap.parse_args()
    ref_attn, ref_kv, ref_model, ref_rope = _import_reference(args.reference)
    import torch
    T = torch.from_numpy
    if args.only in (None, "attention"):
        _attention_fixtures(ref_attn, ref_kv, ref_model, ref_rope, torch, T)
    if args.only in (None, "int4"):
        _int4_fixtures(T)
    if args.only in (None, "rms_norm"):
        _rms_fixtures(T)
    if args.only in (None, "model"):
        _model_fixtures(ref_model, T)
    print("golden fixtures written to", HERE)


def _attention_fixtures(ref_attn, ref_kv, ref_model, ref_rope, torch, T):

    # ---- config 1 -------------------------------------------------------
    c1 = c1_inputs()
    q, k, v = T(c1["q"]), T(c1["k"]), T(c1["v"])
    G = q.shape[1] // k.shape[1]
    o_pre = ref_attn.flash_attention(q, k.repeat_interleave(G, dim=1),
                                     v.repeat_interleave(G, dim=1)).numpy()
    cache = ref_kv.KVCache(1, 8, 128, 64 * 64, 64, torch.device("cpu"))
    cache.block_table[0] = T(c1["block_table"][0])
    cache.free_blocks = []
    # prefill tokens 0..127 through the reference's own store_batch (BHSD -> SHD)
    cache.store_batch(0, 0, 0, k[0].transpose(0, 1), v[0].transpose(0, 1))
    o_dec = []
    for t in range(c1["dq"].shape[0]):
        pos = 128 + t
        cache.store(0, pos // 64, pos % 64, T(c1["dk"][t][0]), T(c1["dv"][t][0]))
        o = ref_attn.paged_attention(T(c1["dq"][t]), cache.k[0], cache.v[0],
                                     cache.block_table, 64, pos + 1)
        o_dec.append(o.numpy())
    np.savez_compressed(HERE / "c1.npz", o_prefill=o_pre, o_decode=np.stack(o_dec),
                        k_pool_sha=digest(cache.k[0].numpy()),
                        v_pool_sha=digest(cache.v[0].numpy()))

    # ---- small prefill (GQA, ragged S) ------------------------------------
    outs = {}
    for S in PREFILL_SMALL_S:
        q, k, v = (T(a) for a in prefill_small_inputs(S))
        G = q.shape[1] // k.shape[1]
        outs[f"o_S{S}"] = ref_attn.flash_attention(
            q, k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)).numpy()
    np.savez_compressed(HERE / "prefill_small.npz", **outs)

    # ---- ragged decode: one reference call per sequence --------------------
    d = decode_ragged_inputs()
    outs = []
    for b, n in enumerate(d["context_lens"]):
        o = ref_attn.paged_attention(T(d["q"][b:b + 1]), T(d["k_cache"]), T(d["v_cache"]),
                                     T(d["block_table"][b:b + 1]), 64, int(n))
        outs.append(o.numpy()[0])
    # the reference's scalar-num_tokens launch over the whole batch (num_tokens = 64)
    bt_all = d["block_table"].copy()
    o_batch64 = ref_attn.paged_attention(
        T(d["q"][2:5]), T(d["k_cache"]), T(d["v_cache"]), T(bt_all[2:5]), 64, 64).numpy()
    np.savez_compressed(HERE / "decode_ragged.npz", o=np.stack(outs), o_batch64=o_batch64)

    # ---- KV slot writes through the reference model's methods ----------------
    c = KV_WRITE
    w = kv_write_inputs()

    class Cfg:
        block_size = c["block"]

    class Stub:
        pass

    stub = Stub()
    stub.config = Cfg()
    stub.kv_cache = ref_kv.KVCache(c["layers"], c["heads"], c["head_dim"], c["max_seq_len"],
                                   c["block"], torch.device("cpu"))
    stub.kv_cache._grow_batch(c["batch"])
    M = ref_model.LlamaForCausalLM
    for layer in range(c["layers"]):
        M._store_kv_prefill(stub, layer, T(w["pk"][layer]), T(w["pv"][layer]))
    bt_after_prefill = stub.kv_cache.block_table.numpy().copy()
    stub._token_count = c["prefill"]
    for t in range(c["decode_steps"]):
        stub._token_count += 1
        for layer in range(c["layers"]):
            M._store_kv_decode(stub, layer, T(w["dk"][t, layer]), T(w["dv"][t, layer]))
    np.savez_compressed(
        HERE / "kv_write.npz",
        bt_after_prefill=bt_after_prefill,
        bt_final=stub.kv_cache.block_table.numpy(),
        num_tokens=np.int64(stub.kv_cache.num_tokens),
        free_blocks=np.array(stub.kv_cache.free_blocks, np.int64),
        k_sha=digest(stub.kv_cache.k.numpy()), v_sha=digest(stub.kv_cache.v.numpy()),
    )
    # ---- RoPE (producer of every K the slot writes store) --------------------
    r = rope_inputs()
    cos, sin = ref_rope.precompute_freqs(128, 4096, 500000.0, torch.device("cpu"))
    pos = torch.tensor(ROPE_PREFILL_POS)
    c16, s16 = cos[pos].to(torch.float16), sin[pos].to(torch.float16)
    qr, kr = ref_rope.apply_rope(T(r["q"]), T(r["k"]), c16, s16)
    dpos = torch.tensor([ROPE_DECODE_POS])
    dc16, ds16 = cos[dpos].to(torch.float16), sin[dpos].to(torch.float16)
    dqr, dkr = ref_rope.apply_rope(T(r["dq"]), T(r["dk"]), dc16, ds16)
    np.savez_compressed(HERE / "rope.npz", cos16=c16.numpy(), sin16=s16.numpy(),
                        dcos16=dc16.numpy(), dsin16=ds16.numpy(), q_rot=qr.numpy(),
                        k_rot=kr.numpy(), dq_rot=dqr.numpy(), dk_rot=dkr.numpy(),
                        cos_fp32_row300=cos[ROPE_DECODE_POS].numpy())


def _rms_fixtures(T):
    """The reference's RMSNorm Triton kernel."""
    from fast_infer.kernels import rms_norm as ref_rms  # type: ignore
    out = {}
    for rows, hidden in RMS_CASES:
        x, w = rms_inputs(rows, hidden)
        out[f"out_{rows}x{hidden}"] = ref_rms.rms_norm(T(x), T(w), 1e-5).numpy()
    np.savez_compressed(HERE / "rms_norm.npz", **out)


def _model_fixtures(ref_model, T):
    """The reference model's forward with its attention, slot writes and KV cache
    recorded at the call sites model.py:113,117,120,123-130."""
    import torch
    from fast_infer.config import LlamaConfig  # type: ignore
    from fast_infer.loader import quantize_int4_groupwise  # type: ignore
    from tests.golden.inputs import MODEL, model_token_ids, model_weights
    c = MODEL
    cfg = LlamaConfig(num_hidden_layers=c["layers"], vocab_size=c["vocab"],
                      max_seq_len=c["max_seq_len"])
    w = model_weights()
    q4 = lambda a: quantize_int4_groupwise(T(a))  # noqa: E731
    layers = []
    for lw in w["layers"]:
        layers.append({
            "input_layernorm": T(lw["input_layernorm"]),
            "post_attention_layernorm": T(lw["post_attention_layernorm"]),
            "self_attn": {n: q4(lw[n]) for n in ("q_proj", "k_proj", "v_proj", "o_proj")},
            "mlp": {n: q4(lw[n]) for n in ("gate_proj", "up_proj", "down_proj")},
        })
    embed = T(w["embed"])
    weights = {"embed_tokens": embed, "layers": layers, "norm": T(w["norm"]), "lm_head": embed}
    model = ref_model.LlamaForCausalLM(cfg, weights, device=torch.device("cpu"),
                                       memory_efficient=True)

    rec = {}
    call = {"i": 0, "layer": 0}
    orig_fa, orig_pa = ref_model.flash_attention, ref_model.paged_attention
    orig_pf, orig_dec = model._store_kv_prefill, model._store_kv_decode

    def key(name):
        return f"f{call['i']}_l{call['layer']}_{name}"

    def fa(q, k, v, sm_scale=None):
        o = orig_fa(q, k, v, sm_scale)
        rec[key("q")] = q.transpose(1, 2).contiguous().numpy()   # [B, S, Hq, D]
        rec[key("o")] = o.transpose(1, 2).contiguous().numpy()
        return o

    def pa(q, k_cache, v_cache, block_table, block_size, num_tokens, sm_scale=None):
        o = orig_pa(q, k_cache, v_cache, block_table, block_size, num_tokens, sm_scale)
        rec[key("q")] = q.contiguous().numpy()                    # [B, Hq, D]
        rec[key("o")] = o.numpy()
        rec[key("num_tokens")] = np.int64(num_tokens)
        call["layer"] += 1
        return o

    def store_pf(layer_idx, k, v):
        rec[key("k")], rec[key("v")] = k.contiguous().numpy(), v.contiguous().numpy()
        orig_pf(layer_idx, k, v)
        call["layer"] += 1

    def store_dec(layer_idx, k, v):
        rec[key("k")], rec[key("v")] = k.contiguous().numpy(), v.contiguous().numpy()
        orig_dec(layer_idx, k, v)

    ref_model.flash_attention, ref_model.paged_attention = fa, pa
    model._store_kv_prefill, model._store_kv_decode = store_pf, store_dec
    prompt, steps = model_token_ids()
    try:
        inputs = [prompt] + [steps[t] for t in range(steps.shape[0])]
        for i, ids in enumerate(inputs):
            call["i"], call["layer"] = i, 0
            logits = model.forward(T(ids))
            kv = model.kv_cache
            rec[f"f{i}_logits"] = logits.numpy()
            rec[f"f{i}_block_table"] = kv.block_table.numpy().copy()
            rec[f"f{i}_free_blocks"] = np.array(kv.free_blocks, np.int64)
            rec[f"f{i}_num_tokens"] = np.int64(kv.num_tokens)
            rec[f"f{i}_k_sha"] = digest(kv.k.numpy())
            rec[f"f{i}_v_sha"] = digest(kv.v.numpy())
    finally:
        ref_model.flash_attention, ref_model.paged_attention = orig_fa, orig_pa
    np.savez_compressed(HERE / "model_forward.npz", **rec)


def _int4_fixtures(T):
    """INT4 group-wise weights and the fused dequant-matmul."""
    ref_loader, ref_matmul = _import_reference_int4()
    out = {}
    for name, n, k, g, ms in INT4_CASES:
        w, xs, g = int4_inputs(name)
        packed, scales = ref_loader.quantize_int4_groupwise(T(w), groupsize=g)
        out[f"{name}_packed"] = packed.numpy()
        out[f"{name}_scales"] = scales.numpy()
        out[f"{name}_dequant"] = ref_loader.dequantize_int4(packed, scales, groupsize=g).numpy()
        out[f"{name}_dequant_storage"] = ref_matmul._dequant_storage(packed, scales, g).numpy()
        for m, x in xs.items():
            out[f"{name}_c_m{m}"] = ref_matmul.int4_matmul(T(x), (packed, scales),
                                                           groupsize=g).numpy()
    np.savez_compressed(HERE / "int4.npz", **out)


if __name__ == "__main__":
    main()
