"""Time the reference's own attention kernels on host cores (Triton interpreter).

Test/measurement infrastructure, not product code. The reference implements the
attention path only as Triton kernels (kernels/attention.py:8-113 prefill,
:116-233 decode); their one CPU form is the Triton interpreter
(``TRITON_INTERPRET=1``: every program of the grid executed with numpy). The
reference checkout does not travel to the GPU box, so this script runs where the
checkout is and writes ``reference_interpret_timing.json`` beside itself; the
bench reports those figures (with the host and core count they were taken on)
next to the CPU baselines it measures on the box itself.

    python oracle/time_reference_interpret.py --reference <path-to-Fast_Infer-checkout>

Workloads (shapes, seeds and length draws of the bench's configs; N(0,1) fp16):
* config 1, in full: causal prefill B1 x S128 (24 heads; K/V expanded with
  ``repeat_interleave(3)`` as model.py:110-111 does) and 16 decode steps
  (context 129..144) through ``paged_attention`` with the scalar ``num_tokens``.
* config 2, subsample: one (sequence, head) of the B4 x S2048 prefill, i.e. 1/96
  of the work; the TFLOP/s extrapolates linearly (every program of the
  reference's grid ``(B*H,)`` does the same work).
* configs 3 and 5, subsample: every 16th / 64th sequence of the ragged batch
  (4 sequences each), one ``paged_attention`` call per sequence because the
  reference has one scalar ``num_tokens`` per call (kernels/attention.py:191-233);
  the GB/s over the sample's algorithmic bytes is the rate for the whole batch
  (the interpreter's time is linear in pages x heads).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import platform
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
HQ, HKV, D, BS = 24, 8, 128, 64


def _import_reference(ref_path: str):
    os.environ["TRITON_INTERPRET"] = "1"
    tmp = tempfile.mkdtemp(prefix="fi_ref_")
    os.symlink(os.path.abspath(ref_path), os.path.join(tmp, "fast_infer"))
    sys.path.insert(0, tmp)
    from fast_infer.kernels import attention as ref_attn  # type: ignore
    return ref_attn


def ragged_lens(n, lo, hi, seed):
    """The bench's length draw (numpy default_rng(seed).integers(lo, hi + 1))."""
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).astype(np.int32)


def decode_bytes(lens, hkv=HKV):
    lens = np.asarray(lens, np.int64)
    return float(lens.sum() * hkv * D * 4 + len(lens) * 3 * hkv * D * 4 +
                 sum(math.ceil(int(n) / BS) for n in lens) * 4)


def causal_flops(b, h, s):
    return float(b) * h * 4.0 * D * s * (s + 1) / 2.0


def _cpu_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def time_prefill(ref_attn, torch, b, h, s, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, s, D, generator=g).half()
    k = torch.randn(b, h, s, D, generator=g).half()
    v = torch.randn(b, h, s, D, generator=g).half()
    t0 = time.perf_counter()
    ref_attn.flash_attention(q, k, v)
    return time.perf_counter() - t0


def time_decode_sequences(ref_attn, torch, lens, seed):
    """One reference paged_attention call per sequence (24 query heads, 8 KV heads,
    shuffled pages); returns total seconds."""
    rng = np.random.default_rng(seed)
    total = 0.0
    for n in lens:
        pages = (int(n) + BS - 1) // BS
        kc = torch.from_numpy(rng.standard_normal((pages, BS, HKV, D), dtype=np.float32)).half()
        vc = torch.from_numpy(rng.standard_normal((pages, BS, HKV, D), dtype=np.float32)).half()
        q = torch.from_numpy(rng.standard_normal((1, HQ, D), dtype=np.float32)).half()
        bt = torch.from_numpy(rng.permutation(pages).astype(np.int32)[None])
        t0 = time.perf_counter()
        ref_attn.paged_attention(q, kc, vc, bt, BS, int(n))
        total += time.perf_counter() - t0
    return total


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    ref_attn = _import_reference(args.reference)
    import torch
    import triton
    cores = os.cpu_count() or 1
    wall0, cpu0 = time.perf_counter(), time.process_time()
    out = {"what": "reference kernels/attention.py under TRITON_INTERPRET=1 on host cores",
           "host_cpu": _cpu_name(), "cores": cores,
           "threads": "numpy's default (BLAS may use every core inside tl.dot); "
                      "cpu_per_wall below = process CPU seconds / wall seconds of the run",
           "triton": triton.__version__, "torch": torch.__version__,
           "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "entries": {}}
    e = out["entries"]

    # config 1 in full
    t_pf = time_prefill(ref_attn, torch, 1, HQ, 128, 0)
    c1_lens = [129 + t for t in range(16)]
    t_dec = time_decode_sequences(ref_attn, torch, c1_lens, 0)
    e["config1_prefill"] = {"seconds": round(t_pf, 3),
                            "tflops": causal_flops(1, HQ, 128) / t_pf / 1e12,
                            "sample": "whole config-1 prefill (B1 x S128, 24 heads)",
                            "extrapolated": False}
    e["config1_decode"] = {"seconds": round(t_dec, 3),
                           "gbs": decode_bytes(c1_lens) / t_dec / 1e9,
                           "sample": "all 16 decode steps of config 1 (context 129..144)",
                           "extrapolated": False}

    # config 2: one (sequence, head) of B4 x S2048 x 24 heads
    t2 = time_prefill(ref_attn, torch, 1, 1, 2048, 1)
    frac = 1.0 / (4 * HQ)
    e["config2_prefill"] = {"seconds_sample": round(t2, 3),
                            "seconds_whole_extrapolated": round(t2 / frac, 1),
                            "tflops": causal_flops(1, 1, 2048) / t2 / 1e12,
                            "sample": "1 of the 96 (sequence, head) programs of config 2 "
                                      "(S2048); whole-config time extrapolated x96",
                            "extrapolated": True}

    # configs 3 and 5: stratified sequence samples of the bench's length draws
    for name, (n, lo, hi, seed, step) in (("config3_decode", (64, 512, 4096, 2, 16)),
                                          ("config5_decode", (256, 1024, 4096, 3, 64))):
        lens = ragged_lens(n, lo, hi, seed)
        idx = np.arange(0, n, step)
        sub = lens[idx]
        t = time_decode_sequences(ref_attn, torch, sub, seed)
        e[name] = {"seconds_sample": round(t, 3),
                   "seconds_whole_extrapolated": round(t * decode_bytes(lens) /
                                                       decode_bytes(sub), 1),
                   "gbs": decode_bytes(sub) / t / 1e9,
                   "sample": f"sequences {idx.tolist()} of {n} (lengths {sub.tolist()}), one "
                             "reference call per sequence; whole-batch time extrapolated by "
                             "algorithmic bytes",
                   "extrapolated": True}
    out["cpu_per_wall"] = round((time.process_time() - cpu0) / (time.perf_counter() - wall0), 2)
    path = HERE / "reference_interpret_timing.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
