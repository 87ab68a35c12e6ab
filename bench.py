"""Benchmark of the attention hot path on B200 (the driver's contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode-attention pass of the serving loop over one layer of a
config-5-shaped batch: 256 sequences, context lengths ~ U[1024, 4096] (seed 3 +
rank), GQA 24/8, head_dim 128, fp16 paged KV (block 64, shuffled block tables),
16 layers of KV cache resident in HBM (~43 GB per GPU; steps rotate layers, so
every step reads a layer larger than L2). A step writes each sequence's new
token into the cache (slot-write kernel) and runs paged decode attention (split
KV + combine). Under torchrun every rank owns its own 256 sequences (sequence
partitioning, no collective on the data path): weak scaling.

Headline ``value``: algorithmic HBM GB/s of the whole job (K/V bytes once + Q/O +
block-table entries, summed over ranks, / max-over-ranks device time).
Extra measurements on the same JSON line: the causal prefill of config 2
(B4 x S2048, TFLOP/s), decode on the config-3 shape, and the INT4 group-wise
dequant-matmul of the Llama-3.2-3B layer projections at decode batch sizes (weight
GB/s), each against the measured roofline in MEASURED_PEAKS.json; ``e2e`` through
the public API with pinned host buffers; ``cpu_baseline`` = the CPU oracle on a
bounded sample.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HQ, HKV, D, BS = 24, 8, 128, 64
DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED = 256, 1024, 4096, 3
DECODE_LAYERS = 16
C3_SEQS, C3_LO, C3_HI, C3_SEED = 64, 512, 4096, 2
PF_B, PF_S, PF_SEED = 4, 2048, 1
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per paged_decode_kernel launch on this workload's shape,
# from one ncu capture of this workload shape (evict-first K/V loads): 2.7374 GB read +
# 6.1 MB written.
DECODE_TRAFFIC_NCU = 2.737407e9 + 6.11712e6
# Memory throughput of that launch as a share of the peak ncu reports (same capture).
DECODE_DRAM_PCT_NCU = 87.0
# INT4 projections of one Llama-3.2-3B layer: (name, N = out features, K = in features).
INT4_SHAPES = (("qkv", 5120, 3072), ("o", 3072, 3072), ("gate_up", 16384, 3072),
               ("down", 3072, 8192))
INT4_LAYERS, INT4_GROUP, INT4_SEED = 8, 128, 6


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------- workloads
def ragged_lens(n, lo, hi, seed):
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).astype(np.int32)


def make_tables(lens, rng):
    nblk = [(int(x) + BS - 1) // BS for x in lens]
    total = sum(nblk)
    perm = rng.permutation(total).astype(np.int32)
    bt = np.full((len(lens), max(nblk) + 1), -1, np.int32)
    p = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[p:p + n]
        p += n
    return bt, total


def decode_bytes(lens, hkv=HKV):
    """Algorithmic HBM bytes of one decode pass over ``hkv`` KV heads (and their 3x
    query heads): every K and V byte once (fp16), Q and O (fp16) and one int32
    block-table entry per page."""
    lens = np.asarray(lens, np.int64)
    return float(lens.sum() * hkv * D * 4 + len(lens) * 3 * hkv * D * 4 +
                 sum(math.ceil(int(n) / BS) for n in lens) * 4)


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons with NVML during the timed region."""

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksThrottleReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksThrottleReasonHwThermalSlowdown", 0x40),
            "sw_power_cap": getattr(nv, "nvmlClocksThrottleReasonSwPowerCap", 0x4),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                for n, bit in names.items():
                    if r & bit:
                        self.reasons.add(n)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        med = float(np.median(self.samples)) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# --------------------------------------------------------------- our arm
class DecodeWorkload:
    def __init__(self, torch, dev, n_seqs, lo, hi, seed, layers, hkv=HKV):
        rng = np.random.default_rng(seed + 1000)
        self.lens = ragged_lens(n_seqs, lo, hi, seed)
        # the step's new token sits at position len-1 (already counted in lens)
        bt, total = make_tables(self.lens, rng)
        self.total_pages = total
        self.torch = torch
        self.layers = layers
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.hkv, self.hq = hkv, 3 * hkv
        self.k = torch.empty(layers, total, BS, hkv, D, dtype=torch.float16, device=dev)
        self.v = torch.empty_like(self.k)
        for l in range(layers):
            self.k[l].normal_(generator=g)
            self.v[l].normal_(generator=g)
        self.bt = torch.from_numpy(bt).to(dev)
        self.ctx = torch.from_numpy(self.lens).to(dev)
        self.start = (self.ctx - 1).contiguous()
        self.q = torch.randn(n_seqs, self.hq, D, device=dev, generator=g).half()
        self.kn = torch.randn(n_seqs, 1, hkv, D, device=dev, generator=g).half()
        self.vn = torch.randn(n_seqs, 1, hkv, D, device=dev, generator=g).half()
        self.max_ctx = int(self.lens.max())
        self.bytes = decode_bytes(self.lens, hkv)
        from fast_infer_b200.kernels.attention import paged_attention_workspace_bytes
        need = paged_attention_workspace_bytes(n_seqs, self.hq, hkv, self.max_ctx)
        self.ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)

    def attend(self, layer, q=None):
        from fast_infer_b200.kernels.attention import paged_attention
        return paged_attention(self.q if q is None else q, self.k[layer], self.v[layer], self.bt,
                               BS, 0, context_lens=self.ctx, max_context_len=self.max_ctx,
                               workspace=self.ws)

    def write(self, layer, kn=None, vn=None):
        from fast_infer_b200._lib import check, load, strides
        torch = self.torch
        kn = self.kn if kn is None else kn
        vn = self.vn if vn is None else vn
        kc, vc = self.k[layer], self.v[layer]
        st = load().fi_kv_write(
            kn.data_ptr(), vn.data_ptr(), kc.data_ptr(), vc.data_ptr(), self.bt.data_ptr(),
            self.start.data_ptr(), 0, None, kn.shape[0], 1, self.hkv, D, kc.shape[0], BS,
            self.bt.shape[1], strides(*kn.stride()), strides(*vn.stride()),
            strides(*kc.stride()), strides(*vc.stride()), strides(*self.bt.stride()), None,
            torch.cuda.current_stream().cuda_stream)
        check(st, "fi_kv_write")


def layer_graphs(torch, dev, fn, n):
    """fn(0..n-1) each captured into its own CUDA graph (run once on a side stream first,
    so one-time set-up stays out of the capture)."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = []
    with torch.cuda.stream(side):
        for layer in range(n):
            fn(layer)
        for layer in range(n):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                fn(layer)
            graphs.append(g)
    torch.cuda.current_stream(dev).wait_stream(side)
    return graphs


def timed(torch, fn, steps, warmup, dist=None, finish=None):
    """Device time of `steps` calls of fn(i) (CUDA events on the current stream),
    bracketed by barrier + synchronize; returns max-over-ranks milliseconds.
    ``finish`` (optional) joins side streams into the current one before the end
    event is recorded."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        fn(warmup + i)
    if finish is not None:
        finish()
    e1.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_ours(args):
    import torch
    import torch.distributed as dist_mod

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=dev)
        dist = dist_mod
    from fast_infer_b200 import _lib
    _lib.load()
    peaks, peak_kind = load_peaks()

    # ---- prefill, config 2 (B4 x S2048, 24/8, seed 1); 4 rotating input sets > L2.
    # Timed first, on its own (the burst tensor peak is its roofline), before the
    # decode legs have run the GPU for seconds.
    sets = prefill_inputs(torch, dev, 4)
    pf_steps = max(args.steps, 50)
    lib = _lib.load()
    with ClockSampler(local) as clk_pf:
        ms_pf = timed(torch, lambda i: prefill_call(torch, lib, sets[i % 4]), pf_steps,
                      args.warmup, dist) / pf_steps
    pf_flops = PF_B * HQ * 4.0 * D * PF_S * (PF_S + 1) / 2.0  # exact causal QK^T + PV
    pf_tflops = pf_flops / (ms_pf * 1e-3) / 1e12
    tc_peak = float(peaks["bf16_tflops"])
    del sets

    # ---- headline: decode step over config-5-shaped batch, one per rank
    wl = DecodeWorkload(torch, dev, DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED + rank,
                        args.layers)
    nl = args.layers

    def step(i):
        layer = i % nl
        wl.write(layer)
        wl.attend(layer)

    with ClockSampler(local) as clk:
        ms = timed(torch, step, args.steps, args.warmup, dist)
    ms_step = ms / args.steps
    total_bytes = wl.bytes
    if dist is not None:  # every rank draws its own lengths: sum the job's bytes
        t = torch.tensor([wl.bytes], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_bytes = float(t.item())
    value = total_bytes / (ms_step * 1e-3) / 1e9

    # dominant op alone (paged decode + combine), for the roofline
    ms_k = timed(torch, lambda i: wl.attend(i % nl), args.steps, args.warmup, None)
    kern_ms = ms_k / args.steps
    achieved = wl.bytes / (kern_ms * 1e-3) / 1e9
    hbm_peak = float(peaks["hbm_gbs"])

    # ---- e2e through the public API with pinned host buffers. Every step copies its
    # inputs (q and the new token's k, v) host->device and its output device->host
    # inside the timed region; the copies run on side streams with double-buffered
    # device tensors, so step i+1's upload and step i-1's download overlap step i's
    # kernels (a serving loop's natural pipeline).
    n = DECODE_SEQS
    nbuf = 2
    hq = [torch.randn(n, HQ, D).half().pin_memory() for _ in range(nbuf)]
    hk = [torch.randn(n, 1, HKV, D).half().pin_memory() for _ in range(nbuf)]
    hv = [torch.randn(n, 1, HKV, D).half().pin_memory() for _ in range(nbuf)]
    ho = [torch.empty(n, HQ, D, dtype=torch.float16).pin_memory() for _ in range(nbuf)]
    dq = [torch.empty(n, HQ, D, dtype=torch.float16, device=dev) for _ in range(nbuf)]
    dk = [torch.empty(n, 1, HKV, D, dtype=torch.float16, device=dev) for _ in range(nbuf)]
    dv = [torch.empty(n, 1, HKV, D, dtype=torch.float16, device=dev) for _ in range(nbuf)]
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_used = [torch.cuda.Event() for _ in range(nbuf)]
    issued = [False] * nbuf

    def e2e_step(i):
        slot, layer = i % nbuf, i % nl
        with torch.cuda.stream(s_in):
            if issued[slot]:
                s_in.wait_event(ev_used[slot])  # the slot's previous step has read it
            dq[slot].copy_(hq[slot], non_blocking=True)
            dk[slot].copy_(hk[slot], non_blocking=True)
            dv[slot].copy_(hv[slot], non_blocking=True)
            ev_in[slot].record(s_in)
        comp.wait_event(ev_in[slot])
        wl.write(layer, dk[slot], dv[slot])
        o = wl.attend(layer, dq[slot])
        ev_used[slot].record(comp)
        issued[slot] = True
        o.record_stream(s_out)
        s_out.wait_event(ev_used[slot])
        with torch.cuda.stream(s_out):
            ho[slot].copy_(o, non_blocking=True)

    def e2e_finish():
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)

    ms_e = timed(torch, e2e_step, args.steps, args.warmup, dist, finish=e2e_finish)
    e2e_step_ms = ms_e / args.steps
    h2d = (hq[0].numel() + hk[0].numel() + hv[0].numel()) * 2
    d2h = ho[0].numel() * 2

    # ---- decode on the config-3 shape (64 seqs, ctx U[512,4096], seed 2)
    wl3 = DecodeWorkload(torch, dev, C3_SEQS, C3_LO, C3_HI, C3_SEED + rank, 8)
    ms3 = timed(torch, lambda i: wl3.attend(i % 8), args.steps, args.warmup, dist) / args.steps
    c3_gbs = wl3.bytes / (ms3 * 1e-3) / 1e9
    del wl3

    # ---- config 5 partitioned by KV head: every rank owns 8/N KV heads (and their
    # query heads) of the same 256 sequences (seed 3 on every rank); no collective;
    # strong scaling. 4 resident layers rotated (each > L2 up to N = 8).
    kvh = None
    if HKV % world == 0:
        wl5 = DecodeWorkload(torch, dev, DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED, 4,
                             hkv=HKV // world)
        # one CUDA graph per layer (the per-rank step is ~60 us at N = 8, short enough
        # for host launch gaps to show in an eager loop)
        g5 = layer_graphs(torch, dev, wl5.attend, 4)
        ms5 = timed(torch, lambda i: g5[i % 4].replay(), args.steps, args.warmup,
                    dist) / args.steps
        del g5
        gbs5 = wl5.bytes * world / (ms5 * 1e-3) / 1e9
        kvh = {"workload": "config 5: 256 seqs, ctx U[1024,4096] (seed 3), GQA 24/8, KV heads "
                           f"sharded {HKV // world} per GPU over {world} GPU(s), paged decode "
                           "(+ combine), 4 layers rotated, one CUDA-graph replay per layer",
               "scaling": "strong", "ms": round(ms5, 4), "gbs": round(gbs5, 1),
               "frac_per_gpu": round(gbs5 / world / hbm_peak, 4),
               "tokens_per_s": round(DECODE_SEQS / (ms5 * 1e-3), 1)}
        del wl5
        kvh["vs_unsharded"] = kvh_vs_unsharded(torch, dev, rank, world, dist)

    stack = run_stack(torch, dev, rank, world, dist) if not args.no_stack else None
    int4 = run_int4(torch, dev, max(args.steps // 8, 20), args.warmup, hbm_peak,
                    cpu=(rank == 0 and world == 1 and not args.no_cpu_baseline))

    launches_per_step = 2 + (1 if _needs_combine(wl) else 0)
    result = {
        "metric": "decode-attn HBM GB/s",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 (fp32 softmax/accumulate)",
        "data": "synthetic: N(0,1) fp16 K/V/Q, seeded ragged lengths and shuffled block tables",
        "config": {
            "workload": "config5-shaped ragged paged decode per rank: 256 seqs, ctx U[1024,4096] "
                        "(seed 3+rank), GQA 24/8, D128, block 64, 16 resident layers rotated; "
                        "step = KV slot write of the new token + paged decode",
            "partition": "sequences (each rank owns 256 sequences x 8 KV heads)",
            "l2": "inputs larger than L2 (one layer of KV = %.2f GB per step)" % (wl.bytes / 1e9),
            "tokens_per_step": DECODE_SEQS * world,
        },
        "tokens_per_s": round(DECODE_SEQS * world / (ms_step * 1e-3), 1),
        "roofline": {
            "kernel": "paged_decode_kernel (+ split-KV combine)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
            "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
            "peak_source": f"{peak_kind} hbm_gbs",
            "traffic": DECODE_TRAFFIC_NCU,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch",
            "peak_note": "hbm_gbs is a read+write copy; this kernel only reads, so frac can "
                         "pass 1. Against the DRAM peak ncu reports, one launch runs at "
                         f"{DECODE_DRAM_PCT_NCU} %",
        },
        "prefill": {
            "workload": "config 2: causal prefill B4 x S2048, GQA 24/8 (K/V not expanded), D128",
            "ms": round(ms_pf, 4), "tflops": round(pf_tflops, 1),
            "roofline": {"bound": "tensor", "achieved": round(pf_tflops, 1), "peak": tc_peak,
                         "unit": "TFLOP/s", "frac": round(pf_tflops / tc_peak, 4),
                         "peak_source": f"{peak_kind} bf16_tflops (burst)"},
            "l2": "4 rotating input sets (536 MB) > L2",
            "clocks": clk_pf.summary(),
        },
        "decode_config3": {
            "workload": "config 3: 64 seqs, ctx U[512,4096] (seed 2), GQA 24/8",
            "ms": round(ms3, 4), "gbs": round(c3_gbs, 1),
            "frac": round(c3_gbs / hbm_peak, 4),
        },
        "decode_kv_head_sharded": kvh,
        "stack": stack,
        "int4_gemm": int4,
        "e2e": {
            "value": round(total_bytes / (e2e_step_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(e2e_step_ms, 5),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "public API: per step H2D of q + new k/v from pinned memory, KV slot "
                    "write, paged_attention(), D2H of the output; copies on side streams, "
                    "double-buffered so they overlap the neighbouring steps' kernels",
        },
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline_decode()
        result["cpu_baselines"] = [result["cpu_baseline"], cpu_baseline_decode_sdpa()] + (
            reference_interpret_records(["config5_decode", "config3_decode",
                                         "config1_decode"]) or [])
        result["prefill"]["cpu_baseline"] = cpu_baseline_prefill()
        result["prefill"]["cpu_baselines"] = [result["prefill"]["cpu_baseline"]] + (
            reference_interpret_records(["config2_prefill", "config1_prefill"]) or [])
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result))


# north_star tolerances (max-abs, relative L2) for the floating-point outputs
TOL_MAX_ABS, TOL_REL_L2 = 2e-3, 1e-3


def _err(torch, out, ref):
    """(max-abs, relative-L2) of out against ref, in float64."""
    o, r = out.double(), ref.double()
    den = r.norm().item()
    return (o - r).abs().max().item(), ((o - r).norm().item() / den if den > 0 else 0.0)


def _reduce(torch, dev, dist, vals, op):
    if dist is None:
        return vals
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op)
    return t.tolist()


def kvh_vs_unsharded(torch, dev, rank, world, dist):
    """Correctness of the KV-head partition on the config-5 shape: every rank runs the
    unsharded decode (8 KV heads, 24 query heads) of one layer of identical data and
    its own shard (KV heads [r*8/N, (r+1)*8/N) of the same pages, their query heads)
    through the same entry point, and compares the shard's heads with the unsharded
    output's. Outside the timed region; reduced over ranks."""
    if world == 1:
        return None
    from fast_infer_b200.kernels.attention import paged_attention
    from fast_infer_b200.shard import head_shard
    wl = DecodeWorkload(torch, dev, DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED, 1)
    full = wl.attend(0)
    sh = head_shard(rank, world, HQ, HKV)
    nkv = sh.num_kv_heads
    part = paged_attention(wl.q[:, sh.q_start:sh.q_end], wl.k[0].narrow(2, sh.kv_start, nkv),
                           wl.v[0].narrow(2, sh.kv_start, nkv), wl.bt, BS, 0,
                           context_lens=wl.ctx, max_context_len=wl.max_ctx)
    ref = full[:, sh.q_start:sh.q_end]
    torch.cuda.synchronize()
    same = 1.0 if torch.equal(part, ref) else 0.0
    max_abs, rel = _err(torch, part, ref)
    del wl
    max_abs, rel = _reduce(torch, dev, dist, [max_abs, rel], dist.ReduceOp.MAX)
    (same,) = _reduce(torch, dev, dist, [same], dist.ReduceOp.MIN)
    return {"bitexact": same == 1.0, "max_abs": max_abs, "rel_l2": rel,
            "ok": max_abs <= TOL_MAX_ABS and rel <= TOL_REL_L2,
            "what": "each rank's KV-head shard of one config-5 layer vs the unsharded decode "
                    "of the same data on that rank (worst rank)"}


def prefill_inputs(torch, dev, nsets):
    g = torch.Generator(device=dev)
    g.manual_seed(PF_SEED)
    sets = []
    for _ in range(nsets):
        q = torch.randn(PF_B, HQ, PF_S, D, device=dev, generator=g).half()
        k = torch.randn(PF_B, HKV, PF_S, D, device=dev, generator=g).half()
        v = torch.randn(PF_B, HKV, PF_S, D, device=dev, generator=g).half()
        sets.append((q, k, v, torch.empty_like(q)))
    return sets


def prefill_call(torch, lib, qkvo):
    from fast_infer_b200._lib import check, strides
    q, k, v, o = qkvo
    st = lib.fi_prefill_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), PF_B,
                            HQ, HKV, PF_S, D, strides(*q.stride()), strides(*k.stride()),
                            strides(*v.stride()), strides(*o.stride()), D ** -0.5, None,
                            torch.cuda.current_stream().cuda_stream)
    check(st, "fi_prefill_fwd")


def run_only(args):
    """One kernel family alone, for profiling (ncu) and quick sweeps."""
    import torch
    from fast_infer_b200._lib import load
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = load()
    peaks, peak_kind = load_peaks()
    out = {"only": args.only, "steps": args.steps, "warmup": args.warmup}
    if args.only == "stack":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world == 1:
            out.update(run_stack(torch, dev, 0, 1, None))
        else:  # under torchrun: one rank per GPU, rank 0 prints
            import datetime
            import torch.distributed as dist
            rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            out.update(run_stack(torch, dev, rank, world, dist))
            dist.barrier()
            dist.destroy_process_group()
            if rank != 0:
                return
    elif args.only == "int4":
        out.update(run_int4(torch, dev, args.steps, args.warmup, float(peaks["hbm_gbs"]),
                            cpu=False))
    elif args.only == "prefill":
        sets = prefill_inputs(torch, dev, 4)
        ms = timed(torch, lambda i: prefill_call(torch, lib, sets[i % 4]), args.steps,
                   args.warmup) / args.steps
        tf = PF_B * HQ * 4.0 * D * PF_S * (PF_S + 1) / 2.0 / (ms * 1e-3) / 1e12
        out.update(ms=round(ms, 4), tflops=round(tf, 1),
                   frac=round(tf / float(peaks["bf16_tflops"]), 4))
    else:
        c3 = args.only == "decode_c3"
        wl = DecodeWorkload(torch, dev, C3_SEQS if c3 else DECODE_SEQS, C3_LO if c3 else DECODE_LO,
                            C3_HI if c3 else DECODE_HI, C3_SEED if c3 else DECODE_SEED,
                            args.layers, hkv=args.hkv)
        ms = timed(torch, lambda i: wl.attend(i % args.layers), args.steps, args.warmup) / args.steps
        gbs = wl.bytes / (ms * 1e-3) / 1e9
        out.update(ms=round(ms, 4), gbs=round(gbs, 1), bytes=wl.bytes, kv_heads=args.hkv,
                   frac=round(gbs / float(peaks["hbm_gbs"]), 4))
    print(json.dumps(out))


STACK_LAYERS, STACK_BATCH, STACK_PROMPT, STACK_STEPS = 28, 16, 1024, 256


def run_stack(torch, dev, rank, world, dist, warmup=1):
    """Config 4: 28-layer attention stack (hidden 3072, 24/8 heads, RoPE 5e5, random
    N(0,0.02) fp16 weights), batch 16, prefill 1024 tokens then 256 decode steps,
    KV heads sharded over the ranks (decode: O projection sharded by head, summed over
    NVLink in the GEMM; prefill: residual stream split by token, all-to-all of head
    outputs, O projection on each rank's tokens). Returns prefill / decode tokens/s of
    the whole job."""
    from fast_infer_b200.stack import AttentionStack
    st = AttentionStack(num_layers=STACK_LAYERS, batch=STACK_BATCH,
                        max_seq_len=STACK_PROMPT + STACK_STEPS, rank=rank, world=world,
                        device=dev, seed=4)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    prompt = (torch.randn(STACK_BATCH, STACK_PROMPT, 3072, device=dev, generator=g) * 0.5).half()
    use_graph = True
    for _ in range(warmup):
        try:
            st.generate(prompt[:, :256], 4, use_graph=use_graph)
        except RuntimeError:
            st.release_graph()
            use_graph = False  # capture not possible here: time the same launches eagerly
            st.generate(prompt[:, :256], 4, use_graph=False)

    def sync_all():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_ms(ms):
        if dist is None:
            return ms
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # prefill timed three times (each pass resets the cache), median kept; the decode
    # steps continue from the last prefill
    pf = []
    for _ in range(3):
        sync_all()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        e[0].record()
        h = st.prefill(prompt)[:, -1:]
        e[1].record()
        torch.cuda.synchronize()
        pf.append(max_ms(e[0].elapsed_time(e[1])))
    pf_ms = sorted(pf)[1]
    sync_all()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    e[0].record()
    st.begin_decode(h)
    for _ in range(STACK_STEPS):
        h = st.decode_step(use_graph=use_graph)
    e[1].record()
    torch.cuda.synchronize()
    dec_ms = max_ms(e[0].elapsed_time(e[1]))
    finite = bool(torch.isfinite(h).all().item())
    peer_errors = ((st._peer.errors() if st._peer is not None else 0) |
                   (st._reduce.errors() if st._reduce is not None else 0))
    checks = stack_checks(torch, dev, rank, world, dist, st, prompt, use_graph, sync_all)
    return {
        "workload": "config 4: 28-layer attention stack (Llama-3.2-3B attention shapes, random "
                    "weights), B16, prefill 1024 then 256 decode steps, KV heads sharded over "
                    f"{world} GPU(s); decode: O projection sharded by head with the cross-rank "
                    "sum over NVLink inside the GEMM (one kernel per layer); prefill: "
                    "residual stream split by token over the ranks, NCCL all-gather of the "
                    "normalised rows for QKV and all-to-all of the head outputs for the O "
                    "projection of each rank's tokens; prefill = median of 3 timed passes",
        "scaling": "strong",
        "prefill_ms": round(pf_ms, 3),
        "prefill_tokens_per_s": round(STACK_BATCH * STACK_PROMPT / (pf_ms * 1e-3), 1),
        "decode_ms_per_step": round(dec_ms / STACK_STEPS, 4),
        "decode_tokens_per_s": round(STACK_BATCH * STACK_STEPS / (dec_ms * 1e-3), 1),
        "cuda_graph": use_graph,
        "finite": finite,
        "peer_errors": peer_errors,
        **checks,
    }


STACK_CHECK_PROMPT, STACK_CHECK_STEPS = 256, 8


def stack_checks(torch, dev, rank, world, dist, st, prompt, use_graph, sync_all):
    """Correctness of the sharded stack, outside the timed region (closes ``st``).

    * reduce_vs_nccl: after a CUDA-graph decode, one more call of the stack's
      O-projection peer reduce (layer 0's weights, seeded inputs per rank) against an
      NCCL all-reduce of the ranks' fp32 partials plus the residual (worst rank).
    * gather_bitexact (decode_exchange "gather" only): every rank's peer-memory gather
      buffer of every layer equals the NCCL all-gather of each rank's own block.
    * ranks_identical: every rank holds the same hidden state.
    * stack_vs_n1: rank 0 runs the same prompt and decode steps through an unsharded
      stack (one GPU, same seed) and compares the decode outputs. Tolerance: relative
      L2 <= 1e-3 and max-abs <= 2e-3 x max|output| (the max-abs
      scaled to the hidden state's magnitude, which grows over 28 residual layers).
    * prefill_vs_n1: the same for the prefill's output (every token of the prompt).
    At N = 1 only the stack itself ran; the entries are null."""
    from fast_infer_b200.shard import gather_heads
    from fast_infer_b200.stack import AttentionStack
    if world == 1:
        st.close()
        sync_all()
        return {"reduce_vs_nccl": None, "gather_bitexact": None, "ranks_identical": None,
                "stack_vs_n1": None, "prefill_vs_n1": None}
    pf_n = st.prefill(prompt[:, :STACK_CHECK_PROMPT]).clone()
    out_n = st.generate(prompt[:, :STACK_CHECK_PROMPT], STACK_CHECK_STEPS, use_graph=use_graph)
    reduce_check = None
    if st._reduce is not None:
        w = st.layers[0]["wo_part"]
        g = torch.Generator(device=dev)
        g.manual_seed(50 + rank)
        x = torch.randn(STACK_BATCH, w.shape[1], generator=g, device=dev).half()
        g.manual_seed(51)  # the residual stream is the same on every rank
        res = torch.randn(STACK_BATCH, w.shape[0], generator=g, device=dev).half()
        out = torch.empty_like(res)
        st._reduce.linear(x, w, res, out, 0)  # the graph's last call used buffer L-1
        ref = x.float() @ w.float().t()
        dist.all_reduce(ref)
        ref += res.float()
        max_abs, rel = _err(torch, out, ref)
        scale = ref.abs().max().item()
        max_abs, rel, scale = _reduce(torch, dev, dist, [max_abs, rel, scale], dist.ReduceOp.MAX)
        reduce_check = {"max_abs": max_abs, "rel_l2": rel, "max_abs_ref": scale,
                        "ok": rel <= TOL_REL_L2 and max_abs <= TOL_MAX_ABS * max(1.0, scale),
                        "what": "O-projection peer reduce (16 x 3072, k = 3072 / N per rank) vs "
                                "NCCL all-reduce of fp32 partials + residual, worst rank"}
    same = 1.0
    if st._peer is not None:
        w = st._peer.row_elems
        for li in range(st._peer.nbuf):
            buf = st._peer.result(li, st.batch)
            ref = gather_heads(buf[:, rank * w:(rank + 1) * w].contiguous())
            if not torch.equal(buf, ref):
                same = 0.0
    (gather_ok,) = _reduce(torch, dev, dist, [same], dist.ReduceOp.MIN)
    r0 = out_n.clone()
    dist.broadcast(r0, 0)
    (ident,) = _reduce(torch, dev, dist, [1.0 if torch.equal(r0, out_n) else 0.0],
                       dist.ReduceOp.MIN)
    had_peer = st._peer is not None
    st.close()
    del st
    torch.cuda.empty_cache()
    vs = pvs = None
    if rank == 0:
        one = AttentionStack(num_layers=STACK_LAYERS, batch=STACK_BATCH,
                             max_seq_len=STACK_PROMPT + STACK_STEPS, rank=0, world=1,
                             device=dev, seed=4)
        pf_1 = one.prefill(prompt[:, :STACK_CHECK_PROMPT])
        max_abs, rel = _err(torch, pf_n, pf_1)
        scale = pf_1.abs().max().item()
        pvs = {"max_abs": max_abs, "rel_l2": rel, "max_abs_ref": scale,
               "ok": rel <= TOL_REL_L2 and max_abs <= TOL_MAX_ABS * max(1.0, scale),
               "what": f"prefill output, every token of a {STACK_CHECK_PROMPT}-token prompt "
                       f"(B{STACK_BATCH}, 28 layers), {world}-GPU sharded stack vs one GPU"}
        del pf_1
        out_1 = one.generate(prompt[:, :STACK_CHECK_PROMPT], STACK_CHECK_STEPS,
                             use_graph=use_graph)
        max_abs, rel = _err(torch, out_n, out_1)
        scale = out_1.abs().max().item()
        vs = {"max_abs": max_abs, "rel_l2": rel, "max_abs_ref": scale,
              "ok": rel <= TOL_REL_L2 and max_abs <= TOL_MAX_ABS * max(1.0, scale),
              "what": f"decode outputs of {STACK_CHECK_STEPS} steps after a "
                      f"{STACK_CHECK_PROMPT}-token prompt (B{STACK_BATCH}, 28 layers), "
                      f"{world}-GPU sharded stack vs the unsharded stack on one GPU"}
        one.close()
        del one
        torch.cuda.empty_cache()
    sync_all()
    return {"reduce_vs_nccl": reduce_check,
            "gather_bitexact": (gather_ok == 1.0) if had_peer else None,
            "ranks_identical": ident == 1.0, "stack_vs_n1": vs, "prefill_vs_n1": pvs}


def int4_weight_bytes(n, k):
    """Bytes a dequant-matmul must read for one weight: nibbles + fp16 group scales."""
    return n * k // 2 + n * (k // INT4_GROUP) * 2


def run_int4(torch, dev, steps, warmup, hbm_peak, cpu=False, ms=(16, 1)):
    """INT4 group-wise dequant-matmul (the reference's default memory-mode projections)
    on the four projections of a Llama-3.2-3B layer, at decode batch M = 16 (config 4)
    and M = 1. Eight layers of random N(0, 0.02) weights quantized on the GPU (440 MB,
    larger than L2) are cycled; one step = all 4 x 8 projections, replayed from one
    CUDA graph. Reports weight-stream GB/s against the HBM roofline."""
    from fast_infer_b200.kernels.matmul import int4_matmul
    from fast_infer_b200.loader import quantize_int4_groupwise
    g = torch.Generator(device=dev)
    g.manual_seed(INT4_SEED)
    layers = [{name: quantize_int4_groupwise(
        (torch.randn(n, k, device=dev, generator=g) * 0.02).half(), INT4_GROUP)
        for name, n, k in INT4_SHAPES} for _ in range(INT4_LAYERS)]
    wbytes = sum(int4_weight_bytes(n, k) for _, n, k in INT4_SHAPES)
    out = {"workload": "Llama-3.2-3B layer projections qkv 5120x3072, o 3072x3072, gate_up "
                       "16384x3072, down 3072x8192, INT4 groupsize 128, 8 layers rotated "
                       "(weights > L2), one CUDA graph per step",
           "weight_bytes_per_layer": wbytes}
    for m in ms:
        xs = {name: torch.randn(m, k, device=dev, generator=g).half() for name, _, k in INT4_SHAPES}

        def body():
            for w in layers:
                for name, _, _ in INT4_SHAPES:
                    int4_matmul(xs[name], w[name], groupsize=INT4_GROUP)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            body()  # sizes the side stream's split-K workspace before capture
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                body()
        torch.cuda.current_stream(dev).wait_stream(side)
        ms_step = timed(torch, lambda i: graph.replay(), steps, warmup) / steps
        gbs = wbytes * INT4_LAYERS / (ms_step * 1e-3) / 1e9
        out[f"m{m}"] = {"us_per_layer": round(ms_step * 1e3 / INT4_LAYERS, 2),
                        "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4),
                        "launches_per_layer": len(INT4_SHAPES)}
        del graph
    if cpu:
        out["cpu_baseline"] = cpu_baseline_int4()
    return out


def cpu_baseline_int4(reps=3):
    """The CPU oracle's dequant-matmul (numpy, one thread of BLAS) on the o projection
    (3072 x 3072, M = 16): weight GB/s."""
    from oracle.int4_oracle import int4_matmul, quantize_int4_groupwise
    rng = np.random.default_rng(INT4_SEED)
    n = k = 3072
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16)
    packed, scales = quantize_int4_groupwise(w, INT4_GROUP)
    x = rng.standard_normal((16, k), dtype=np.float32).astype(np.float16)
    from threadpoolctl import threadpool_limits
    best = float("inf")
    with threadpool_limits(1):
        for _ in range(reps):
            t0 = time.perf_counter()
            int4_matmul(x, packed, scales, INT4_GROUP)
            best = min(best, time.perf_counter() - t0)
    return {"value": round(int4_weight_bytes(n, k) / best / 1e9, 3), "unit": "GB/s", "cores": 1,
            "kind": "port", "sample": "oracle int4_matmul, o projection 3072x3072, M=16"}


def _needs_combine(wl):
    from fast_infer_b200.kernels.attention import paged_attention_workspace_bytes
    return paged_attention_workspace_bytes(DECODE_SEQS, HQ, HKV, wl.max_ctx) > 0


# --------------------------------------------------------- CPU baselines
# The decode CPU baselines (the oracle port in both arms, PyTorch SDPA) run on one fixed,
# stated sample of the config-5-shaped workload: every CPU_SAMPLE_STEP-th sequence of the
# 256 (seed-3 lengths), i.e. 64 sequences whose pages and query come from per-sequence
# seeds. The port runs one worker process per host core (at most one per sequence).
CPU_SAMPLE_STEP = 4


def cpu_sample():
    """(indices, lengths) of the decode CPU sample."""
    lens = ragged_lens(DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED)
    idx = np.arange(0, DECODE_SEQS, CPU_SAMPLE_STEP)
    return idx, lens[idx]


def _ref_inputs(idx):
    """Sequence ``idx`` of the decode workload for the CPU baselines: pages and query
    from a per-sequence seed (the length is the workload's)."""
    n = int(ragged_lens(DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED)[idx])
    rng = np.random.default_rng(10_000 + idx)
    pages = (n + BS - 1) // BS
    kc = rng.standard_normal((pages, BS, HKV, D), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((pages, BS, HKV, D), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((1, HQ, D), dtype=np.float32).astype(np.float16)
    bt = rng.permutation(pages).astype(np.int32)[None]
    return q, kc, vc, bt, np.array([n], np.int32)


def _ref_worker(conn, seqs):
    """One host core: owns the sample sequences ``seqs``; runs their paged decode with
    the CPU oracle (the reference's per-page online-softmax algorithm restated in
    numpy) once per step message and replies with their algorithmic bytes."""
    from oracle.attention_oracle import paged_attention_vectorized
    inputs = [_ref_inputs(int(i)) for i in seqs]
    nbytes = sum(decode_bytes(x[4]) for x in inputs)
    conn.send("ready")
    while True:
        msg = conn.recv()
        if msg is None:
            break
        for q, kc, vc, bt, lens in inputs:
            paged_attention_vectorized(q, kc, vc, bt, BS, lens)
        conn.send(nbytes)


def cpu_decode_port(steps, warmup):
    """The oracle port on the CPU sample, one worker process per host core; returns
    (GB/s, seconds per step, workers). Workers are spawned (the caller may already
    have initialised CUDA)."""
    import multiprocessing as mp
    idx, _ = cpu_sample()
    workers = max(1, min(os.cpu_count() or 1, len(idx)))
    saved = {v: os.environ.get(v) for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS",
                                            "MKL_NUM_THREADS")}
    for var in saved:
        os.environ[var] = "1"  # the parallelism is one process per core
    ctx = mp.get_context("spawn")
    pipes, procs = [], []
    try:
        for w in range(workers):
            a, b = ctx.Pipe()
            pr = ctx.Process(target=_ref_worker, args=(b, idx[w::workers].tolist()), daemon=True)
            pr.start()
            pipes.append(a)
            procs.append(pr)
    finally:
        for var, val in saved.items():
            if val is None:
                os.environ.pop(var, None)
            else:
                os.environ[var] = val
    try:
        for c in pipes:
            c.recv()

        def step():
            for c in pipes:
                c.send(1)
            return sum(c.recv() for c in pipes)

        for _ in range(warmup):
            step()
        t0 = time.perf_counter()
        total = 0.0
        for _ in range(steps):
            total += step()
        secs = time.perf_counter() - t0
    finally:
        for c in pipes:
            c.send(None)
        for pr in procs:
            pr.join(timeout=30)
    return total / secs / 1e9, secs / max(1, steps), workers


def _sample_desc():
    idx, sub = cpu_sample()
    lens = ragged_lens(DECODE_SEQS, DECODE_LO, DECODE_HI, DECODE_SEED)
    return (f"every {CPU_SAMPLE_STEP}th sequence of the config-5-shaped decode batch "
            f"({len(idx)} of {DECODE_SEQS}, mean context {sub.mean():.0f} vs {lens.mean():.0f} "
            f"for the batch), one layer")


def cpu_baseline_decode(steps=3, warmup=1):
    """The oracle port (numpy, the reference's decode algorithm) on the CPU sample with
    every host core, the same sample and cores as the reference arm."""
    gbs, step_s, workers = cpu_decode_port(steps, warmup)
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": workers, "kind": "port",
            "sample": f"{_sample_desc()}; numpy oracle paged_attention_vectorized, one worker "
                      f"process per core; {step_s:.3f} s per pass"}


def cpu_baseline_decode_sdpa(reps=2):
    """The PyTorch SDPA CPU equivalent of the decode on the CPU sample: per sequence,
    fp32 ``scaled_dot_product_attention(enable_gqa=True)`` of its query over its
    gathered pages (all host threads); best of ``reps`` passes."""
    import torch
    ncores = os.cpu_count() or 1
    torch.set_num_threads(ncores)
    idx, _ = cpu_sample()
    data, nbytes = [], 0.0
    for i in idx:
        q, kc, vc, bt, lens = _ref_inputs(int(i))
        n = int(lens[0])
        order = torch.from_numpy(bt[0].astype(np.int64))
        k = torch.from_numpy(kc).float()[order].reshape(-1, HKV, D)[:n].transpose(0, 1)[None]
        v = torch.from_numpy(vc).float()[order].reshape(-1, HKV, D)[:n].transpose(0, 1)[None]
        data.append((torch.from_numpy(q).float()[:, :, None], k.contiguous(), v.contiguous()))
        nbytes += decode_bytes(lens)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        for q, k, v in data:
            torch.nn.functional.scaled_dot_product_attention(q, k, v, enable_gqa=True)
        best = min(best, time.perf_counter() - t0)
    return {"value": round(nbytes / best / 1e9, 4), "unit": "GB/s", "cores": ncores,
            "kind": "port",
            "sample": f"{_sample_desc()}; fp32 PyTorch scaled_dot_product_attention("
                      f"enable_gqa) per sequence over its gathered pages, best of {reps}: "
                      f"{best:.3f} s"}


def reference_interpret_records(which):
    """The reference's own Triton kernels timed under TRITON_INTERPRET=1, as recorded by
    oracle/time_reference_interpret.py where the reference checkout is (it does not
    travel to the GPU box): the host, core count and sample it states."""
    path = os.path.join(ROOT, "oracle", "reference_interpret_timing.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        rec = json.load(f)
    out = []
    for name in which:
        e = rec["entries"].get(name)
        if e is None:
            continue
        unit = "TFLOP/s" if "tflops" in e else "GB/s"
        out.append({"value": round(e["tflops"] if "tflops" in e else e["gbs"], 6), "unit": unit,
                    "cores": rec["cores"], "kind": "reference-triton-interpret",
                    "workload": name, "extrapolated": e["extrapolated"],
                    "sample": e["sample"],
                    "measured_on": f"{rec['host_cpu']} ({rec['cores']} cores; recorded "
                                   f"{rec['when']}, not this box: the reference checkout "
                                   f"stays where it was timed)"})
    return out


def cpu_baseline_prefill(reps=2):
    """The CPU equivalent of the prefill on the host cores: fp32 causal attention with
    GQA through PyTorch's scaled_dot_product_attention (all threads) on the whole
    config-2 shape; best of ``reps``, TFLOP/s of the exact causal count."""
    import torch
    ncores = os.cpu_count() or 1
    torch.set_num_threads(ncores)
    g = torch.Generator().manual_seed(PF_SEED)
    q = torch.randn(PF_B, HQ, PF_S, D, generator=g)
    k = torch.randn(PF_B, HKV, PF_S, D, generator=g)
    v = torch.randn(PF_B, HKV, PF_S, D, generator=g)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True,
                                                         enable_gqa=True)
        best = min(best, time.perf_counter() - t0)
    flops = PF_B * HQ * 4.0 * D * PF_S * (PF_S + 1) / 2.0
    return {"value": round(flops / best / 1e12, 4), "unit": "TFLOP/s", "cores": ncores,
            "kind": "port",
            "sample": f"whole config-2 prefill (B4 x S2048, 24/8 heads), fp32 PyTorch "
                      f"scaled_dot_product_attention(is_causal, enable_gqa) on the CPU, "
                      f"best of {reps}: {best:.2f} s"}


def run_reference(args):
    """Reference arm: the reference's decode algorithm on the host cores. The
    reference implements it only as a Triton kernel (its CPU form is the Triton
    interpreter, which needs the reference checkout that does not travel to this box);
    the oracle's restatement of that algorithm stands in. Each step runs the fixed CPU
    sample of the decode workload (``cpu_sample``) with one worker process per host
    core. Value = algorithmic bytes / wall time over the timed steps."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    value, step_s, workers = cpu_decode_port(args.steps, args.warmup)
    sample_desc = (f"per step {_sample_desc()}; numpy oracle paged_attention_vectorized, "
                   f"one worker process per core ({workers})")
    result = {
        "metric": "decode-attn HBM GB/s", "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (numpy)", "data": "synthetic", "impl": "reference",
        "config": {"workload": "config5-shaped ragged paged decode: 256 seqs, ctx U[1024,4096] "
                               "(seed 3), GQA 24/8, D128, block 64"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": workers,
                         "kind": "port", "sample": sample_desc},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "reference_triton_interpret": reference_interpret_records(["config5_decode"]),
    }
    print(json.dumps(result))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-stack", action="store_true", help="skip the config-4 stack section")
    ap.add_argument("--only", choices=["decode", "decode_c3", "prefill", "stack", "int4"],
                    default=None,
                    help="time one kernel family alone (profiling runs); prints one JSON line")
    ap.add_argument("--layers", type=int, default=DECODE_LAYERS,
                    help="resident KV-cache layers of the decode workload")
    ap.add_argument("--hkv", type=int, default=HKV,
                    help="KV heads of the --only decode workloads (with 3x as many query heads): "
                         "8 / N times the per-rank share of an N-GPU KV-head partition")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.only:
        run_only(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
