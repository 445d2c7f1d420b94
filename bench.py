"""Benchmark of the weight-only quantized GEMV hot path on B200.

Default workload: the W8A16 lm_head GEMV with fused greedy argmax, int8 weights
[151936, 2048] with per-row bf16 scales, one step = one call at each of M = 1, 4 and 16
tokens.  The weights (311 MB) exceed the 126 MB L2, so every call streams them from HBM.
Metric: HBM GB/s of algorithmic bytes (weights + scales + activations + logits +
argmax), whole-job aggregate; µs per call is reported beside it.  The same run (one GPU)
also measures the routed NVFP4 MoE layer (512 experts x 2048 x 512, top-10 + shared
expert, M = 1 and 16) and the NVFP4 GEMV 4096 x 2048 (M = 1), each with its roofline
and CPU baseline, under ``workloads`` in the one JSON line (``--no-extra`` skips them).

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload lm_head|draft_head|nvfp4|moe|norm_gated|router|draft_step|stack]
                    [--layers L]   # stack: L MoE layers + the lm_head per step (default 48)
    python bench.py --impl reference ...   # the reference's CPU path (torch restatement)

With N > 1 (torchrun, one rank per GPU) the lm_head is vocab-sharded: each rank streams
V/N rows and computes its shard's greedy keys, and the MAX of the keys over ranks is taken
inside the same launch over NVLink peer memory (``--exchange nccl``: an NCCL MAX
all-reduce instead); strong scaling, total work fixed.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "µs/call and HBM GB/s (% of ~8 TB/s) for NVFP4 MoE & W8A16 GEMV at M=1–16"
UNIT = "GB/s"
FALLBACK_HBM = 6650.0
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload",
                    choices=["lm_head", "draft_head", "nvfp4", "moe", "norm_gated", "router",
                             "draft_step", "stack"],
                    default="lm_head")
    ap.add_argument("--ms", type=str, default=None, help="comma-separated token counts")
    ap.add_argument("--layers", type=int, default=48, help="MoE layers of --workload stack")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--moe-three", action="store_true",
                    help="MoE: the three-launch layer instead of the fused one")
    ap.add_argument("--moe-path", choices=["auto", "fused"], default="auto",
                    help="MoE one-launch layer: decode-width kernel for M = 1 (auto) or the "
                         "general one at every M (fused)")
    ap.add_argument("--no-extra", action="store_true",
                    help="default workload: skip the MoE and NVFP4 GEMV lines")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: greedy-key MAX inside the GEMV over NVLink (p2p) or by an "
                         "NCCL all-reduce")
    return ap.parse_args()


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM, "fallback (6.65 TB/s earlier pool measurement)"


def traffic_for(profile: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum of one ncu
    capture, keyed by token count) from the committed summary profiles/<profile>.md,
    whose line `traffic_bytes_per_launch: {...}` holds them; None when absent."""
    p = os.path.join(ROOT, "profiles", f"{profile}.md")
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return json.loads(line.split(":", 1)[1])
    except Exception:
        return None
    return None


# ------------------------------------------------------------------ clocks sampler
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.2)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline
def cpu_lm_head_sample(head_w, head_s, xs, rows: int, min_seconds: float):
    """The reference's CPU path (dequantise then fp32 matmul, bf16 logits, argmax; torch on
    all host threads) on the first `rows` rows, repeated for at least `min_seconds`.
    Returns (GB/s, seconds, reps, cores)."""
    from flash_next_rtxpro6000_b200 import synthetic as syn
    from oracle import cpu_path

    cores = _cpu_threads()
    w = head_w[:rows]
    s = head_s[:rows]
    K = w.shape[1]
    nbytes = sum(syn.w8_head_bytes(rows, K, x.shape[0]) for x in xs)
    for x in xs:  # warm-up
        cpu_path.lm_head_argmax(x, w, s)
    reps, t0 = 0, time.perf_counter()
    while True:
        for x in xs:
            cpu_path.lm_head_argmax(x, w, s)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return nbytes * reps / el / 1e9, el, reps, cores


def _cpu_threads():
    import torch

    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def cpu_nvfp4_sample(x, w, min_seconds: float):
    """The reference's CPU path of config 0 (dequantise + fp32 matmul, torch, all cores),
    repeated for at least min_seconds.  Returns (GB/s, seconds, calls, cores)."""
    from flash_next_rtxpro6000_b200 import synthetic as syn
    from oracle import cpu_path

    cores = _cpu_threads()
    cpu_path.nvfp4_gemv(x, w.wq, w.bs, w.gscale)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_path.nvfp4_gemv(x, w.wq, w.bs, w.gscale)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    b = syn.nvfp4_bytes(w.wq.shape[0], 2 * w.wq.shape[1], x.shape[0])
    return b * n / el / 1e9, el, n, cores


def cpu_moe_sample(layer, x, ids, wts, nbytes: int, min_seconds: float):
    """The reference's CPU path of config 2 (moe_reference restated in torch, all cores)
    on one routing, repeated for at least min_seconds (at least one call).  Returns
    (GB/s, seconds, calls, cores)."""
    from oracle import cpu_path

    cores = _cpu_threads()
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_path.moe_layer(x, ids, wts, layer)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return nbytes * n / el / 1e9, el, n, cores


def run_reference(args):
    """--impl reference: the reference's CPU path (torch dequantise-then-matmul, restated
    in oracle/cpu_path.py because the reference's source does not travel to the GPU box),
    on rank 0 with all host threads; the other ranks exit without work.  Each step is a
    bounded sample of the default workload: the first 16,384 of the lm_head's rows at
    every M.  The same run samples the MoE layer and the NVFP4 GEMV (``workloads``)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from flash_next_rtxpro6000_b200 import synthetic as syn
    from oracle import cpu_path

    cores = _cpu_threads()
    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    V = syn.VOCAB if args.workload != "draft_head" else syn.DRAFT_VOCAB
    rows = 16384
    head = syn.w8_head(rows, syn.HIDDEN, seed=0)
    xs = [syn.activations(m, seed=1) for m in Ms]
    step_bytes = sum(syn.w8_head_bytes(rows, syn.HIDDEN, m) for m in Ms)
    for _ in range(max(1, args.warmup)):
        for x in xs:
            cpu_path.lm_head_argmax(x, head.w, head.scale)
    steps = max(1, min(args.steps, 200))
    t0 = time.perf_counter()
    for _ in range(steps):
        for x in xs:
            cpu_path.lm_head_argmax(x, head.w, head.scale)
    el = time.perf_counter() - t0
    value = step_bytes * steps / el / 1e9
    sample = (f"first {rows} of {V} rows of the int8 lm_head, M={Ms}, per step; torch fp32 "
              "dequantise + matmul + bf16 round + argmax")
    res = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(el / steps * 1e3, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8/bf16", "data": "synthetic",
        "config": {"workload": f"w8a16_{args.workload}_{V}x{syn.HIDDEN}_argmax", "M": Ms},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if args.workload == "lm_head" and not args.no_extra:
        w0 = syn.nvfp4_weight(syn.NVFP4_N, syn.HIDDEN, seed=0)
        gbs, el0, n0, _ = cpu_nvfp4_sample(syn.activations(1, seed=1), w0, min_seconds=3.0)
        L = syn.moe_layer(syn.EXPERTS, syn.HIDDEN, syn.INTER, seed=0)
        moe = {}
        for M in (1, 16):
            ids, wts = syn.routing(M, E=syn.EXPERTS, seed=1000 * M)
            b = syn.moe_bytes(int(torch.unique(ids).numel()), M=M)
            g, e, n, _ = cpu_moe_sample(L, syn.activations(M, seed=3), ids, wts, b, 2.0)
            moe[str(M)] = {"value": round(g, 4), "calls": n, "seconds": round(e, 2)}
        res["workloads"] = {
            "nvfp4": {"config": {"workload": "nvfp4_gemv_4096x2048", "M": [1]},
                      "value": round(gbs, 3), "sample": f"{n0} calls in {el0:.1f} s"},
            "moe": {"config": {"workload": "nvfp4_moe_512x2048x512_top10_shared", "M": [1, 16]},
                    "per_m": moe}}
    print(json.dumps(res), flush=True)


# ------------------------------------------------------------------ our arm
def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import _lib
    from flash_next_rtxpro6000_b200 import synthetic as syn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _lib.lib()
    fx.prealloc(dev)

    if args.workload in ("lm_head", "draft_head"):
        res = bench_lm_head(args, fx, syn, dev, rank, world)
        if args.workload == "lm_head" and world == 1 and not args.no_extra:
            res["workloads"] = extra_workloads(args, fx, syn, dev)
    elif args.workload == "nvfp4":
        res = bench_nvfp4(args, fx, syn, dev)
    elif args.workload == "norm_gated":
        res = bench_norm_gated(args, fx, syn, dev)
    elif args.workload == "router":
        res = bench_router(args, fx, syn, dev)
    elif args.workload == "draft_step":
        res = bench_draft_step(args, fx, syn, dev)
    elif args.workload == "stack":
        res = bench_stack(args, fx, syn, dev)
    else:
        res = (bench_moe_sharded(args, fx, syn, dev, rank, world) if world > 1
               else bench_moe(args, fx, syn, dev))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


def _timed(fn, steps, warmup, dev, world, sampler=None):
    """Device time (ms) of `steps` calls of fn, max over ranks."""
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    # the clock sampler (a subprocess) starts before the barrier, so no rank enters the
    # timed region while another is still spawning it
    if sampler:
        sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    if world > 1:
        dist.barrier()
    ms = s.elapsed_time(e)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clocks


def _gpu_id(dev):
    import torch

    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index)


def bench_lm_head(args, fx, syn, dev, rank, world):
    import torch
    import torch.distributed as dist

    from flash_next_rtxpro6000_b200 import _lib

    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    V = syn.VOCAB if args.workload == "lm_head" else syn.DRAFT_VOCAB
    K = syn.HIDDEN
    if V % world:
        raise SystemExit(f"vocab {V} not divisible by {world} ranks")
    shard = V // world
    # every rank generates the full seeded head and keeps its own row slice
    head = syn.w8_head(V, K, seed=0)
    r0 = rank * shard
    w = head.w[r0:r0 + shard].contiguous().to(dev)
    s = head.scale[r0:r0 + shard].contiguous().to(dev)
    # weight copies rotated call by call so that at least 2x L2 of weights lie between
    # two reads of one copy (the draft head, 100 MB, and vocab shards fit in L2 alone)
    copies = max(1, -(-2 * L2_BYTES // (shard * K)))
    wl = [w] + [w.clone() for _ in range(copies - 1)]
    rot = [0]
    xs = [syn.activations(m, seed=1).to(dev) for m in Ms]
    ys = [torch.empty(m, shard, dtype=torch.bfloat16, device=dev) for m in Ms]
    ams = [torch.empty(m, dtype=torch.int64, device=dev) for m in Ms]
    keys = [torch.empty(m, dtype=torch.int64, device=dev) for m in Ms]
    lib = _lib_handle()
    import ctypes

    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    ws = _workspace(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    pdl = 1

    from flash_next_rtxpro6000_b200 import sharded

    p2p = world > 1 and args.exchange == "p2p"
    ex = sharded.PeerExchange(dev) if p2p else None

    def call(i, x):
        # the operator API's C call, with the raw key output for the sharded reduction
        wc = wl[rot[0] % copies]
        rot[0] += 1
        if p2p:  # the shard's GEMV with the greedy-key MAX over ranks in its last CTA
            rc = lib.fnx_w8a16_gemv_vocab_sharded(
                x.data_ptr(), x.stride(0), wc.data_ptr(), wc.stride(0), _lib.W_INT8,
                s.data_ptr(), _lib.SCALE_BF16_ROW, ys[i].data_ptr(), ys[i].stride(0), 0,
                ams[i].data_ptr(), r0, x.shape[0], shard, K, ex.buf, None, ctypes.byref(ws.c),
                pdl, stream)
            if rc:
                raise RuntimeError(_lib.last_error())
            return
        rc = lib.fnx_w8a16_gemv(
            x.data_ptr(), x.stride(0), wc.data_ptr(), wc.stride(0), _lib.W_INT8, s.data_ptr(),
            _lib.SCALE_BF16_ROW, ys[i].data_ptr(), ys[i].stride(0), None, 0, 0, 0,
            ams[i].data_ptr() if world == 1 else None,
            keys[i].data_ptr() if world > 1 else None, r0, x.shape[0], shard, K, None,
            ctypes.byref(ws.c), pdl, stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    def step():
        for i, x in enumerate(xs):
            call(i, x)
            if world > 1 and not p2p:
                dist.all_reduce(keys[i], op=dist.ReduceOp.MAX)
                lib.fnx_argmax_decode(keys[i].data_ptr(), ams[i].data_ptr(), x.shape[0], stream)

    # per-M kernel durations (for the roofline and µs/call): back-to-back launches
    per_m = {}
    for i, x in enumerate(xs):
        reps = max(50, args.steps // 4)
        ms_i, _ = _timed(lambda: call(i, x), reps, max(3, args.warmup // 4), dev, world)
        per_m[Ms[i]] = ms_i / reps * 1e3  # µs per launch
    sampler = ClockSampler(_gpu_id(dev)) if rank == 0 else None
    ms, clocks = _timed(step, args.steps, max(3, args.warmup), dev, world, sampler)
    total_bytes_step = sum(syn.w8_head_bytes(V, K, m) for m in Ms)
    value = total_bytes_step * args.steps / (ms / 1e3) / 1e9
    peak, peak_src = measured_peak()
    # roofline of the GEMV kernel: per-launch algorithmic bytes of this rank's shard
    kbytes = sum(syn.w8_head_bytes(shard, K, m) for m in Ms)
    kus = sum(per_m.values())
    achieved = kbytes / (kus * 1e-6) / 1e9
    traffic = traffic_for(f"dense_gemv_int8_{args.workload}")
    tr = None
    if traffic and world == 1:
        got = [traffic[str(m)] for m in Ms if str(m) in traffic]
        tr = round(sum(got) / len(got)) if got else None
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8/bf16 (fp32 accumulate)", "data": "synthetic",
        "config": {"workload": f"w8a16_{args.workload}_{V}x{K}_argmax", "M": Ms,
                   "weights": "int8 per-row bf16 scale",
                   "l2": f"{copies} weight cop{'y' if copies == 1 else 'ies'} of "
                         f"{shard * K / 1e6:.0f} MB rotated per call (>= 2x the 126 MB L2 "
                         "between reads of one copy), no flush",
                   "parallelism": (f"vocab-sharded x{world}, greedy-key MAX over NVLink peer "
                                   "memory inside the GEMV" if p2p else
                                   f"vocab-sharded x{world} + NCCL MAX all-reduce of argmax keys")
                   if world > 1 else "single GPU"},
        "us_per_call": {str(m): round(v, 3) for m, v in per_m.items()},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": tr, "peak_source": peak_src,
                     "kernel": "dense_gemv_kernel<int8>", "bytes_per_launch_avg": kbytes // len(Ms)},
        "clocks": clocks,
        "gpu_launches": args.steps * len(Ms) * (2 if world > 1 and not p2p else 1),
    }
    if not args.no_e2e:
        res["e2e"] = e2e_lm_head(args, fx, syn, dev, wl, s, Ms, world, rank, r0, shard, V, K,
                                 ex)
    if ex is not None:
        ex.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, el, reps, cores = cpu_lm_head_sample(head.w, head.scale, [x.cpu() for x in xs],
                                                  rows=16384, min_seconds=10.0)
        res["cpu_baseline"] = {"value": round(gbs, 3), "unit": UNIT, "cores": cores,
                               "kind": "port",
                               "sample": f"16384 of {V} rows, M={Ms}, {reps} reps in {el:.1f} s "
                                         "(torch fp32 dequantise+matmul, bf16 round, argmax, "
                                         "all host threads)"}
    return res


def extra_workloads(args, fx, syn, dev):
    """The MoE layer (M = 1, 16) and the NVFP4 GEMV (M = 1) of the default run."""
    import copy

    out = {}
    a = copy.copy(args)
    a.ms = "1,16"
    out["moe"] = bench_moe(a, fx, syn, dev, cpu=not args.no_cpu_baseline)
    a.ms = "1"
    out["nvfp4"] = bench_nvfp4(a, fx, syn, dev, cpu=not args.no_cpu_baseline)
    for k in ("metric", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "data"):
        for v in out.values():
            v.pop(k, None)
    return out


def _lib_handle():
    from flash_next_rtxpro6000_b200 import _lib

    return _lib.lib()


def e2e_lm_head(args, fx, syn, dev, wl, s, Ms, world, rank, r0, shard, V, K, ex=None):
    """Public API end to end: pinned host x -> device, w8a16_gemv(argmax_out=...),
    argmax -> pinned host, one host sync per step."""
    import torch
    import torch.distributed as dist

    hx = [syn.activations(m, seed=1).pin_memory() for m in Ms]
    dx = [torch.empty(m, K, dtype=torch.bfloat16, device=dev) for m in Ms]
    dam = [torch.empty(m, dtype=torch.int64, device=dev) for m in Ms]
    ham = [torch.empty(m, dtype=torch.int64).pin_memory() for m in Ms]
    ys = [torch.empty(m, shard, dtype=torch.bfloat16, device=dev) for m in Ms]
    from flash_next_rtxpro6000_b200 import sharded

    rot = [0]

    def step():
        for i, m in enumerate(Ms):
            w = wl[rot[0] % len(wl)]  # rotated like the device-timed calls
            rot[0] += 1
            dx[i].copy_(hx[i], non_blocking=True)
            if world == 1:
                fx.w8a16_gemv(dx[i], w, s, out=ys[i], argmax_out=dam[i], pdl=True)
            elif ex is not None:
                sharded.vocab_sharded_lm_head(dx[i], w, s, r0, ex, out=ys[i], argmax_out=dam[i])
            else:
                sharded.sharded_lm_head_argmax(dx[i], w, s, r0, out=ys[i], argmax_out=dam[i])
            ham[i].copy_(dam[i], non_blocking=True)
        torch.cuda.current_stream().synchronize()

    steps = max(20, args.steps // 4)
    ms, _ = _timed(step, steps, max(3, args.warmup // 4), dev, world)
    total = sum(syn.w8_head_bytes(V, K, m) for m in Ms)
    return {"value": round(total * steps / (ms / 1e3) / 1e9, 2), "unit": UNIT,
            "h2d_bytes_per_step": sum(m * K * 2 for m in Ms),
            "d2h_bytes_per_step": sum(m * 8 for m in Ms), "steps": steps}


def _graph_of(calls, warm=3):
    """Capture a list of zero-argument launches into one CUDA graph (after warm-up)."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warm):
            for c in calls:
                c()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    torch.cuda.synchronize()
    return g


def _roofline_per_m(per_m, peak, src, kernel, traffic_key=None, traffic_per_m=None):
    """Roofline object of a workload measured at several M: achieved = total algorithmic
    bytes / total launch time over the M values; per-M achieved / frac (and ncu traffic
    where captured) beside it; traffic = ncu DRAM bytes per launch from profiles/,
    averaged over the M values, when every M value has a capture, else None."""
    tot_b = sum(v["bytes_per_call"] for v in per_m.values())
    tot_us = sum(v["us_per_call"] for v in per_m.values())
    ach = tot_b / (tot_us * 1e-6) / 1e9
    tr = traffic_per_m if traffic_per_m is not None else (traffic_for(traffic_key) if traffic_key else None)
    tr = tr or {}
    got = [tr[m] for m in per_m if m in tr]
    traffic = round(sum(got) / len(got)) if got and len(got) == len(per_m) else None
    return {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
            "frac": round(ach / peak, 4), "traffic": traffic, "peak_source": src,
            "kernel": kernel, "bytes_per_launch_avg": tot_b // len(per_m),
            "per_m": {m: dict({"achieved": v["GBps"], "frac": round(v["GBps"] / peak, 4)},
                              **({"traffic": tr[m]} if m in tr else {}))
                      for m, v in per_m.items()}}


def bench_nvfp4(args, fx, syn, dev, cpu=False):
    """Config 0 (NVFP4 4096 x 2048): 64 weight copies rotated (> 4x L2) inside one CUDA
    graph, so the timing is device time, not Python dispatch."""
    import torch

    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    copies = 64
    host = [syn.nvfp4_weight(syn.NVFP4_N, syn.HIDDEN, seed=i) for i in range(copies)]
    ws = [(w.wq.to(dev), w.bs.to(dev), w.gscale.to(dev)) for w in host]
    peak, src = measured_peak()
    per_m, total_bytes, total_ms = {}, 0, 0.0
    sampler = ClockSampler(_gpu_id(dev))
    clocks = None
    launches = 0
    for M in Ms:
        x = syn.activations(M, seed=1).to(dev)
        y = torch.empty(M, syn.NVFP4_N, dtype=torch.bfloat16, device=dev)
        calls = [(lambda w=w: fx.w4a16_nvfp4_gemv(x, w[0], w[1], w[2], out=y, pdl=True))
                 for w in ws]
        g = _graph_of(calls)
        reps = max(3, args.steps // copies)
        ms, ck = _timed(g.replay, reps, max(3, args.warmup // copies), dev, 1,
                        sampler if M == Ms[-1] else None)
        clocks = ck or clocks
        us = ms / (reps * copies) * 1e3
        b = syn.nvfp4_bytes(syn.NVFP4_N, syn.HIDDEN, M)
        per_m[str(M)] = {"us_per_call": round(us, 3), "GBps": round(b / (us * 1e-6) / 1e9, 1),
                         "bytes_per_call": b}
        total_bytes += b * reps * copies
        total_ms += ms
        launches += reps * copies  # one GEMV launch per call
        del g
    value = total_bytes / (total_ms / 1e3) / 1e9
    res = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "nvfp4/bf16 (fp32 accumulate)", "data": "synthetic",
           "config": {"workload": "nvfp4_gemv_4096x2048", "M": Ms,
                      "l2": f"{copies} weight copies rotated in one CUDA graph (> 4x L2)"},
           "per_m": per_m,
           "roofline": _roofline_per_m(per_m, peak, src, "dense_gemv_kernel<nvfp4>",
                                       "dense_gemv_nvfp4_config0"),
           "clocks": clocks, "gpu_launches": launches}
    if cpu:
        x = syn.activations(Ms[0], seed=1)
        gbs, el, n, cores = cpu_nvfp4_sample(x, host[0], min_seconds=3.0)
        res["cpu_baseline"] = {"value": round(gbs, 3), "unit": UNIT, "cores": cores,
                               "kind": "port",
                               "sample": f"M={Ms[0]}, {n} calls in {el:.1f} s (torch fp32 "
                                         "dequantise + matmul, bf16 out, all host threads)"}
    return res


def bench_norm_gated(args, fx, syn, dev):
    """The fused gated-RMSNorm GEMV at the reference's out_proj shape
    (kernels/microbench/h1/h1_check.py:21-27: N = 2560, K = 48 x 128, group 128, fp8
    weights with fp32 per-row scales, sigmoid gate): 12 weight copies rotated (> L2)
    inside one CUDA graph.  `plain_gemv_us` is the same GEMV without the norm."""
    import torch

    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    N, K, G, copies = 2560, 48 * 128, 128, 12
    gen = torch.Generator().manual_seed(0)
    ws = [((torch.randn(N, K, generator=gen) * 64).to(torch.float8_e4m3fn)).to(dev)
          for _ in range(copies)]
    s = (torch.rand(N, generator=gen) / 448).to(dev)
    nw = (torch.randn(G, generator=gen) * 0.3 + 1.0).bfloat16().to(dev)
    peak, src = measured_peak()
    per_m, total_bytes, total_ms = {}, 0, 0.0
    sampler = ClockSampler(_gpu_id(dev))
    clocks = None
    launches = 0  # both timed variants: one launch per call each
    for M in Ms:
        x = (torch.randn(M, K, generator=gen) * 0.5).bfloat16().to(dev)
        z = (torch.randn(M, K, generator=gen) * 0.5).bfloat16().to(dev)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        reps = max(3, args.steps // copies)
        res = {}
        for name, fn in (("norm", lambda w: fx.w8a16_gemv_norm_gated(
                              x, w, s, z, nw, G, 1e-6, sigmoid_gate=True, out=y)),
                         ("plain", lambda w: fx.w8a16_gemv(x, w, s, out=y))):
            g = _graph_of([(lambda w=w: fn(w)) for w in ws])
            ms, ck = _timed(g.replay, reps, max(3, args.warmup // copies), dev, 1,
                            sampler if (M == Ms[-1] and name == "norm") else None)
            clocks = ck or clocks
            res[name] = (ms, ms / (reps * copies) * 1e3)
            launches += reps * copies
            del g
        b = N * K + 4 * N + 2 * G + 4 * M * K + 2 * M * N
        us = res["norm"][1]
        per_m[str(M)] = {"us_per_call": round(us, 3), "GBps": round(b / (us * 1e-6) / 1e9, 1),
                         "plain_gemv_us": round(res["plain"][1], 3)}
        total_bytes += b * reps * copies
        total_ms += res["norm"][0]
    value = total_bytes / (total_ms / 1e3) / 1e9
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8/bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": "w8a16_norm_gated_2560x6144_g128", "M": Ms,
                       "l2": f"{copies} weight copies rotated in one CUDA graph (> L2)"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(value / peak, 4), "traffic": None, "peak_source": src},
            "clocks": clocks, "gpu_launches": launches}


def bench_router(args, fx, syn, dev):
    """The fused MoE router (router GEMV 512 x 2048 bf16 + softmax top-10, renormalised)
    at the draft MoE's shape: 128 router-weight copies (256 MB, > 2x L2) rotated inside
    one CUDA graph.  `unfused_us` is router_gemv + route_softmax_fast (two launches)."""
    import torch

    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    E, K, k, copies = syn.EXPERTS, syn.HIDDEN, 10, 128
    gen = torch.Generator().manual_seed(0)
    ws = [((torch.randn(E, K, generator=gen) * 0.05).bfloat16()).to(dev) for _ in range(copies)]
    peak, src = measured_peak()
    per_m, total_bytes, total_ms = {}, 0, 0.0
    sampler = ClockSampler(_gpu_id(dev))
    clocks = None
    launches = 0  # fused: one launch per call; unfused: router_gemv + softmax top-k
    for M in Ms:
        x = syn.activations(M, seed=1).to(dev)
        reps = max(3, args.steps // copies)
        res = {}
        for name, fn in (("fused", lambda w: fx.router_topk(x, w, None, k, True, pdl=True)),
                         ("unfused", lambda w: fx.route_softmax_fast(
                             fx.router_gemv(x, w, pdl=True), None, k, True, pdl=True))):
            g = _graph_of([(lambda w=w: fn(w)) for w in ws])
            ms, ck = _timed(g.replay, reps, max(3, args.warmup // copies), dev, 1,
                            sampler if (M == Ms[-1] and name == "fused") else None)
            clocks = ck or clocks
            res[name] = (ms, ms / (reps * copies) * 1e3)
            launches += reps * copies * (1 if name == "fused" else 2)
            del g
        b = 2 * E * K + 2 * M * K + 4 * M * E + 8 * M * k
        us = res["fused"][1]
        per_m[str(M)] = {"us_per_call": round(us, 3), "GBps": round(b / (us * 1e-6) / 1e9, 1),
                         "unfused_us": round(res["unfused"][1], 3)}
        total_bytes += b * reps * copies
        total_ms += res["fused"][0]
    value = total_bytes / (total_ms / 1e3) / 1e9
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"router_topk_{E}x{K}_top{k}", "M": Ms,
                       "l2": f"{copies} router-weight copies rotated in one CUDA graph (> 2x L2)"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(value / peak, 4), "traffic": None, "peak_source": src},
            "clocks": clocks, "gpu_launches": launches}


def bench_draft_step(args, fx, syn, dev):
    """The greedy draft step at the draft head's shape (49,152-token hot vocabulary, int8
    49152 x 2048): draft_head_topk1 (GEMV + argmax + token map + draft_tokens + positions
    in one launch) against w8a16_gemv followed by draft_topk1_postprocess (`unfused_us`).
    3 weight copies (> 2x L2) rotated inside one CUDA graph."""
    import torch

    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    V, K, copies = syn.DRAFT_VOCAB, syn.HIDDEN, 3
    head = syn.w8_head(V, K, seed=0)
    ws = [head.w.to(dev)] + [head.w.to(dev) for _ in range(copies - 1)]
    s = head.scale.to(dev)
    hot = (torch.randperm(V, generator=torch.Generator().manual_seed(1)) + 1000).to(dev)
    peak, src = measured_peak()
    per_m, total_bytes, total_ms = {}, 0, 0.0
    sampler = ClockSampler(_gpu_id(dev))
    clocks = None
    launches = 0  # fused: one launch per call; unfused: GEMV + draft_topk1
    for M in Ms:
        x = syn.activations(M, seed=1).to(dev)
        pos = torch.zeros(M, dtype=torch.int64, device=dev)
        dt = torch.zeros(M, 8, dtype=torch.int64, device=dev)
        y = torch.empty(M, V, dtype=torch.bfloat16, device=dev)
        n = 12  # calls per graph, rotating the copies
        reps = max(3, args.steps // n)
        res = {}
        for name, fn in (("fused", lambda w: fx.draft_head_topk1(x, w, s, pos, dt, 1, hot,
                                                                 out=y, pdl=True)),
                         ("unfused", lambda w: fx.draft_topk1_postprocess(
                             fx.w8a16_gemv(x, w, s, out=y, pdl=True), pos, dt, 1, hot,
                             pdl=True))):
            g = _graph_of([(lambda w=ws[i % copies]: fn(w)) for i in range(n)])
            ms, ck = _timed(g.replay, reps, max(3, args.warmup // n), dev, 1,
                            sampler if (M == Ms[-1] and name == "fused") else None)
            clocks = ck or clocks
            res[name] = (ms, ms / (reps * n) * 1e3)
            launches += reps * n * (1 if name == "fused" else 2)
            del g
        b = syn.w8_head_bytes(V, K, M) + 8 * V  # + the token map
        us = res["fused"][1]
        per_m[str(M)] = {"us_per_call": round(us, 3), "GBps": round(b / (us * 1e-6) / 1e9, 1),
                         "unfused_us": round(res["unfused"][1], 3)}
        total_bytes += b * reps * n
        total_ms += res["fused"][0]
    value = total_bytes / (total_ms / 1e3) / 1e9
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8/bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"draft_step_{V}x{K}_hot_map", "M": Ms,
                       "l2": f"{copies} weight copies rotated in one CUDA graph (> 2x L2)"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(value / peak, 4), "traffic": None, "peak_source": src},
            "clocks": clocks, "gpu_launches": launches}


def bench_moe(args, fx, syn, dev, cpu=False):
    """Config 2 (NVFP4 MoE, 512 experts, top-10 + shared expert).  48 routings rotate over
    shifted expert sets (> 4x L2 across the rotation) inside one CUDA graph.  The layer
    runs as one fused launch (``--moe-three`` times the three-launch form instead)."""
    import torch

    from flash_next_rtxpro6000_b200.w4a16_nvfp4_gemv import swizzle_blockscale

    Ms = [int(m) for m in (args.ms or "1,2,4,8,16").split(",")]
    L = syn.moe_layer(syn.EXPERTS, syn.HIDDEN, syn.INTER, seed=0)
    d = dict(w13=L.w13.to(dev), s13=swizzle_blockscale(L.s13.to(dev)), g13=L.g13.to(dev),
             w2=L.w2.to(dev), s2=swizzle_blockscale(L.s2.to(dev)), g2=L.g2.to(dev))
    shared = fx.SharedExpert(L.sh_w13.to(dev), swizzle_blockscale(L.sh_s13.to(dev)),
                             L.sh_g13.to(dev), L.sh_w2.to(dev), swizzle_blockscale(L.sh_s2.to(dev)),
                             L.sh_g2.to(dev))
    fused = not args.moe_three
    ws = fx.make_workspace(num_routes=10, hidden_size=syn.HIDDEN, intermediate_size=syn.INTER,
                           device=dev, fused=fused)
    prev_path = fx.set_moe_path(getattr(args, "moe_path", "auto"))
    try:
        return _bench_moe_body(args, fx, syn, dev, cpu, L, d, shared, fused, ws)
    finally:
        fx.set_moe_path(prev_path)


def _bench_moe_body(args, fx, syn, dev, cpu, L, d, shared, fused, ws):
    import torch

    Ms = [int(m) for m in (args.ms or "1,2,4,8,16").split(",")]
    results = {}
    peak, src = measured_peak()
    total_bytes, total_ms = 0, 0.0
    sampler = ClockSampler(_gpu_id(dev))
    clocks = None
    n_rot = 48
    launches = 0
    first_routing = {}
    for M in Ms:
        rots, nbytes = [], 0
        for r in range(n_rot):
            ids, wts = syn.routing(M, E=syn.EXPERTS, seed=1000 * M + r)
            # shift the expert ids per rotation: successive calls touch different experts,
            # as consecutive decode layers do
            ids = ((ids.long() + 97 * r) % syn.EXPERTS).to(torch.int32)
            nbytes += syn.moe_bytes(int(torch.unique(ids).numel()), M=M)
            rots.append((ids.to(dev), wts.to(dev)))
            if r == 0:
                first_routing[M] = (ids, wts)
        x = syn.activations(M, seed=3).to(dev)
        out = torch.empty(M, syn.HIDDEN, dtype=torch.bfloat16, device=dev)

        def call(ids, wts):
            fx.draft_moe_gemv(hidden_states=x, topk_ids=ids, topk_weights=wts,
                              w13_weight=d["w13"], w13_blockscale_swizzled=d["s13"],
                              w13_weight_scale_2=d["g13"], w2_weight=d["w2"],
                              w2_blockscale_swizzled=d["s2"], w2_weight_scale_2=d["g2"],
                              workspace=ws, shared_expert=shared, out=out,
                              cfg=fx.DraftMoeGemvConfig(pdl=True))

        g = _graph_of([(lambda r=r: call(*r)) for r in rots])
        reps = max(3, args.steps // n_rot)
        ms, ck = _timed(g.replay, reps, 3, dev, 1, sampler if M == Ms[-1] else None)
        clocks = ck or clocks
        us = ms / (reps * n_rot) * 1e3
        bytes_per_call = nbytes / n_rot
        results[str(M)] = {"us_per_call": round(us, 3),
                           "GBps": round(bytes_per_call / (us * 1e-6) / 1e9, 1),
                           "bytes_per_call": int(bytes_per_call)}
        total_bytes += bytes_per_call * reps * n_rot
        total_ms += ms
        launches += reps * n_rot * fx.moe_launches_per_call(syn.HIDDEN, syn.INTER, fused,
                                                             num_tokens=M)
        del g
    value = total_bytes / (total_ms / 1e3) / 1e9
    res = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "nvfp4/bf16 (fp32 accumulate)", "data": "synthetic",
           "config": {"workload": "nvfp4_moe_512x2048x512_top10_shared", "M": Ms,
                      "l2": f"{n_rot} routings over shifted expert sets in one CUDA graph (> 4x L2)"},
           "per_m": results,
           "roofline": _roofline_per_m(results, peak, src, " | ".join(dict.fromkeys(
                                           fx.moe_kernel_name(syn.HIDDEN, syn.INTER, fused,
                                                              num_tokens=M) for M in Ms)),
                                       traffic_per_m=_moe_traffic(fx, syn, fused, Ms)),
           "clocks": clocks, "gpu_launches": launches}
    if cpu:
        cb = {}
        for M in Ms:
            ids, wts = first_routing[M]
            b = syn.moe_bytes(int(torch.unique(ids).numel()), M=M)
            gbs, el, n, cores = cpu_moe_sample(L, syn.activations(M, seed=3), ids, wts, b,
                                               min_seconds=2.0)
            cb[str(M)] = {"value": round(gbs, 4), "calls": n, "seconds": round(el, 2)}
        tot = sum(results[m]["bytes_per_call"] for m in cb)
        sec = sum(cb[m]["seconds"] / cb[m]["calls"] for m in cb)
        res["cpu_baseline"] = {"value": round(tot / sec / 1e9, 4), "unit": UNIT, "cores": cores,
                               "kind": "port", "per_m": cb,
                               "sample": "one routing per M, whole layer (torch moe_reference "
                                         "restated: per route dequantise + gate/up + silu*up "
                                         "+ down, fp32, all host threads)"}
    return res


def _moe_traffic(fx, syn, fused, Ms):
    """ncu DRAM bytes per launch of the kernel each M runs, from its profiles/ summary."""
    keys = {"moe_lean_kernel": "moe_lean_config2_m1", "moe_fused_kernel": "moe_fused_config2_m16",
            "moe_up_kernel + moe_down_kernel + moe_sum_kernel": "moe_nvfp4_config2"}
    out = {}
    for M in Ms:
        key = keys.get(fx.moe_kernel_name(syn.HIDDEN, syn.INTER, fused, num_tokens=M))
        t = traffic_for(key) if key else None
        if t and str(M) in t:
            out[str(M)] = t[str(M)]
    return out


def _device_moe_layer(fx, syn, dev, seed, experts=None):
    """One config-2 MoE layer (512 experts + shared expert) generated on the device: code
    bytes uniform over 0-255, e4m3 block scales |N(0,1)|*0.5, global scales 1/448.  The
    scales are drawn directly in the 128x4-swizzled order (a fixed permutation of
    independent draws has the same distribution), so no swizzle pass is needed."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    E, H, I = experts or syn.EXPERTS, syn.HIDDEN, syn.INTER

    def codes(*shape):
        return torch.randint(0, 256, shape, generator=g, dtype=torch.uint8, device=dev)

    def scales(*shape):
        s = torch.randn(*shape, generator=g, device=dev).abs_().mul_(0.5)
        return s.to(torch.float8_e4m3fn).view(torch.uint8)

    gs = 1.0 / 448.0
    d = dict(w13=codes(E, 2 * I, H // 2), s13=scales(E, 2 * I, H // 16),
             g13=torch.full((E, 2), gs, device=dev), w2=codes(E, H, I // 2),
             s2=scales(E, H, I // 16), g2=torch.full((E,), gs, device=dev))
    shared = fx.SharedExpert(codes(1, 2 * I, H // 2), scales(1, 2 * I, H // 16),
                             torch.tensor([gs], device=dev), codes(1, H, I // 2),
                             scales(1, H, I // 16), torch.tensor([gs], device=dev))
    return d, shared


def bench_stack(args, fx, syn, dev):
    """Config 3: a decode step of 48 MoE layers (config 2 each, with its own weights:
    about 43.5 GB of NVFP4 resident) chained layer to layer, ending in the config-1 int8
    lm_head with greedy argmax.  One CUDA graph per M holds the whole step; the step's
    weights are far larger than L2, so every layer streams from HBM."""
    import torch

    Ms = [int(m) for m in (args.ms or "1,4,16").split(",")]
    n_layers = args.layers
    layers = [_device_moe_layer(fx, syn, dev, seed=layer) for layer in range(n_layers)]
    head = syn.w8_head(syn.VOCAB, syn.HIDDEN, seed=0)
    hw, hs = head.w.to(dev), head.scale.to(dev)
    del head
    ws = fx.make_workspace(num_routes=syn.TOPK, hidden_size=syn.HIDDEN,
                           intermediate_size=syn.INTER, device=dev)
    moe_cfg = fx.DraftMoeGemvConfig(pdl=True)
    peak, src = measured_peak()
    sampler = ClockSampler(_gpu_id(dev))
    clocks = None
    per_m, total_bytes, total_ms, launches = {}, 0, 0.0, 0
    reps = max(5, min(args.steps, 50))
    for M in Ms:
        routes, step_bytes = [], syn.w8_head_bytes(syn.VOCAB, syn.HIDDEN, M)
        for layer in range(n_layers):
            ids, wts = syn.routing(M, E=syn.EXPERTS, seed=100_000 + 1000 * M + layer)
            step_bytes += syn.moe_bytes(int(torch.unique(ids).numel()), M=M)
            routes.append((ids.to(dev), wts.to(dev)))
        bufs = [syn.activations(M, seed=3).to(dev),
                torch.empty(M, syn.HIDDEN, dtype=torch.bfloat16, device=dev)]
        logits = torch.empty(M, syn.VOCAB, dtype=torch.bfloat16, device=dev)
        am = torch.empty(M, dtype=torch.int64, device=dev)

        def layer_call(layer):
            (d, shared), (ids, wts) = layers[layer], routes[layer]
            fx.draft_moe_gemv(hidden_states=bufs[layer % 2], topk_ids=ids, topk_weights=wts,
                              w13_weight=d["w13"], w13_blockscale_swizzled=d["s13"],
                              w13_weight_scale_2=d["g13"], w2_weight=d["w2"],
                              w2_blockscale_swizzled=d["s2"], w2_weight_scale_2=d["g2"],
                              workspace=ws, shared_expert=shared, out=bufs[(layer + 1) % 2],
                              cfg=moe_cfg)

        calls = [(lambda layer=layer: layer_call(layer)) for layer in range(n_layers)]
        calls.append(lambda: fx.w8a16_gemv(bufs[n_layers % 2], hw, hs, out=logits,
                                           argmax_out=am, pdl=True))
        g = _graph_of(calls)
        ms, ck = _timed(g.replay, reps, max(3, args.warmup // 10), dev, 1,
                        sampler if M == Ms[-1] else None)
        clocks = ck or clocks
        us = ms / reps * 1e3
        per_m[str(M)] = {"us_per_step": round(us, 2),
                         "GBps": round(step_bytes / (us * 1e-6) / 1e9, 1),
                         "bytes_per_step": int(step_bytes),
                         "argmax": am.cpu().tolist()}
        total_bytes += step_bytes * reps
        total_ms += ms
        # MoE launches per layer (one fused, or gate/up + down + route sum); the lm_head
        launches += reps * (fx.moe_launches_per_call(syn.HIDDEN, syn.INTER, num_tokens=M)
                            * n_layers + 1)
        del g
    value = total_bytes / (total_ms / 1e3) / 1e9
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1,
            "steps": reps * len(Ms), "warmup": args.warmup,
            "ms_per_step": round(total_ms / (reps * len(Ms)), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "nvfp4+int8/bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"decode_stack_{n_layers}x_moe512x2048x512_top10_shared"
                                   f"+lm_head{syn.VOCAB}", "M": Ms, "layers": n_layers,
                       "l2": "whole step's weights (about 0.91 GB per layer) far above L2",
                       "chain": "layer l output is layer l+1 input; the last feeds the lm_head"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(value / peak, 4), "traffic": None, "peak_source": src},
            "clocks": clocks, "gpu_launches": launches}


def bench_moe_sharded(args, fx, syn, dev, rank, world):
    """Config 4, second part: the config-2 MoE layer expert-sharded over the ranks (rank g
    holds experts [g*512/G, (g+1)*512/G) and the shared expert lives on rank 0); every rank
    runs the routed GEMVs of its own experts into an fp32 partial [M, 2048], one NCCL SUM
    all-reduce combines them and a bf16 rounding gives the layer output.  48 routings over
    shifted expert sets are captured, collective included, in one CUDA graph per M; the
    step time is the max over ranks."""
    import torch
    import torch.distributed as dist

    from flash_next_rtxpro6000_b200 import sharded

    Ms = [int(m) for m in (args.ms or "16").split(",")]
    if syn.EXPERTS % world:
        raise SystemExit(f"{syn.EXPERTS} experts not divisible by {world} ranks")
    E_local = syn.EXPERTS // world
    e0 = rank * E_local
    d, shared = _device_moe_layer(fx, syn, dev, seed=rank, experts=E_local)
    if rank != 0:
        shared = None
    ws = fx.make_workspace(num_routes=syn.TOPK, hidden_size=syn.HIDDEN,
                           intermediate_size=syn.INTER, device=dev)
    peak, src = measured_peak()
    sampler = ClockSampler(_gpu_id(dev)) if rank == 0 else None
    clocks = None
    n_rot = 48
    per_m, total_bytes, total_ms, launches = {}, 0, 0.0, 0
    for M in Ms:
        rots, nbytes, local_bytes = [], 0, 0
        for r in range(n_rot):
            ids, wts = syn.routing(M, E=syn.EXPERTS, seed=1000 * M + r)
            ids = ((ids.long() + 97 * r) % syn.EXPERTS).to(torch.int32)
            uniq = torch.unique(ids)
            nbytes += syn.moe_bytes(int(uniq.numel()), M=M)
            mine = int(((uniq >= e0) & (uniq < e0 + E_local)).sum())
            local_bytes += syn.moe_bytes(mine, M=M, shared=(rank == 0))
            rots.append((ids.to(dev), wts.to(dev)))
        x = syn.activations(M, seed=3).to(dev)
        part = torch.empty(M, syn.HIDDEN, dtype=torch.float32, device=dev)
        out = torch.empty(M, syn.HIDDEN, dtype=torch.bfloat16, device=dev)

        def call(ids, wts):
            fx.draft_moe_gemv(hidden_states=x, topk_ids=ids, topk_weights=wts,
                              w13_weight=d["w13"], w13_blockscale_swizzled=d["s13"],
                              w13_weight_scale_2=d["g13"], w2_weight=d["w2"],
                              w2_blockscale_swizzled=d["s2"], w2_weight_scale_2=d["g2"],
                              workspace=ws, shared_expert=shared, expert_offset=e0,
                              out=part, out_f32=True, cfg=fx.DraftMoeGemvConfig(pdl=True))
            dist.all_reduce(part, op=dist.ReduceOp.SUM)
            out.copy_(part)

        call(*rots[0])  # NCCL communicator up before the capture
        torch.cuda.synchronize()
        g = _graph_of([(lambda r=r: call(*r)) for r in rots])
        reps = max(3, args.steps // n_rot)
        ms, ck = _timed(g.replay, reps, 3, dev, world, sampler if M == Ms[-1] else None)
        clocks = ck or clocks
        us = ms / (reps * n_rot) * 1e3
        per_m[str(M)] = {"us_per_call": round(us, 3),
                         "GBps_aggregate": round(nbytes / n_rot / (us * 1e-6) / 1e9, 1),
                         "bytes_per_call": int(nbytes / n_rot),
                         "rank0_local_bytes_per_call": int(local_bytes / n_rot)}
        total_bytes += nbytes * reps
        total_ms += ms
        # the MoE kernels (the NCCL sum and the bf16 copy are library kernels)
        launches += reps * n_rot * fx.moe_launches_per_call(syn.HIDDEN, syn.INTER, num_tokens=M,
                                                             num_experts=E_local)
        torch.cuda.synchronize()
        del g
    value = total_bytes / (total_ms / 1e3) / 1e9
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "nvfp4/bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": "nvfp4_moe_512x2048x512_top10_shared", "M": Ms,
                       "parallelism": f"expert-sharded x{world} ({E_local} experts per rank) + "
                                      "NCCL SUM all-reduce of fp32 partials",
                       "l2": f"{n_rot} routings over shifted expert sets in one CUDA graph"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "achieved": round(value / world, 1), "peak": peak,
                         "unit": "GB/s per GPU", "frac": round(value / world / peak, 4),
                         "traffic": None, "peak_source": src},
            "clocks": clocks, "gpu_launches": launches}


if __name__ == "__main__":
    main()
