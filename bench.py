#!/usr/bin/env python3
"""Benchmark of the W4A16 AWQ decode datapath on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl anvilq|reference]
                    [--workload proj05b|proj7b]

One step = one pass of the W4A16 AWQ GEMV over every projection of every layer of
a batch-1 decode step (each projection has its own weights; all resident in HBM),
replayed as one CUDA graph.  Default workload: the Qwen2.5-0.5B decode-step
projection set (24 layers x q,k,v,o,gate,up,down; 186 MB of int4 weights, larger
than the 126 MB L2, so no L2 flush is needed between steps).

value  = algorithmic HBM bytes of all ranks' steps / max-over-ranks device time (GB/s)
e2e    = same metric through the public ProjectionStream API with every
         projection's activations copied from pinned host memory and every output
         copied back inside the timed step.
With N GPUs, each rank runs an independent replica (weak scaling, no collective).

--impl reference times the CPU restatement of the reference's golden GEMV
(FP32Model.linear, anvil-q1/tests/official_weights.py:418-437) on all host
cores over a bounded column sample of the same projection set.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "W4A16 GEMV HBM GB/s (% of B200 peak); decode tok/s at 0.5B/7B shapes"
WORKLOADS = {
    "proj05b": dict(name="Qwen2.5-0.5B decode-step W4A16 projections: 24 layers x (q 896x896+bias, "
                         "k,v 896x128+bias, o 896x896, gate,up 896x4864, down 4864x896), G128, M=1",
                    layers=24, projections="QWEN05B_PROJECTIONS"),
    "proj7b": dict(name="Llama-7B-class decode-step W4A16 projections: 32 layers x (q,k,v,o 4096x4096, "
                        "gate,up 4096x11008, down 11008x4096), G128, M=1",
                   layers=32, projections="LLAMA7B_PROJECTIONS"),
}


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.proc = None
        self.lines = []
        smi = shutil.which("nvidia-smi")
        if smi is None:
            return
        import torch
        target = []
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            target = ["-i", uuid if uuid.startswith("GPU-") else "GPU-" + uuid]
        except Exception:
            target = []
        self.cmd = [smi, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100", *target]

    def __enter__(self):
        if hasattr(self, "cmd"):
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------- CPU baseline
def cpu_sample(projections, fraction, seed=17):
    """Bounded sample of one layer's projections: all K rows, the first `fraction` of columns."""
    import numpy as np
    from anvilq_b200 import synthetic
    rng = np.random.default_rng(seed)
    cases = []
    for K, N, bias in projections:
        layer = synthetic.awq_layer(K, N, 128, rng=rng, bias=bias)
        x = synthetic.activations(1, K, rng=rng).astype(np.float32)
        nc = max(8, int(N * fraction) // 8 * 8)
        b = synthetic.gemv_bytes(1, K, nc, 128, bias)
        cases.append((x, layer, nc, b))
    return cases


def run_cpu(cases, threads):
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    total = 0
    t0 = time.perf_counter()
    for x, layer, nc, b in cases:
        oracle.gemv_fp32(x, layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits, 128,
                         threads=threads, n_range=(0, nc))
        total += b
    return total, time.perf_counter() - t0


def cpu_baseline(projections, target_s=12.0):
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    threads = oracle.max_threads()
    cases = cpu_sample(projections, 1 / 64)
    b, dt = run_cpu(cases, threads)
    frac = min(1.0, (1 / 64) * target_s / max(dt, 1e-3) / 4)
    cases = cpu_sample(projections, frac)
    reps, total_b, total_t = 0, 0, 0.0
    while total_t < target_s / 2 or reps < 1:
        b, dt = run_cpu(cases, threads)
        total_b += b
        total_t += dt
        reps += 1
    return {"value": round(total_b / total_t / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle/awq_oracle.c FP32Model.linear restatement over one layer's 7 projections, "
                      f"all K rows x first {frac:.4f} of the columns, {reps} repetitions, "
                      f"{total_t:.1f} s, {threads} threads"}


# --------------------------------------------------------------------- arms
def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def reference_arm(args, world, rank):
    from anvilq_b200 import stream as st
    wl = WORKLOADS[args.workload]
    projections = getattr(st, wl["projections"])
    if rank != 0:
        return 0
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    threads = oracle.max_threads()
    probe = cpu_sample(projections, 1 / 64)
    _, dt = run_cpu(probe, threads)
    frac = min(1.0, (1 / 64) * 20.0 / max(1, args.steps + args.warmup) / max(dt, 1e-3))
    cases = cpu_sample(projections, frac)
    for _ in range(args.warmup):
        run_cpu(cases, threads)
    total_b, total_t = 0, 0.0
    for _ in range(args.steps):
        b, dt = run_cpu(cases, threads)
        total_b += b
        total_t += dt
    value = total_b / total_t / 1e9
    sample = (f"oracle/awq_oracle.c FP32Model.linear restatement, one layer's 7 projections, all K rows x "
              f"first {frac:.4f} of the columns per step, {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_t / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE value distributions)",
            "config": {"workload": wl["name"], "sample": "column sample, see cpu_baseline"},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def anvilq_arm(args, world, rank, local):
    import torch
    from anvilq_b200 import stream as st
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    wl = WORKLOADS[args.workload]
    projections = getattr(st, wl["projections"])
    peak, peak_kind = load_peaks()

    s = st.ProjectionStream(projections, wl["layers"], M=1, seed=17 + rank, device=dev).capture()
    e2e = st.ProjectionStream(projections, wl["layers"], M=1, seed=17 + rank, device=dev, host_io=True).capture()
    step_bytes = s.algorithmic_bytes()

    def timed(stream_obj, steps, sync_each):
        for _ in range(args.warmup):
            stream_obj.run()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream_obj.stream)
        for _ in range(steps):
            stream_obj.run()
            if sync_each:
                stream_obj.stream.synchronize()
        end.record(stream_obj.stream)
        torch.cuda.synchronize(dev)
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
            torch.distributed.barrier()
        return ms

    with ClockSampler(dev.index) as clocks:
        ms = timed(s, args.steps, False)
    ms_e2e = timed(e2e, args.steps, True)
    from anvilq_b200 import ops
    ops.raise_device_errors(dev)

    ms_step = ms / args.steps
    value = step_bytes * world * args.steps / (ms / 1e3) / 1e9
    per_launch_ms = ms_step / s.launches()
    achieved = step_bytes / s.launches() / (per_launch_ms / 1e3) / 1e9
    traffic = None   # DRAM bytes per launch from the committed ncu capture (profiles/)
    prof = REPO / "profiles" / "traffic.json"
    if prof.exists():
        entry = json.loads(prof.read_text()).get(f"gemv_tma_kernel/{args.workload}")
        if entry:
            traffic = int(step_bytes / s.launches() * entry["ratio_read_over_algorithmic"])
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 activations x int4 weights, fp32 accumulate",
        "data": "synthetic (seeded; x~N(0,1), u4 uniform, scales |N(0,1)|*0.01+1e-3)",
        "config": {"workload": wl["name"], "M": 1, "group": 128, "layers": wl["layers"],
                   "step_bytes": step_bytes, "launches_per_step": s.launches(),
                   "l2": "inputs larger than L2 (no flush)", "parallelism": f"replicas x{world}",
                   "graph": "one CUDA graph per step"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "frac_of_8tbs_nominal": round(achieved / 8000.0, 4), "traffic": traffic,
                     "kernel": "gemv_tma_kernel",
                     "launch_avg_us": round(per_launch_ms * 1e3, 4)},
        "e2e": {"value": round(step_bytes * world * args.steps / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": e2e.h2d_bytes(), "d2h_bytes_per_step": e2e.d2h_bytes(),
                "ms_per_step": round(ms_e2e / args.steps, 5)},
        "gpu_launches": s.launches() * args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(projections)
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("anvilq", "reference"), default="anvilq")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="proj05b")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return reference_arm(args, world, rank)
    world, rank, local = dist_init()
    try:
        return anvilq_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
