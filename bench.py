#!/usr/bin/env python3
"""Benchmark of the W4A16 AWQ decode datapath on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl anvilq|reference]
                    [--workload decode05b|decode7b|proj05b|proj7b|attn|tp70b] [--no-extras] [--fused]

decode05b (default): one step = one greedy decode token of a Qwen2.5-0.5B-shape
W4A16 AWQ model (24 layers, hidden 896, 14/2 heads of 64, intermediate 4864,
vocab 151936, tied fp16 lm_head; random-init weights with the reference's value
distributions), batch 1, at context 1024, as one CUDA graph.  value = tokens/s;
the step moves ~472 MB (186 MB int4 weights, 272 MB lm_head, 12.6 MB KV), larger
than the 126 MB L2, so no flush is needed between steps.  The roofline object
times the step's 96 W4A16 GEMVs (same weights, buffers and fused modes) as a
graph of their own in the same run.  e2e drives the public Decoder API with the
input token copied from pinned host memory and the chosen token copied back
inside every step, and the host waiting for it.  Unless --no-extras, the same
line carries four more measurements taken in the same run, on every rank:
"decode7b" (the same decode step for a Llama-7B-class model, tok/s, one replica
per GPU), "proj7b" (the W4A16 GEMVs of a Llama-7B-class decode step, GB/s, one replica
per GPU), "tp70b" (the 70B-class layer column-split over the N GPUs and
all-gathered, GB/s, strong scaling) and "attn" (decode attention over a
64-sequence batch at context 32768 sharded over the N GPUs, GB/s).

proj05b / proj7b: one step = the W4A16 GEMV over every projection of a decode
step (Qwen2.5-0.5B or Llama-7B-class shapes), value in GB/s.

attn: one step = one decode-attention launch over the rank's share of a
64-sequence batch at context 32768 (32/8 heads of 128); value = KV bytes
streamed per second over all ranks (strong scaling, batch-sharded, no
collective).  e2e copies q from pinned host memory and the output back
every step.

tp70b: one step = the three 70B-class layer projections, each column-split over
the N GPUs (strong scaling) and all-gathered, as one CUDA graph; at M = 1 on
several GPUs the all-gather is fused into each GEMV (every rank stores its slice
into every rank's output over NVLink and the ranks exchange completion flags),
otherwise NCCL all-gathers follow the GEMMs; value = full-layer algorithmic GB/s
over the max-over-ranks time; --tokens sets the token rows (1 for the GEMV, 16/64
for the verify GEMM).

With N GPUs, decode05b and the projection sets run one independent replica per
rank (weak scaling, no collective); attn shards its batch (no collective).

--impl reference times the CPU restatement of the reference's golden model on
the host cores over a bounded sample of the same workload: FP32Model.token
(anvil-q1/tests/official_weights.py:451-509, binary64 numpy port) for decode05b,
FP32Model.linear (:418-437, C port, bit-exact) for the projection sets.
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
    "decode05b": dict(name="Qwen2.5-0.5B-shape greedy decode step, batch 1, context 1024: 24 layers, hidden 896, "
                           "14 q / 2 kv heads of 64, intermediate 4864, W4A16 AWQ G128 projections, RMSNorm eps 1e-6, "
                           "RoPE theta 1e6, fp16 KV cache, tied fp16 lm_head [151936, 896], greedy argmax",
                      context=1024, shape="QWEN05B_SHAPE"),
    "decode7b": dict(name="Llama-7B-class greedy decode step, batch 1, context 1024: 32 layers, hidden 4096, 32 heads "
                          "of 128 (no grouping), intermediate 11008, W4A16 AWQ G128 projections without bias, RMSNorm "
                          "eps 1e-6, RoPE theta 1e6, fp16 KV cache, tied fp16 lm_head [32000, 4096], greedy argmax",
                     context=1024, shape="LLAMA7B_SHAPE", device_init=True, qkv_bias=False),
    "proj05b": dict(name="Qwen2.5-0.5B decode-step W4A16 projections: 24 layers x (q 896x896+bias, "
                         "k,v 896x128+bias, o 896x896, gate,up 896x4864, down 4864x896), G128, M=1",
                    layers=24, projections="QWEN05B_PROJECTIONS"),
    "proj7b": dict(name="Llama-7B-class decode-step W4A16 projections: 32 layers x (q,k,v,o 4096x4096, "
                        "gate,up 4096x11008, down 11008x4096), G128, M=1",
                   layers=32, projections="LLAMA7B_PROJECTIONS"),
    "attn": dict(name="GQA decode attention over an fp16 KV cache: 32 q / 8 kv heads of 128, global batch 64 at "
                      "context 32768 (every sequence full), scale 1/sqrt(128); the batch is sharded over the GPUs "
                      "(rank r holds sequences [64r/W, 64(r+1)/W)), no collective",
                 batch=64, context=32768, hq=32, hkv=8, d=128),
    "tp70b": dict(name="70B-class W4A16 AWQ layer projections (K,N) in (8192,8192), (8192,28672), (28672,8192), "
                       "G128, column-split over the GPUs (rank r holds columns [rN/W, (r+1)N/W)), y all-gathered "
                       "over NCCL after every projection",
                  shapes=((8192, 8192), (8192, 28672), (28672, 8192))),
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


def max_over_ranks(ms, world, dev):
    """Device time of the slowest rank (every rank calls this at the same point)."""
    if world == 1:
        return ms
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(run, stream, steps, warmup, world, dev, sync_each=False):
    """W warm-up steps, then K steps between CUDA events on `stream`, bracketed by
    a barrier and device synchronisation; the max over ranks in ms.  `run`
    enqueues one step on `stream`; sync_each makes the host wait for every step."""
    import torch
    for _ in range(warmup):
        run()
        if sync_each:
            stream.synchronize()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        run()
        if sync_each:
            stream.synchronize()
    end.record(stream)
    torch.cuda.synchronize(dev)
    return max_over_ranks(start.elapsed_time(end), world, dev)


def traffic_entry(key):
    """DRAM bytes over algorithmic bytes from the committed ncu capture for `key`."""
    prof = REPO / "profiles" / "traffic.json"
    if not prof.exists():
        return None
    return json.loads(prof.read_text()).get(key)


def weighted_traffic(name, launches):
    """DRAM bytes per launch for a set of launches [(algorithmic bytes, kernel)], each scaled
    by its kernel's captured ratio for workload `name`; None if a kernel has no capture."""
    total = 0.0
    for nbytes, kernel in launches:
        entry = traffic_entry(f"{kernel}/{name}")
        if entry is None:
            return None
        total += nbytes * entry["ratio_read_over_algorithmic"]
    return int(total / len(launches)) if launches else None


# ------------------------------------------------------------ decode05b
def _decode_oracle_sample(context, seed=17):
    """One layer of the decode step plus 1/24 of the lm_head rows, in the binary64
    oracle (the per-token CPU time is 24x this sample)."""
    import numpy as np
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    from anvilq_b200 import decoder
    L, H, I, QH, KVH, D, G, V, SEQ = decoder.QWEN05B_SHAPE
    shape = (1, H, I, QH, KVH, D, G, V // L, SEQ)
    w = decoder.synthetic_weights(shape, seed=seed)
    o = oracle.DecodeOracle(w)
    rng = np.random.default_rng(seed)
    for t in range(context):   # synthetic context in the cache
        o.cache[0, t] = (rng.standard_normal((KVH, D)), rng.standard_normal((KVH, D)))
    return o


def _decode_cpu(o, context, steps):
    t0 = time.perf_counter()
    for i in range(steps):
        o.step(5, context + i)
    return time.perf_counter() - t0


def decode_cpu_baseline(context, target_s=15.0):
    o = _decode_oracle_sample(context)
    dt = _decode_cpu(o, context, 1)
    n = max(1, int(target_s / max(dt, 1e-3)))
    dt = _decode_cpu(o, context + 1, n)
    per_token = dt / n * 24
    return {"value": round(1.0 / per_token, 5), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle.DecodeOracle (binary64 numpy restatement of FP32Model.token) on 1 of 24 layers "
                      f"+ 1/24 of the lm_head rows at context {context}, {n} steps in {dt:.1f} s, scaled x24; "
                      f"numpy/BLAS threads as available"}


def decode_reference_arm(args, world, rank):
    if rank != 0:
        return 0
    wl = WORKLOADS["decode05b"]
    ctx = wl["context"]
    o = _decode_oracle_sample(ctx)
    _decode_cpu(o, ctx, args.warmup)
    dt = _decode_cpu(o, ctx + args.warmup, args.steps)
    sample_ms = dt / args.steps * 1e3          # what one step actually measured
    per_token = dt / args.steps * 24           # the whole token: 24 such samples
    value = 1.0 / per_token
    sample = ("oracle.DecodeOracle (binary64 numpy restatement of FP32Model.token); one step = a bounded sample "
              "of one token: 1 of the 24 layers + 1/24 of the lm_head rows; tokens/s = 1 / (24 x the sample "
              "time); ms_per_step is the sample's own measured time")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sample_ms, 3),
            "token_ms_extrapolated": round(per_token * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded; x ~ N(0,1), u4 uniform, scales |N(0,1)|*0.01+1e-3)",
            "config": {"workload": wl["name"], "sample": sample},
            "cpu_baseline": {"value": round(value, 5), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 5), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def decode_measure(args, world, rank, dev, name):
    """One greedy decode token per step of the workload's model (decode05b or
    decode7b), as one CUDA graph; the line without the CPU baseline."""
    import torch
    from anvilq_b200 import decoder
    wl = WORKLOADS[name]
    shape = getattr(decoder, wl["shape"])
    ctx = wl["context"]
    peak, peak_kind = load_peaks()
    if wl.get("device_init"):
        w = decoder.device_synthetic_weights(shape, dev, seed=17 + rank, qkv_bias=wl["qkv_bias"])
    else:
        w = decoder.synthetic_weights(shape, seed=17 + rank)
    total_steps = 2 * (args.warmup + args.steps) + 4
    d = decoder.Decoder(w, dev, max_seq=ctx + total_steps + 8, fused=True if args.fused else False)
    del w
    d.fill_context(ctx, seed=rank)
    d.token.fill_(1000)
    d.token_in.fill_(1000)
    g_dev = d.record(False)
    g_e2e = d.record(True)
    # the dominant kernel timed on its own: the fused layers kernel, or the step's GEMVs
    g_roof = d.record_layers() if d.fused else d.record_gemvs()

    def replay(graph):
        def run():
            with torch.cuda.stream(d.stream):
                graph.replay()
        return run

    with ClockSampler(dev.index) as clocks:
        ms = timed(replay(g_dev), d.stream, args.steps, args.warmup, world, dev)
    d.pos.fill_(ctx)
    ms_e2e = timed(replay(g_e2e), d.stream, args.steps, args.warmup, world, dev, sync_each=True)
    pos_roof = int(d.pos.item())
    ms_roof = timed(replay(g_roof), d.stream, args.steps, args.warmup, world, dev)
    d.check_errors()

    L = shape[0]
    tok_s = world * args.steps / (ms / 1e3)
    step_bytes = d.bytes_per_step(ctx + args.warmup + args.steps // 2)
    if d.fused:
        roof_kernel, roof_launches = "decode_step_kernel", 1
        roof_bytes = d.layer_bytes_per_step(pos_roof + 1)
        roof_on = f"the fused layers kernel (all {L} layers of a token, no lm_head) as its own CUDA graph, same run"
    else:
        roof_kernel, roof_launches = "gemv_tma_kernel", 4 * L
        roof_bytes = d.gemv_bytes_per_step()
        roof_on = f"the step's {4 * L} W4A16 GEMVs as their own CUDA graph, same run"
    per_launch_s = ms_roof / 1e3 / args.steps / roof_launches
    achieved = roof_bytes / roof_launches / per_launch_s / 1e9
    entry = traffic_entry(f"{roof_kernel}/{name}")
    traffic = int(roof_bytes / roof_launches * entry["ratio_read_over_algorithmic"]) if entry else None
    line = {
        "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 activations x int4 weights, fp32 accumulate; fp16 KV and lm_head",
        "data": "synthetic (seeded random-init weights and context; u4 uniform, scales |N(0,1)|*0.01+1e-3)",
        "config": {"workload": wl["name"], "batch": 1, "context": ctx, "layers": L,
                   "step_bytes": step_bytes, "kernels_per_step": d.kernels_per_step(),
                   "l2": "inputs larger than L2 (no flush)", "parallelism": f"replicas x{world}",
                   "graph": "one CUDA graph per token", "fused_layers_kernel": bool(d.fused)},
        "hbm_gbs": round(step_bytes * tok_s / world / 1e9, 2),
        "hbm_frac_of_measured_peak": round(step_bytes * tok_s / world / 1e9 / peak, 4),
        "roofline": {"bound": "hbm", "kernel": roof_kernel, "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "frac_of_8tbs_nominal": round(achieved / 8000.0, 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": int(roof_bytes / roof_launches),
                     "launch_avg_us": round(per_launch_s * 1e6, 4), "measured_on": roof_on},
        "e2e": {"value": round(world * args.steps / (ms_e2e / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                "ms_per_step": round(ms_e2e / args.steps, 5)},
        "gpu_launches": d.kernels_per_step() * args.steps,
        "clocks": clocks.summary(),
    }
    del g_dev, g_e2e, g_roof, d
    torch.cuda.empty_cache()
    return line


def decode_arm(args, world, rank, local):
    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    name = args.workload
    line = decode_measure(args, world, rank, dev, name)
    if name == "decode05b" and not args.no_extras:
        for key, fn in (("decode7b", lambda: decode_measure(args, world, rank, dev, "decode7b")),
                        ("proj7b", lambda: proj_measure(args, world, rank, dev, "proj7b", e2e=False)),
                        ("tp70b", lambda: tp_measure(args, world, rank, dev, 1, e2e=False)),
                        ("attn", lambda: attn_measure(args, world, rank, dev, e2e=False))):
            try:
                line[key] = summary(fn())
            except Exception as e:   # reported in the line; the headline above stands
                line[key] = {"error": f"{type(e).__name__}: {e}"[:400]}
            torch.cuda.empty_cache()
            line["gpu_launches"] += line[key].get("gpu_launches", 0)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and name == "decode05b":
        line["cpu_baseline"] = decode_cpu_baseline(WORKLOADS[name]["context"])
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def summary(m):
    """The fields of a workload line kept when it rides on the headline line."""
    keep = ("metric", "value", "unit", "ms_per_step", "scaling", "roofline", "gpu_launches", "clocks")
    out = {k: m[k] for k in keep if k in m}
    out["config"] = {k: v for k, v in m["config"].items() if k != "workload"}
    out["workload"] = m["config"]["workload"]
    return out


# ------------------------------------------------------------ projection sets
def proj_measure(args, world, rank, dev, name, e2e=True):
    from anvilq_b200 import ops, synthetic
    from anvilq_b200 import stream as st
    wl = WORKLOADS[name]
    projections = getattr(st, wl["projections"])
    peak, peak_kind = load_peaks()
    s = st.ProjectionStream(projections, wl["layers"], M=1, seed=17 + rank, device=dev, device_init=True).capture()
    step_bytes = s.algorithmic_bytes()
    with ClockSampler(dev.index) as clocks:
        ms = timed(s.run, s.stream, args.steps, args.warmup, world, dev)
    ms_e2e = se = None
    if e2e:
        se = st.ProjectionStream(projections, wl["layers"], M=1, seed=17 + rank, device=dev, host_io=True,
                                 device_init=True).capture()
        ms_e2e = timed(se.run, se.stream, args.steps, args.warmup, world, dev, sync_each=True)
    ops.raise_device_errors(dev)
    plans = sorted({(K, N): ops.gemv_plan(K, N)["kernel"] for K, N, _ in projections}.items())
    ms_step = ms / args.steps
    value = step_bytes * world * args.steps / (ms / 1e3) / 1e9
    per_launch_ms = ms_step / s.launches()
    achieved = step_bytes / s.launches() / (per_launch_ms / 1e3) / 1e9
    kernels = sorted({"gemv_stream_kernel" if k == 1 else "gemv_tma_kernel" for _, k in plans})
    kernel = " + ".join(kernels)
    kind = dict(plans)
    traffic = weighted_traffic(name, [(synthetic.gemv_bytes(1, K, N, 128, bias),
                                       "gemv_stream_kernel" if kind[(K, N)] == 1 else "gemv_tma_kernel")
                                      for K, N, bias in projections])
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 activations x int4 weights, fp32 accumulate",
        "data": "synthetic (seeded on the device; x~N(0,1), u4 uniform, scales |N(0,1)|*0.01+1e-3)",
        "config": {"workload": wl["name"], "M": 1, "group": 128, "layers": wl["layers"],
                   "step_bytes": step_bytes, "launches_per_step": s.launches(),
                   "plans": {f"{K}x{N}": ("stream" if k == 1 else "cluster") for (K, N), k in plans},
                   "l2": "inputs larger than L2 (no flush)", "parallelism": f"replicas x{world}",
                   "graph": "one CUDA graph per step, programmatic dependent launch between GEMVs"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "frac_of_8tbs_nominal": round(achieved / 8000.0, 4), "traffic": traffic,
                     "kernel": kernel, "algorithmic_bytes_per_launch": int(step_bytes / s.launches()),
                     "launch_avg_us": round(per_launch_ms * 1e3, 4)},
        "gpu_launches": s.launches() * args.steps,
        "clocks": clocks.summary(),
    }
    if ms_e2e is not None:
        line["e2e"] = {"value": round(step_bytes * world * args.steps / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                       "h2d_bytes_per_step": se.h2d_bytes(), "d2h_bytes_per_step": se.d2h_bytes(),
                       "ms_per_step": round(ms_e2e / args.steps, 5)}
    return line


def anvilq_arm(args, world, rank, local):
    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    line = proj_measure(args, world, rank, dev, args.workload)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from anvilq_b200 import stream as st
        line["cpu_baseline"] = cpu_baseline(getattr(st, WORKLOADS[args.workload]["projections"]))
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def reference_arm(args, world, rank):
    if args.workload == "decode7b":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the CPU restatement of FP32Model.token is timed "
                              "on the 0.5B decode workload (decode05b); a 7B-class token takes hours in it"}))
        return 0
    if args.workload == "decode05b":
        return decode_reference_arm(args, world, rank)
    if args.workload == "attn":
        return attn_reference_arm(args, world, rank)
    from anvilq_b200 import stream as st
    wl = WORKLOADS[args.workload]
    projections = (tuple((K, N, False) for K, N in wl["shapes"]) if "shapes" in wl
                   else getattr(st, wl["projections"]))
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
    sample = (f"oracle/awq_oracle.c FP32Model.linear restatement, one layer's {len(projections)} projections, "
              f"all K rows x first {frac:.4f} of the columns per step, {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_t / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; x ~ N(0,1), u4 uniform, scales |N(0,1)|*0.01+1e-3)",
            "config": {"workload": wl["name"], "sample": "column sample, see cpu_baseline"},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ attn
def attn_bytes(B, T, Hq, Hkv, D):
    """Algorithmic HBM bytes of one decode-attention launch: K and V once, q in, out."""
    return B * T * Hkv * D * 2 * 2 + 2 * B * Hq * D * 2


def attn_cpu(args_steps, wl, target_s):
    """fp64 numpy restatement of attention() (fp64_reference.py:164-170) on whole
    sequences of the workload; returns (q, k, v, sequences per step)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    from anvilq_b200 import synthetic
    T, Hq, Hkv, D = wl["context"], wl["hq"], wl["hkv"], wl["d"]
    q, k, v = synthetic.kv_case(1, Hq, Hkv, D, T, seed=17)
    t0 = time.perf_counter()
    oracle.attention_f64(q[0], k[0], v[0])
    dt = time.perf_counter() - t0
    n = max(1, int(target_s / max(args_steps, 1) / max(dt, 1e-3)))
    return q, k, v, n


def attn_reference_arm(args, world, rank):
    if rank != 0:
        return 0
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    wl = WORKLOADS["attn"]
    T, Hq, Hkv, D = wl["context"], wl["hq"], wl["hkv"], wl["d"]
    q, k, v, n = attn_cpu(args.steps + args.warmup, wl, 60.0)
    for _ in range(args.warmup):
        for _ in range(n):
            oracle.attention_f64(q[0], k[0], v[0])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(n):
            oracle.attention_f64(q[0], k[0], v[0])
    dt = time.perf_counter() - t0
    value = args.steps * n * attn_bytes(1, T, Hq, Hkv, D) / dt / 1e9
    sample = (f"oracle.attention_f64 (fp64 numpy restatement of fp64_reference.attention) on {n} whole "
              f"sequences of context {T} per step; numpy/BLAS threads as available")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded; q, K, V ~ N(0,1) fp16)",
            "config": {"workload": wl["name"], "sample": "whole sequences, see cpu_baseline"},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def attn_measure(args, world, rank, dev, e2e=True):
    import torch
    from anvilq_b200 import ops
    wl = WORKLOADS["attn"]
    Bg, T, Hq, Hkv, D = wl["batch"], wl["context"], wl["hq"], wl["hkv"], wl["d"]
    if Bg % world:
        raise SystemExit(f"batch {Bg} does not split over {world} GPUs")
    B = Bg // world
    peak, peak_kind = load_peaks()
    gen = torch.Generator(device=dev)
    gen.manual_seed(17 + rank)
    k = torch.randn((B, T, Hkv, D), generator=gen, device=dev, dtype=torch.float16)
    v = torch.randn((B, T, Hkv, D), generator=gen, device=dev, dtype=torch.float16)
    q = torch.randn((B, Hq, D), generator=gen, device=dev, dtype=torch.float16)
    out = torch.empty_like(q)
    seqlens = torch.full((B,), T, dtype=torch.int32, device=dev)
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=torch.float16).pin_memory()
    stream = torch.cuda.Stream(dev)
    step_bytes = attn_bytes(B, T, Hq, Hkv, D)

    def step(host_io):
        def run():
            with torch.cuda.stream(stream):
                if host_io:
                    q.copy_(q_host, non_blocking=True)
                ops.gqa_decode(q, k, v, seqlens, out=out)
                if host_io:
                    out_host.copy_(out, non_blocking=True)
        return run

    with ClockSampler(dev.index) as clocks:
        ms = timed(step(False), stream, args.steps, args.warmup, world, dev)
    ms_e2e = timed(step(True), stream, args.steps, args.warmup, world, dev, sync_each=True) if e2e else None
    ops.raise_device_errors(dev)
    ms_step = ms / args.steps
    value = step_bytes * world * args.steps / (ms / 1e3) / 1e9
    achieved = step_bytes / (ms_step / 1e3) / 1e9   # one launch per step
    entry = traffic_entry("gqa_decode_kernel/attn")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16 q/K/V, fp32 scores and softmax",
        "data": "synthetic (seeded; q, K, V ~ N(0,1) fp16)",
        "config": {"workload": wl["name"], "batch": Bg, "batch_per_gpu": B, "context": T, "q_heads": Hq,
                   "kv_heads": Hkv, "head_dim": D, "step_bytes_per_gpu": step_bytes,
                   "l2": "KV per GPU larger than L2 (no flush)", "parallelism": f"batch-sharded x{world}"},
        "roofline": {"bound": "hbm", "kernel": "gqa_decode_kernel", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": int(step_bytes * entry["ratio_read_over_algorithmic"]) if entry else None,
                     "algorithmic_bytes_per_launch": step_bytes,
                     "launch_avg_us": round(ms_step * 1e3, 3)},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if ms_e2e is not None:
        line["e2e"] = {"value": round(step_bytes * world * args.steps / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                       "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": out.numel() * 2,
                       "ms_per_step": round(ms_e2e / args.steps, 5)}
    del k, v
    return line


def attn_arm(args, world, rank, local):
    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    line = attn_measure(args, world, rank, dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle
        wl = WORKLOADS["attn"]
        T, Hq, Hkv, D = wl["context"], wl["hq"], wl["hkv"], wl["d"]
        qc, kc, vc, n = attn_cpu(1, wl, 12.0)
        t0 = time.perf_counter()
        for _ in range(n):
            oracle.attention_f64(qc[0], kc[0], vc[0])
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {
            "value": round(n * attn_bytes(1, T, Hq, Hkv, D) / dt / 1e9, 4), "unit": "GB/s",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle.attention_f64 (fp64 numpy restatement of fp64_reference.attention) on {n} whole "
                      f"sequences of context {T}, {dt:.1f} s; numpy/BLAS threads as available"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ tp70b
def tp_measure(args, world, rank, dev, M, e2e=True):
    """Column-split 70B-class projections: per step, each rank's GEMM on its N/W slice
    and the all-gather of y, for the three layer shapes, as one CUDA graph."""
    import torch
    import torch.distributed as dist
    from anvilq_b200 import ops, synthetic
    wl = WORKLOADS["tp70b"]
    peak, peak_kind = load_peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    layers = []
    full_bytes = 0
    shard_bytes = 0
    for K, N in wl["shapes"]:
        n = N // world
        qw, qz, sc, _ = synthetic.device_awq_layer(K, n, 128, g, dev)
        x = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(7)).half()
        y = torch.empty(M, n, dtype=torch.float16, device=dev)
        yg = torch.empty(world * M, n, dtype=torch.float16, device=dev)
        layers.append((x, qw, qz, sc, y, yg, K, N))
        full_bytes += synthetic.gemv_bytes(M, K, N)
        shard_bytes += synthetic.gemv_bytes(M, K, n)
    stream = torch.cuda.Stream(dev)
    # at M = 1 the rank's slices run as one chain with one CTA shape (ops.chain_plans)
    plans = ops.chain_plans([(K, N // world) for K, N in wl["shapes"]]) if M == 1 else None

    def rank_gemm(i, x, qw, qz, sc, y, overlap=True):
        if plans is None:
            ops.gemm(x, qw, qz, sc, None, 128, out=y, overlap_prior=overlap)
        else:
            ops.gemv_planned(x, qw, qz, sc, None, 128, plan=plans[i], out=y.view(-1), overlap_prior=overlap)

    def step(gather=True):
        for i, (x, qw, qz, sc, y, yg, K, N) in enumerate(layers):
            rank_gemm(i, x, qw, qz, sc, y)
            if gather and world > 1:
                dist.all_gather_into_tensor(yg, y)

    def capture(fn):
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                fn()
        return graph

    g_full, g_comp = capture(lambda: step(True)), capture(lambda: step(False))
    # at M = 1 on several GPUs: the all-gather fused into each GEMV (peer stores over NVLink)
    fused = world > 1 and M == 1
    g_fused = outs = flins = None
    if fused:
        from anvilq_b200 import tp
        outs = tp.PeerOutputs(max(l[7] for l in layers), slots=len(layers), device=dev)
        flins = [tp.FusedTPLinear(qw, qz, sc, None, 128, outs, i, sharded=True)
                 for i, (x, qw, qz, sc, y, yg, K, N) in enumerate(layers)]

        def step_fused():
            for lin, l in zip(flins, layers):
                lin(l[0][0], flags=1)

        g_fused = capture(step_fused)
    # the projections chained through their gathered rows (each output row is the
    # next projection's x) with the deferred exchange: a call raises its flag and
    # moves on, the next call waits for every rank before reading x, and a flag
    # wait ends the step, so the exchange overlaps the next weight stream
    chained = (world > 1 and M == 1 and all(p["kernel"] == 1 for p in plans) and
               all(layers[i][7] == layers[i + 1][6] for i in range(len(layers) - 1)))
    g_chain = outs_c = clins = None
    if chained:
        from anvilq_b200 import tp
        outs_c = tp.PeerOutputs(max(l[7] for l in layers), slots=len(layers), device=dev)
        clins = [tp.FusedTPLinear(qw, qz, sc, None, 128, outs_c, i, sharded=True, plan=plans[i], deferred=True)
                 for i, (x, qw, qz, sc, y, yg, K, N) in enumerate(layers)]

        def step_chain(x0=None):
            y = layers[0][0][0] if x0 is None else x0
            for lin in clins:
                y = lin(y, flags=1)
            outs_c.wait()
            return y

        g_chain = capture(step_chain)

    def replay(graph):
        def run():
            with torch.cuda.stream(stream):
                graph.replay()
        return run

    with ClockSampler(dev.index) as clocks:
        ms = ms_nccl = timed(replay(g_full), stream, args.steps, args.warmup, world, dev)
        ms_fused = timed(replay(g_fused), stream, args.steps, args.warmup, world, dev) if fused else None
        ms_chain = timed(replay(g_chain), stream, args.steps, args.warmup, world, dev) if chained else None
    ms_comp = timed(replay(g_comp), stream, args.steps, args.warmup, world, dev)
    # the step runs whichever exchange was fastest here (max over ranks, so every rank agrees)
    best = min([("nccl", ms_nccl)] + ([("fused", ms_fused)] if fused else []) +
               ([("chain", ms_chain)] if chained else []), key=lambda t: t[1])
    path, ms = best
    fused, chained = path == "fused", path == "chain"
    ms_e2e = h2d = d2h = None
    if e2e:
        # activations from pinned host memory in, gathered outputs back to the host, every step
        x_host = [torch.randn(M, l[6]).half().pin_memory() for l in layers]
        y_host = [torch.empty(M, l[7], dtype=torch.float16).pin_memory() for l in layers]
        h2d = sum(t.numel() * 2 for t in x_host)
        d2h = sum(t.numel() * 2 for t in y_host)

        if chained:   # the chain's input row in, its last gathered row out
            h2d, d2h = x_host[0].numel() * 2, y_host[-1].numel() * 2

        def e2e_step():
            with torch.cuda.stream(stream):
                if chained:
                    x0 = layers[0][0]
                    x0.copy_(x_host[0], non_blocking=True)
                    y_host[-1].copy_(step_chain(x0[0]).view(1, -1), non_blocking=True)
                    return
                for i, ((x, qw, qz, sc, y, yg, K, N), xh, yh) in enumerate(zip(layers, x_host, y_host)):
                    x.copy_(xh, non_blocking=True)
                    if fused:
                        yh.copy_(flins[i](x[0]).view(1, -1), non_blocking=True)
                        continue
                    rank_gemm(i, x, qw, qz, sc, y, overlap=False)
                    if world > 1:
                        dist.all_gather_into_tensor(yg, y)
                        yh.copy_(yg.view(world, M, -1).permute(1, 0, 2).reshape(M, -1), non_blocking=True)
                    else:
                        yh.copy_(y, non_blocking=True)

        ms_e2e = timed(e2e_step, stream, args.steps, args.warmup, world, dev, sync_each=True)
    # every rank learns whether any rank's kernels flagged an error (a bounded
    # wait that expired, say) before anyone raises, so that all ranks release
    # the peer buffers together and leave at the same point
    bits = int(ops.device_error_word(dev).item())
    any_bits = int(max_over_ranks(float(bits), world, dev))
    del g_full, g_comp, g_fused, g_chain
    for o in (outs, outs_c):
        if o is not None:
            o.close()
    if bits:
        ops.raise_device_errors(dev)
    if any_bits:
        raise RuntimeError(f"another rank's kernels flagged device error bits {any_bits}")
    launches = 3
    value = full_bytes * args.steps / (ms / 1e3) / 1e9
    per_launch = ms_comp / args.steps / launches
    achieved = shard_bytes / launches / (per_launch / 1e3) / 1e9
    kernel_of = lambda pl: "gemv_stream_kernel" if pl["kernel"] == 1 else "gemv_tma_kernel"
    kernel = kernel_of(plans[0]) if M == 1 else "verify_tc_kernel"
    traffic = weighted_traffic("tp70b", [(synthetic.gemv_bytes(M, K, N // world), kernel_of(pl))
                                         for (K, N), pl in zip(wl["shapes"], plans)]) if M == 1 else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 activations x int4 weights, fp32 accumulate",
        "data": "synthetic (seeded on the device; x~N(0,1), u4 uniform, scales |N(0,1)|*0.01+1e-3)",
        "config": {"workload": wl["name"], "M": M, "group": 128, "full_bytes_per_step": full_bytes,
                   "shard_bytes_per_rank": shard_bytes, "parallelism": f"tp{world} (column split)",
                   "graph": ("one CUDA graph per step: 3 GEMVs chained through their gathered rows, each "
                             "storing its slice into every rank's output over NVLink and raising its flag; "
                             "each waits for every rank before reading x, a flag wait ends the step"
                             if chained else
                             "one CUDA graph per step: 3 GEMVs, each storing its slice into every rank's "
                             "output over NVLink and exchanging completion flags (all-gather fused in)" if fused
                             else "one CUDA graph per step: 3 GEMMs + 3 NCCL all-gathers" if world > 1
                             else "one CUDA graph per step: 3 GEMMs (one GPU holds every column)"),
                   "nccl_allgather_path_ms_per_step": round(ms_nccl / args.steps, 5),
                   "fused_allgather_path_ms_per_step": None if ms_fused is None else round(ms_fused / args.steps, 5),
                   "deferred_chain_path_ms_per_step": None if ms_chain is None else round(ms_chain / args.steps, 5),
                   "exchange_path": path,
                   "compute_only_ms_per_step": round(ms_comp / args.steps, 5),
                   "exchange_ms_per_step": round(max(0.0, ms - ms_comp) / args.steps, 5),
                   "rank_plans": plans,
                   "l2": "weights larger than L2 (no flush)"},
        "roofline": {"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                     "algorithmic_bytes_per_launch": int(shard_bytes / launches),
                     "launch_avg_us": round(per_launch * 1e3, 4),
                     "measured_on": "the rank's three GEMVs without the exchange, same run"},
        "gpu_launches": launches * args.steps,
        "clocks": clocks.summary(),
    }
    if ms_e2e is not None:
        line["e2e"] = {"value": round(full_bytes * args.steps / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "ms_per_step": round(ms_e2e / args.steps, 5)}
    return line


def tp_arm(args, world, rank, local):
    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    line = tp_measure(args, world, rank, dev, args.tokens)
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("anvilq", "reference"), default="anvilq")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode05b")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode05b: skip the proj7b / tp70b / attn measurements on the same line")
    ap.add_argument("--tokens", type=int, default=1, help="token rows per projection (tp70b)")
    ap.add_argument("--fused", action="store_true",
                    help="decode05b: the fused layers kernel instead of one kernel per operation")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return reference_arm(args, world, rank)
    world, rank, local = dist_init()
    try:
        if args.workload in ("decode05b", "decode7b"):
            return decode_arm(args, world, rank, local)
        if args.workload == "tp70b":
            return tp_arm(args, world, rank, local)
        if args.workload == "attn":
            return attn_arm(args, world, rank, local)
        return anvilq_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
