"""Small, self-contained launch sequences of one kernel, for profiling with ncu.

    python -m anvilq_b200.profile_case gemv --K 4096 --N 11008 --M 1 --sets 8 --reps 2
    python -m anvilq_b200.profile_case gemv --K 4096 --N 11008 --plan '{"kernel": 1, "band_cols": 256,
        "cluster": 1, "kc": 1, "warps": 8, "stages": 3, "ctas": 296}'
    python -m anvilq_b200.profile_case attn --B 8 --T 32768 --reps 4

Allocates `sets` independent weight sets of one shape (chosen so that together
they exceed the 126 MB L2; the default 8 x 23.5 MB = 188 MB) and launches the
GEMM once per set per repetition, so that every profiled launch reads its
weights from HBM.  The launches are replayed as one CUDA graph (unless --no-graph) and timed with
CUDA events; prints the mean time per launch and the algorithmic bytes per
launch.  The attn case launches decode attention (32/8 heads of 128, every
sequence at full length) over a KV cache of B x T rows (1 GB at B=8,
T=32768).  Numbers taken under a profiler are not results.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops, synthetic


def gemv_sets(args, dev):
    """`sets` independent (x, qweight, qzeros, scales, y) of one shape, drawn on the device."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed)
    sets = []
    for _ in range(args.sets):
        qw, qz, sc, _ = synthetic.device_awq_layer(args.K, args.N, args.G, gen, dev)
        x = torch.randn((args.M, args.K), generator=gen, device=dev).half()
        sets.append((x, qw, qz, sc, torch.empty((args.M, args.N), dtype=torch.float16, device=dev)))
    return sets


def gemv_case(args, sets=None):
    dev = torch.device("cuda", 0)
    sets = sets if sets is not None else gemv_sets(args, dev)
    plan = json.loads(args.plan) if args.plan else None
    stream = torch.cuda.Stream(dev)

    def enqueue():
        for x, qw, qz, sc, y in sets:
            if plan is not None:
                ops.gemv_planned(x, qw, qz, sc, None, args.G, plan=plan, out=y, overlap_prior=args.overlap)
            else:
                ops.gemm(x, qw, qz, sc, None, args.G, out=y, overlap_prior=args.overlap)

    with torch.cuda.stream(stream):
        enqueue()                        # warm: workspaces, module load
    stream.synchronize()
    graph = None
    if args.graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            enqueue()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(2):
            graph.replay() if graph is not None else enqueue()
        start.record(stream)
        for _ in range(args.reps):
            graph.replay() if graph is not None else enqueue()
        end.record(stream)
    stream.synchronize()
    ops.raise_device_errors(dev)
    n = args.reps * args.sets
    us = start.elapsed_time(end) * 1e3 / n
    b = synthetic.gemv_bytes(args.M, args.K, args.N, args.G)
    used = plan if plan is not None else (ops.gemv_plan(args.K, args.N, args.G) if args.M == 1 else None)
    print(json.dumps({"case": "gemv", "M": args.M, "K": args.K, "N": args.N, "launches": n,
                      "graph": bool(args.graph), "overlap_prior": bool(args.overlap), "plan": used,
                      "us_per_launch": round(us, 3), "bytes_per_launch": b, "GBps": round(b / us / 1e3, 1)}),
          flush=True)


def attn_case(args):
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed)
    Hq, Hkv, D = 32, 8, 128
    k = torch.randn((args.B, args.T, Hkv, D), generator=gen, device=dev, dtype=torch.float16)
    v = torch.randn((args.B, args.T, Hkv, D), generator=gen, device=dev, dtype=torch.float16)
    q = torch.randn((args.B, Hq, D), generator=gen, device=dev, dtype=torch.float16)
    out = torch.empty_like(q)
    seqlens = torch.full((args.B,), args.T, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(2):
            ops.gqa_decode(q, k, v, seqlens, out=out)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.reps):
            ops.gqa_decode(q, k, v, seqlens, out=out)
        end.record(stream)
    stream.synchronize()
    ops.raise_device_errors(dev)
    us = start.elapsed_time(end) * 1e3 / args.reps
    b = args.B * args.T * Hkv * D * 2 * 2 + 2 * args.B * Hq * D * 2
    print(json.dumps({"case": "attn", "B": args.B, "T": args.T, "heads": [Hq, Hkv, D], "launches": args.reps,
                      "us_per_launch": round(us, 3), "bytes_per_launch": b, "GBps": round(b / us / 1e3, 1)}))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("case", choices=("gemv", "attn"))
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--T", type=int, default=32768)
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--N", type=int, default=11008)
    ap.add_argument("--G", type=int, default=128)
    ap.add_argument("--sets", type=int, default=8)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--seed", type=int, default=17)
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch eagerly from Python instead of replaying a CUDA graph")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="launch without programmatic dependent launch")
    ap.add_argument("--plan", default=None,
                    help="M = 1: a GEMV plan as JSON (the fields of anvilq_gemv_plan) instead of the default")
    args = ap.parse_args(argv)
    attn_case(args) if args.case == "attn" else gemv_case(args)


if __name__ == "__main__":
    main()
