"""Small, self-contained launch sequences of one kernel, for profiling with ncu.

    python -m anvilq_b200.profile_case gemv --K 4096 --N 11008 --M 1 --sets 8 --reps 2

Allocates `sets` independent weight sets of one shape (chosen so that together
they exceed the 126 MB L2; the default 8 x 23.5 MB = 188 MB) and launches the
GEMM once per set per repetition, so that every profiled launch reads its
weights from HBM.  Prints the mean device time per launch (CUDA events) and the
algorithmic bytes per launch; numbers taken under a profiler are not results.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import ops, synthetic


def gemv_case(args):
    dev = torch.device("cuda", 0)
    sets = []
    rng = np.random.default_rng(args.seed)
    for _ in range(args.sets):
        lay = synthetic.awq_layer(args.K, args.N, args.G, rng=rng)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        sets.append((t(synthetic.activations(args.M, args.K, rng=rng)), t(lay.qweight), t(lay.qzeros),
                     t(lay.scales), torch.empty((args.M, args.N), dtype=torch.float16, device=dev)))
    for x, qw, qz, sc, y in sets:       # warm: workspaces, module load
        ops.gemm(x, qw, qz, sc, None, args.G, out=y)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.reps):
        for x, qw, qz, sc, y in sets:
            ops.gemm(x, qw, qz, sc, None, args.G, out=y)
    end.record()
    torch.cuda.synchronize()
    ops.raise_device_errors(dev)
    n = args.reps * args.sets
    us = start.elapsed_time(end) * 1e3 / n
    b = synthetic.gemv_bytes(args.M, args.K, args.N, args.G)
    print(json.dumps({"case": "gemv", "M": args.M, "K": args.K, "N": args.N, "launches": n,
                      "us_per_launch_incl_host": round(us, 3), "bytes_per_launch": b,
                      "GBps": round(b / us / 1e3, 1)}))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("case", choices=("gemv",))
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--N", type=int, default=11008)
    ap.add_argument("--G", type=int, default=128)
    ap.add_argument("--sets", type=int, default=8)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--seed", type=int, default=17)
    args = ap.parse_args(argv)
    gemv_case(args)


if __name__ == "__main__":
    main()
