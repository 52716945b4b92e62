"""CUDA-graph captured sequences of W4A16 AWQ GEMMs over resident weights.

A decode step reads every projection of every layer once.  ``ProjectionStream``
holds such a set of layers in HBM and replays all their GEMMs as one CUDA graph,
so per-launch host overhead disappears and consecutive kernels overlap their
tails.  ``host_io=True`` adds, inside the same graph, the copy of every
projection's activations from pinned host memory and the copy of every output
back to pinned host memory: the end-to-end form of the step.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops, synthetic

# Qwen2.5-0.5B (anvil-q1/tests/official_weights.py:21 DEFAULT_SHAPE and :72-85):
# hidden 896, intermediate 4864, 14/2 heads of 64 -> q 896, k/v 128.
QWEN05B_PROJECTIONS = ((896, 896, True), (896, 128, True), (896, 128, True), (896, 896, False),
                       (896, 4864, False), (896, 4864, False), (4864, 896, False))
# Llama-7B-class layer: q,k,v,o 4096x4096, gate/up 4096x11008, down 11008x4096.
LLAMA7B_PROJECTIONS = ((4096, 4096, False),) * 4 + ((4096, 11008, False),) * 2 + ((11008, 4096, False),)


class ProjectionStream:
    def __init__(self, projections, layers: int, M: int = 1, group: int = 128, seed: int = 17,
                 device="cuda", host_io: bool = False, device_init: bool = False):
        """device_init: draw the weights and activations on the device (a seeded
        torch generator, same value distributions) instead of on the host --
        gigabytes of 7B-class layers in well under a second."""
        self.device = torch.device(device)
        self.M, self.group, self.host_io = M, group, host_io
        self.layers = []
        rng = np.random.default_rng(seed)
        gen = None
        if device_init:
            gen = torch.Generator(device=self.device)
            gen.manual_seed(seed)
        for _ in range(layers):
            for K, N, bias in projections:
                if gen is not None:
                    qw, qz, sc, b = synthetic.device_awq_layer(K, N, group, gen, self.device, bias=bias)
                    x = torch.randn((M, K), generator=gen, device=self.device).half()
                    entry = dict(K=K, N=N, qweight=qw, qzeros=qz, scales=sc, bias=b, x=x)
                    x_np = x.cpu().numpy() if host_io else None
                else:
                    lay = synthetic.awq_layer(K, N, group, rng=rng, bias=bias)
                    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(self.device)
                    x_np = synthetic.activations(M, K, rng=rng)
                    entry = dict(K=K, N=N, qweight=t(lay.qweight), qzeros=t(lay.qzeros), scales=t(lay.scales),
                                 bias=t(lay.bias), x=t(x_np))
                entry["y"] = torch.empty((M, N), dtype=torch.float16, device=self.device)
                if host_io:
                    entry["x_host"] = torch.from_numpy(x_np).pin_memory()
                    entry["y_host"] = torch.empty((M, N), dtype=torch.float16).pin_memory()
                self.layers.append(entry)
        self.graph = None
        self.stream = torch.cuda.Stream(self.device)

    # -- accounting ---------------------------------------------------------
    def algorithmic_bytes(self) -> int:
        return sum(synthetic.gemv_bytes(self.M, e["K"], e["N"], self.group, e["bias"] is not None)
                   for e in self.layers)

    def h2d_bytes(self) -> int:
        return sum(e["x"].numel() * 2 for e in self.layers) if self.host_io else 0

    def d2h_bytes(self) -> int:
        return sum(e["y"].numel() * 2 for e in self.layers) if self.host_io else 0

    def launches(self) -> int:
        return len(self.layers) * ((self.M + 7) // 8)

    # -- execution ------------------------------------------------------------
    def _enqueue(self):
        for e in self.layers:
            if self.host_io:
                e["x"].copy_(e["x_host"], non_blocking=True)
            ops.gemm(e["x"], e["qweight"], e["qzeros"], e["scales"], e["bias"], self.group, out=e["y"],
                     overlap_prior=True)
            if self.host_io:
                e["y_host"].copy_(e["y"], non_blocking=True)

    def capture(self):
        with torch.cuda.stream(self.stream):
            self._enqueue()                    # warm: workspaces allocated, kernels loaded
        self.stream.synchronize()
        ops.raise_device_errors(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._enqueue()
        return self

    def run(self):
        """Enqueue one step on ``self.stream`` (graph replay if captured)."""
        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._enqueue()

    def outputs(self):
        return [e["y"] for e in self.layers]
