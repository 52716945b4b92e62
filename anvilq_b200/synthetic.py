"""Seeded synthetic AWQ layers and KV caches with the reference's value distributions.

No dataset or checkpoint is available offline, so every workload is generated
from a seed (17 by default; 43 and 89 are the reference's extra seeds,
anvil-q1/design/SPEC.md:316):

* activations fp16 ~ N(0, 1);
* int4 weights and zero points uniform on 0..15, AWQ-packed 8 per int32.  A
  uniformly random 32-bit word holds 8 independent uniform nibbles whatever
  the packing order, so packed words are drawn directly;
* scales fp16 = |N(0, 1)| * 0.01 + 1e-3;
* attention Q/K/V fp16 ~ N(0, 1).

Arrays are numpy, host side; callers move them to the device.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class AwqLayer:
    """One W4A16 AWQ linear layer in the reference's storage layout.

    qweight int32 [K, N/8], qzeros int32 [K/G, N/8], scales fp16 [K/G, N],
    bias fp16 [N] or None (anvil-q1/tests/official_weights.py:76-85).
    """
    qweight: np.ndarray
    qzeros: np.ndarray
    scales: np.ndarray
    bias: np.ndarray | None
    group: int

    @property
    def K(self) -> int:
        return self.qweight.shape[0]

    @property
    def N(self) -> int:
        return self.qweight.shape[1] * 8

    @property
    def scales_bits(self) -> np.ndarray:
        return self.scales.view(np.uint16)

    @property
    def bias_bits(self) -> np.ndarray | None:
        return None if self.bias is None else self.bias.view(np.uint16)

    def nbytes(self) -> int:
        b = self.qweight.nbytes + self.qzeros.nbytes + self.scales.nbytes
        return b + (0 if self.bias is None else self.bias.nbytes)


def awq_layer(K: int, N: int, G: int = 128, seed: int = 17, bias: bool = False,
              rng: np.random.Generator | None = None) -> AwqLayer:
    if K % G or N % 8:
        raise ValueError("K must be a multiple of G and N a multiple of 8")
    rng = rng if rng is not None else np.random.default_rng(seed)
    qweight = rng.integers(0, 2**32, size=(K, N // 8), dtype=np.uint32).view(np.int32)
    qzeros = rng.integers(0, 2**32, size=(K // G, N // 8), dtype=np.uint32).view(np.int32)
    scales = (np.abs(rng.standard_normal((K // G, N), dtype=np.float32)) * 0.01 + 1e-3).astype(np.float16)
    b = rng.standard_normal(N, dtype=np.float32).astype(np.float16) if bias else None
    return AwqLayer(qweight, qzeros, scales, b, G)


def device_awq_layer(K: int, N: int, G: int, generator, device, bias: bool = False):
    """(qweight, qzeros, scales, bias or None) drawn on the device from a seeded
    torch generator with the distributions of ``awq_layer`` (u4 uniform weights
    and zeros, scales |N(0,1)| * 0.01 + 1e-3, bias N(0,1)); for benchmark-sized
    layers that would take seconds to draw on the host."""
    import torch
    if K % G or N % 8:
        raise ValueError("K must be a multiple of G and N a multiple of 8")
    qw = torch.randint(-2**31, 2**31 - 1, (K, N // 8), dtype=torch.int32, device=device, generator=generator)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), dtype=torch.int32, device=device, generator=generator)
    sc = (torch.randn((K // G, N), device=device, generator=generator).abs() * 0.01 + 1e-3).half()
    b = torch.randn(N, device=device, generator=generator).half() if bias else None
    return qw, qz, sc, b


def activations(M: int, K: int, seed: int = 17, rng: np.random.Generator | None = None) -> np.ndarray:
    rng = rng if rng is not None else np.random.default_rng(seed)
    return rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)


def gemv_case(M: int, K: int, N: int, G: int = 128, seed: int = 17, bias: bool = False):
    """(x fp16 [M,K], AwqLayer) drawn from one seeded stream: x first, then the layer."""
    rng = np.random.default_rng(seed)
    x = activations(M, K, rng=rng)
    return x, awq_layer(K, N, G, rng=rng, bias=bias)


def kv_case(B: int, Hq: int, Hkv: int, D: int, T: int, seed: int = 17):
    """q fp16 [B,Hq,D], k/v caches fp16 [B,T,Hkv,D] ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, Hq, D), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((B, T, Hkv, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((B, T, Hkv, D), dtype=np.float32).astype(np.float16)
    return q, k, v


def gemv_bytes(M: int, K: int, N: int, G: int = 128, bias: bool = False) -> int:
    """Algorithmic HBM bytes of one W4A16 GEMM launch: each byte moved once.

    K*N/2 (int4 weights) + (K/G)*(N/8)*4 (zeros) + (K/G)*N*2 (scales)
    + M*K*2 (x) + M*N*2 (y) [+ N*2 bias].
    """
    b = K * N // 2 + (K // G) * (N // 8) * 4 + (K // G) * N * 2 + M * K * 2 + M * N * 2
    return b + (N * 2 if bias else 0)


def attention_bytes(B: int, Hq: int, Hkv: int, D: int, T: int) -> int:
    """K and V read once plus q in and out written: B*T*Hkv*D*2*2 + 2*B*Hq*D*2."""
    return B * T * Hkv * D * 4 + 2 * B * Hq * D * 2
