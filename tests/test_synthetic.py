"""The seeded synthetic inputs follow the value distributions the benchmark
configurations name: x ~ N(0,1) fp16; int4 weights and zeros uniform 0..15 in
AWQ packing; scales fp16 = |N(0,1)| * 0.01 + 1e-3 (G = 128); attention Q/K/V
~ N(0,1) fp16.  Also the algorithmic byte counts the bench divides by."""
import numpy as np

import oracle
from anvilq_b200 import synthetic


def test_awq_layer_distributions():
    lay = synthetic.awq_layer(4096, 4096, 128, seed=17, bias=True)
    assert lay.qweight.shape == (4096, 512) and lay.qzeros.shape == (32, 512) and lay.scales.shape == (32, 4096)
    codes = oracle.unpack_lanes(lay.qweight.view(np.uint32), 4096)
    counts = np.bincount(codes.ravel(), minlength=16)
    assert counts.size == 16 and counts.min() > 0
    assert np.abs(counts / counts.sum() - 1 / 16).max() < 0.002          # uniform 0..15
    zeros = oracle.unpack_lanes(lay.qzeros.view(np.uint32), 4096)
    assert zeros.min() == 0 and zeros.max() == 15
    s = lay.scales.astype(np.float64)
    assert s.min() >= 1e-3 - 1e-6                                          # |N(0,1)| * 0.01 + 1e-3
    assert abs(s.mean() - (0.01 * np.sqrt(2 / np.pi) + 1e-3)) < 2e-4
    assert lay.bias is not None and abs(float(lay.bias.astype(np.float64).std()) - 1.0) < 0.05


def test_activations_and_kv_are_standard_normal_fp16():
    x = synthetic.activations(4, 8192, seed=43)
    assert x.dtype == np.float16 and abs(float(x.astype(np.float64).mean())) < 0.03
    assert abs(float(x.astype(np.float64).std()) - 1.0) < 0.02
    q, k, v = synthetic.kv_case(2, 32, 8, 128, 256, seed=89)
    assert q.shape == (2, 32, 128) and k.shape == (2, 256, 8, 128) and v.dtype == np.float16
    assert abs(float(k.astype(np.float64).std()) - 1.0) < 0.02


def test_generators_are_seeded():
    a = synthetic.gemv_case(1, 896, 4864, 128, 17)
    b = synthetic.gemv_case(1, 896, 4864, 128, 17)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].qweight, b[1].qweight)
    c = synthetic.gemv_case(1, 896, 4864, 128, 43)
    assert not np.array_equal(a[1].qweight, c[1].qweight)


def test_algorithmic_bytes():
    """K N/2 + (K/G)(N/8) 4 + (K/G) N 2 + M K 2 + M N 2 (+ N 2 bias)."""
    assert synthetic.gemv_bytes(1, 896, 4864, 128) == 2_275_712
    assert synthetic.gemv_bytes(1, 4096, 11008, 128) == 23_455_232
    assert synthetic.gemv_bytes(1, 28672, 8192, 128) == 122_101_760
    assert synthetic.gemv_bytes(1, 896, 4864, 128, bias=True) == 2_275_712 + 4864 * 2
    assert synthetic.attention_bytes(64, 32, 8, 128, 32768) == 64 * 32768 * 8 * 128 * 2 * 2 + 2 * 64 * 32 * 128 * 2
