"""GPU parity of the bit-accurate Q16.16 integer GEMV (anvilq_w4a16_gemm_q16).

The reference's integer model (anvil-q1/tests/official_weights.py:592-612) is exact
integer arithmetic, so the bar is bit-identical outputs: against the integer
outputs the reference itself produced (tests/golden/linear.npz `*_yq16`), and
against the oracle's C restatement (pinned to those fixtures) at larger sizes.
"""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _fixture_cases(g):
    names = ["official_p0", "official_p1", "official_p4"] + [str(n) for n in g["case_names"]]
    for key in names:
        if key + "_yq16" not in g:
            continue
        G = int(g[key + "_G"]) if key + "_G" in g else 128
        bias = g[key + "_bias"] if key + "_bias" in g else None
        yield key, g[key + "_xq16"], g[key + "_qweight"], g[key + "_qzeros"], g[key + "_scales"], bias, G, \
            g[key + "_yq16"]


def test_reference_integer_outputs(dev, golden_dir):
    """Every integer-model output the reference produced, reproduced bit for bit."""
    from anvilq_b200 import ops
    g = np.load(golden_dir / "linear.npz")
    n = 0
    for key, xq, qw, qz, sc, bias, G, yref in _fixture_cases(g):
        y = ops.gemm_q16(T(np.atleast_2d(xq).astype(np.int32), dev), T(qw.view(np.int32), dev),
                         T(qz.view(np.int32), dev), T(sc.view(np.float16), dev),
                         None if bias is None else T(bias.view(np.float16), dev), G)
        ops.raise_device_errors(dev)
        assert np.array_equal(y.cpu().numpy().reshape(np.shape(yref)), yref), key
        n += 1
    assert n >= 3


def _q16_activations(M, K, seed):
    rng = np.random.default_rng(seed)
    return np.round(rng.standard_normal((M, K)) * 65536.0).astype(np.int32)


@pytest.mark.parametrize("M,K,N,G,bias", [(1, 896, 4864, 128, False), (1, 896, 896, 128, True),
                                          (2, 4096, 4096, 128, False), (1, 1000, 256, 128, True),
                                          (1, 768, 128, 64, True), (3, 256, 64, 32, False)])
def test_matches_oracle(dev, M, K, N, G, bias):
    from anvilq_b200 import ops
    Kg = -(-K // G) * G
    _, layer = synthetic.gemv_case(1, Kg, N, G, K + N, bias=bias)
    if Kg != K:   # a partial last group: drop rows, keep the group's zero points and scales
        layer.qweight = np.ascontiguousarray(layer.qweight[:K])
    x = _q16_activations(M, K, G + M)
    ref = oracle.gemv_q16(x, layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits, G,
                          threads=oracle.max_threads())
    y = ops.gemm_q16(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev),
                     None if layer.bias is None else T(layer.bias, dev), G)
    ops.raise_device_errors(dev)
    assert np.array_equal(y.cpu().numpy(), ref)


def test_wide_cancellation_and_saturation(dev):
    """verify.py:536-615 test_case 0 (K=9216, G=8, scale 0x7bff): column 1 saturates positive,
    column 2 negative, and the second half cancels the others to zero (needs > 64-bit sums)."""
    from anvilq_b200 import ops
    K, G = 9216, 8
    x = np.where(np.arange(K) < 4608, 8388352, -8388352).astype(np.int32)[None, :]
    qweight = np.where(np.arange(K) < 4608, 0xFFFFFF0F, 0xFFF0FF0F).astype(np.uint32)[:, None]
    qzeros = np.where(np.arange(K // G) < 576, 0x000000F0, 0).astype(np.uint32)[:, None]
    scales = np.full((K // G, 8), 0x7BFF, np.uint16)
    y = ops.gemm_q16(T(x, dev), T(qweight.view(np.int32), dev), T(qzeros.view(np.int32), dev),
                     T(scales.view(np.float16), dev), None, G)
    ops.raise_device_errors(dev)
    assert y[0].tolist() == [0, 0x7FFFFFFF, -0x80000000, 0, 0, 0, 0, 0]


def test_invalid_parameters_fail(dev):
    from anvilq_b200 import ops, AnvilqError
    _, layer = synthetic.gemv_case(1, 256, 64, 128, 5, bias=True)
    x = T(_q16_activations(1, 256, 1), dev)
    for bad in (0x7C00, 0xFE00, 0x8001):
        sc = layer.scales_bits.copy()
        sc[1, 9] = bad
        ops.gemm_q16(x, T(layer.qweight, dev), T(layer.qzeros, dev), T(sc.view(np.float16), dev), None, 128)
        with pytest.raises(AnvilqError):
            ops.raise_device_errors(dev)
    b = layer.bias_bits.copy()
    b[3] = 0x7E00
    ops.gemm_q16(x, T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), T(b.view(np.float16), dev),
                 128)
    with pytest.raises(AnvilqError):
        ops.raise_device_errors(dev)


def test_shared_workspace_counters_stay_zero(dev):
    """The Q16 kernel shares ops.workspace with the split-K kernels, whose arrival
    counters (the first ANVILQ_WORKSPACE_COUNTER_BYTES) must stay zero between calls."""
    from anvilq_b200 import ops
    _, layer = synthetic.gemv_case(1, 4096, 4096, 128, 3)
    x = T(_q16_activations(2, 4096, 4), dev)
    ops.gemm_q16(x, T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 128)
    ops.raise_device_errors(dev)
    ws = ops.workspace(dev, 1)
    assert int(ws[:65536].count_nonzero()) == 0


def test_golden_api_linear_q16(dev):
    """GpuLinear.linear_q16: the integer model's projection over the checkpoint, bit-identical."""
    from anvilq_b200.checkpoint import ArrayCheckpoint, gemv_shape
    from anvilq_b200.golden_api import GpuLinear
    _, layer = synthetic.gemv_case(1, 512, 128, 128, 61, bias=True)
    x = _q16_activations(1, 512, 62)[0]
    ckpt = ArrayCheckpoint({(0, 0): layer})
    y = GpuLinear(ckpt, gemv_shape(512, 128, 128, 0)).linear_q16([int(v) for v in x], 0, 0)
    ref = oracle.gemv_q16(x[None], layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits, 128)
    assert y == [int(v) for v in ref[0]]
