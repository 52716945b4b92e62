"""GPU parity of the tensor-core (tcgen05 + TMEM) speculative-verify GEMM.

Every row of the verify GEMM is FP32Model.linear (anvil-q1/tests/official_weights.py:418-437)
of one token; the oracle's C restatement of it is the reference here.  The
kernel feeds the exact integer deltas q - z to the tensor cores and applies each
group's scale in fp32, so its only departures from the reference are the
accumulation order and the final fp16 rounding of y.
"""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import synthetic

pytestmark = pytest.mark.gpu

# anvil-q1-fp/design/SPEC.md:311-317 per-operator tolerance (as for the other GEMM paths)
TOL_ERR, TOL_COS = 2e-3, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _run(dev, M, K, N, seed, bias=False, forced=True):
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(M, K, N, 128, seed, bias=bias)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                           layer.bias_bits, 128, threads=oracle.max_threads())
    args = (T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev),
            None if layer.bias is None else T(layer.bias, dev), 128)
    fn = ops.verify_gemm if forced else ops.gemm
    y1 = fn(*args)
    y2 = fn(*args)                 # tickets re-armed by the first call; fixed summation order
    ops.raise_device_errors(dev)
    assert torch.equal(y1, y2), "verify GEMM is not run-to-run deterministic"
    err, cos = oracle.normalized_error(y1.float().cpu().numpy(), ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (M, K, N, err, cos)
    return y1, ref


# the speculative-verify grid: M in {16, 32, 64} x the 7B projection shapes
@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("M", [16, 32, 64])
def test_verify_grid(dev, M, K, N):
    _run(dev, M, K, N, seed=100 + M, forced=False)


@pytest.mark.parametrize("M", [1, 4, 5, 8, 17, 33, 48, 100])
def test_tensor_core_path_any_m(dev, M):
    """Forced onto the tensor cores: MPAD 16/32/48/64 and the 64-row chunking (M = 100)."""
    _run(dev, M, 896, 4864, seed=7 + M, bias=(M % 2 == 1))


@pytest.mark.parametrize("K,N", [(128, 32), (1024, 4128), (896, 896), (256, 160)])
def test_partial_tiles_and_single_group(dev, K, N):
    """Column tiles past N (zero-filled by the TMA unit) and a single-group K."""
    _run(dev, 24, K, N, seed=K + N, bias=True)


def test_tensor_cores_match_cuda_cores(dev):
    """At M = 8 both paths exist; both stay within tolerance of the reference."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(8, 4096, 4096, 128, 5)
    args = (T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 128)
    y_tc = ops.verify_gemm(*args).float().cpu().numpy()
    y_cc = ops.gemm(*args).float().cpu().numpy()
    ops.raise_device_errors(dev)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, None, 128,
                           threads=oracle.max_threads())
    for y in (y_tc, y_cc):
        err, cos = oracle.normalized_error(y, ref)
        assert err <= TOL_ERR and cos >= TOL_COS


def test_invalid_scale_raises(dev):
    from anvilq_b200 import ops, AnvilqError
    x, layer = synthetic.gemv_case(16, 512, 256, 128, 17)
    for bad in (0x7C00, 0xFE00, 0x8001):
        sc = layer.scales_bits.copy()
        sc[3, 200] = bad
        ops.verify_gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(sc.view(np.float16), dev),
                        None, 128)
        with pytest.raises(AnvilqError):
            ops.raise_device_errors(dev)


def test_unsupported_shape_is_refused(dev):
    from anvilq_b200 import ops, AnvilqError
    x, layer = synthetic.gemv_case(16, 192, 256, 64, 3)   # group 64: not the tensor-core layout
    with pytest.raises(AnvilqError):
        ops.verify_gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 64)
    y = ops.gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 64)
    ops.raise_device_errors(dev)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, None, 64)
    err, cos = oracle.normalized_error(y.float().cpu().numpy(), ref)
    assert err <= TOL_ERR and cos >= TOL_COS


def _unpack_tc_layout(packed, K, N):
    """Inverse of the packed layout (anvilq.h: anvilq_w4a16_tc_pack): u4 codes [K, N]."""
    awq_lane = [0, 2, 4, 6, 1, 3, 5, 7]
    tiles, groups = -(-N // 128), K // 128
    words = packed.reshape(tiles, groups, 2, 4, 2, 32, 4).astype(np.uint32)   # t g h q half lane j
    codes = np.zeros((K, tiles * 128), np.uint8)
    t, g, h, q, half, lane, j = np.indices(words.shape)
    blk = half * 4 + j
    r, l = lane // 4, lane % 4
    col = t * 128 + q * 32 + 8 * l + np.take(awq_lane, r)
    for jj in range(8):
        k = g * 128 + 64 * h + 8 * blk + awq_lane[jj]
        codes[k, col] = (words >> np.uint32(4 * jj)) & np.uint32(0xF)
    return codes[:, :N]


@pytest.mark.parametrize("K,N", [(256, 288), (4096, 4096)])
def test_tc_pack_layout_round_trip(dev, K, N):
    """The resident layout holds exactly the AWQ nibbles (bit-exact round trip)."""
    from anvilq_b200 import ops
    _, layer = synthetic.gemv_case(1, K, N, 128, 3)
    packed = ops.tc_pack(T(layer.qweight, dev)).cpu().numpy().view(np.uint32)
    codes = oracle.unpack_rows(layer.qweight.view(np.uint32), N)
    assert np.array_equal(_unpack_tc_layout(packed, K, N), codes)


@pytest.mark.parametrize("M,K,N", [(16, 4096, 11008), (64, 11008, 4096), (5, 896, 4864), (24, 1024, 4128)])
def test_packed_verify_gemm_matches_unpacked(dev, M, K, N):
    """Packed and AWQ-layout kernels compute the same sums in the same order: bit-identical."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(M, K, N, 128, 9, bias=True)
    args = (T(layer.qzeros, dev), T(layer.scales, dev), T(layer.bias, dev), 128)
    xd, qw = T(x, dev), T(layer.qweight, dev)
    y_std = ops.verify_gemm(xd, qw, *args)
    y_pk = ops.verify_gemm_packed(xd, ops.tc_pack(qw), *args)
    ops.raise_device_errors(dev)
    assert torch.equal(y_std, y_pk)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits,
                           128, threads=oracle.max_threads())
    err, cos = oracle.normalized_error(y_pk.float().cpu().numpy(), ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (M, K, N, err, cos)
