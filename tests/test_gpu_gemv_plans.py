"""GPU parity of the batch-1 GEMV plans against the oracle (FP32Model.linear,
anvil-q1/tests/official_weights.py:418-437), through the C ABI.

Covers the 70B-class layer shapes whole and as the column slices of a 2/4/8-way
tensor-parallel split, the M = 16 / 64 verify rows at those shapes, the
stream-K kernel's plans and edge shapes, and the cluster kernel's split-K
workspace fix-up (kc > 1), each called twice on one workspace so that the
tickets are shown to re-arm.  Large shapes are compared on sampled column
ranges (the oracle is exact but sequential)."""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import _lib, synthetic

pytestmark = pytest.mark.gpu

# Per-operator tolerance of anvil-q1-fp/design/SPEC.md:311-317: cosine >= 0.9999 and
# max|y - ref| / max(1, max|ref|) <= 0.002.  The kernels differ from FP32Model.linear
# by accumulation order (split-K, fp32 partial sums) and the final fp16 rounding.
TOL_ERR, TOL_COS = 2e-3, 0.9999
SHAPES_70B = [(8192, 8192), (8192, 28672), (28672, 8192)]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def device_layer(layer, dev):
    return (T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev),
            None if layer.bias is None else T(layer.bias, dev))


def sample_ranges(N, width=512):
    width = min(width, N)
    mid = (N // 2) // 8 * 8
    return sorted({(0, width), (mid, min(N, mid + width)), (N - width, N)})


def check_sampled(y, x, layer, what, ranges=None):
    """y [M, N] against the oracle on sampled column ranges."""
    y = np.atleast_2d(y)
    N = layer.qweight.shape[1] * 8
    for a, b in ranges or sample_ranges(N):
        ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                               layer.bias_bits, layer.group, threads=oracle.max_threads(), n_range=(a, b))
        err, cos = oracle.normalized_error(y[:, a:b], ref[:, a:b])
        assert err <= TOL_ERR and cos >= TOL_COS, (what, (a, b), err, cos)


def slice_layer(layer, rank, world):
    """Rank r's column slice [r N/W, (r+1) N/W) of an AWQ layer (anvilq_b200.tp.shard_awq on numpy)."""
    W8 = layer.qweight.shape[1]
    w0, w1 = rank * W8 // world, (rank + 1) * W8 // world
    b = None if layer.bias is None else layer.bias[8 * w0:8 * w1]
    return synthetic.AwqLayer(np.ascontiguousarray(layer.qweight[:, w0:w1]),
                              np.ascontiguousarray(layer.qzeros[:, w0:w1]),
                              np.ascontiguousarray(layer.scales[:, 8 * w0:8 * w1]), b, layer.group)


def test_default_plans(dev):
    from anvilq_b200 import ops
    for K, N in [(896, 4864), (4864, 896), (4096, 4096), (4096, 11008), (4096, 22016)]:
        assert ops.gemv_plan(K, N)["kernel"] == _lib.GEMV_KERNEL_CLUSTER, (K, N)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    for K, N in [(11008, 4096), (8192, 3584), (28672, 1024)] + SHAPES_70B:
        plan = ops.gemv_plan(K, N)
        assert plan["kernel"] == _lib.GEMV_KERNEL_STREAM, (K, N, plan)
        assert plan["ctas"] == max(nsm, -(-N // 256)) and plan["stages"] == 2, plan
    for kernel in (_lib.GEMV_KERNEL_CLUSTER, _lib.GEMV_KERNEL_STREAM):   # either kernel on demand
        assert ops.gemv_plan(4096, 11008, kernel=kernel)["kernel"] == kernel


@pytest.mark.parametrize("K,N", SHAPES_70B)
def test_70b_shapes_m1(dev, K, N):
    """The whole 70B-class layer at M = 1 (default plan), twice on one workspace."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(1, K, N, 128, seed=K + N)
    w = device_layer(layer, dev)
    y1 = ops.gemm(T(x, dev), *w, 128)
    y2 = ops.gemm(T(x, dev), *w, 128)
    ops.raise_device_errors(dev)
    assert torch.equal(y1, y2)
    check_sampled(y1.float().cpu().numpy(), x, layer, (K, N))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("K,N", SHAPES_70B)
def test_70b_column_slices_m1(dev, K, N, world):
    """Each rank's N/W column slice of a 70B-class layer (the tensor-parallel split)."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(1, K, N, 128, seed=3 * K + N)
    for rank in (0, world - 1):
        part = slice_layer(layer, rank, world)
        y = ops.gemm(T(x, dev), *device_layer(part, dev), 128)
        ops.raise_device_errors(dev)
        check_sampled(y.float().cpu().numpy(), x, part, (K, N, world, rank))


@pytest.mark.parametrize("M", [16, 64])
@pytest.mark.parametrize("K,N", SHAPES_70B)
def test_70b_shapes_verify_rows(dev, K, N, M):
    """M = 16 / 64 token rows at the 70B-class shapes (tensor-core verify GEMM)."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(M, K, N, 128, seed=K + N + M)
    y = ops.gemm(T(x, dev), *device_layer(layer, dev), 128)
    ops.raise_device_errors(dev)
    check_sampled(y.float().cpu().numpy(), x, layer, (K, N, M), ranges=sample_ranges(N, 256))


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("M", [16, 64])
def test_70b_down_slice_verify_rows(dev, world, M):
    """A rank's column slice of the 28672 x 8192 projection at M = 16 / 64."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(M, 28672, 8192, 128, seed=world + M)
    part = slice_layer(layer, world - 1, world)
    y = ops.gemm(T(x, dev), *device_layer(part, dev), 128)
    ops.raise_device_errors(dev)
    check_sampled(y.float().cpu().numpy(), x, part, (world, M),
                  ranges=sample_ranges(part.qweight.shape[1] * 8, 256))


STREAM_VARIANTS = [(8, 3), (8, 2), (8, 4), (16, 2), (16, 3), (4, 4)]


def stream_plan(warps, stages, ctas):
    return dict(kernel=_lib.GEMV_KERNEL_STREAM, band_cols=256, cluster=1, kc=1, warps=warps, stages=stages,
                ctas=ctas)


@pytest.mark.parametrize("warps,stages", STREAM_VARIANTS)
def test_stream_plan_variants(dev, warps, stages):
    """Every stream-K variant and CTA count on 4096 x 11008, whole output against the oracle."""
    from anvilq_b200 import ops
    K, N = 4096, 11008
    x, layer = synthetic.gemv_case(1, K, N, 128, seed=warps * 10 + stages)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, None, 128,
                           threads=oracle.max_threads())
    w = device_layer(layer, dev)
    bands = -(-N // 256)
    for ctas in (bands, 148, 296, 1000):
        y1 = ops.gemv_planned(T(x, dev), *w, 128, plan=stream_plan(warps, stages, ctas))
        y2 = ops.gemv_planned(T(x, dev), *w, 128, plan=stream_plan(warps, stages, ctas))
        ops.raise_device_errors(dev)
        assert torch.equal(y1, y2), ctas
        err, cos = oracle.normalized_error(y1.float().cpu().numpy()[None], ref)
        assert err <= TOL_ERR and cos >= TOL_COS, (warps, stages, ctas, err, cos)


@pytest.mark.parametrize("K,N,bias", [(256, 96, True), (1024, 4128, True), (4096, 288, False), (128, 8192, False),
                                      (2048, 2080, True)])
def test_stream_edge_shapes(dev, K, N, bias):
    """Partial last bands (N not a multiple of 256), one-group K, bias, many CTAs per band."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(1, K, N, 128, seed=K + N, bias=bias)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits,
                           128, threads=oracle.max_threads())
    w = device_layer(layer, dev)
    bands, cpb = -(-N // 256), K // 32
    for ctas in sorted({bands, min(bands * cpb, 2 * bands), bands * cpb}):
        y = ops.gemv_planned(T(x, dev), *w, 128, plan=stream_plan(8, 3, ctas))
        ops.raise_device_errors(dev)
        err, cos = oracle.normalized_error(y.float().cpu().numpy()[None], ref)
        assert err <= TOL_ERR and cos >= TOL_COS, (K, N, ctas, err, cos)


def test_stream_invalid_scale_fails_operation(dev):
    from anvilq_b200 import ops, AnvilqError
    x, layer = synthetic.gemv_case(1, 4096, 4096, 128, seed=5)
    for bad, where in ((0x7C00, (3, 100)), (0xBC00, (31, 4095)), (0x7E00, (0, 0))):
        sc = layer.scales_bits.copy()
        sc[where] = bad
        ops.gemv_planned(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(sc.view(np.float16), dev),
                         None, 128, plan=stream_plan(8, 3, 296))
        with pytest.raises(AnvilqError):
            ops.raise_device_errors(dev)


def test_stream_plan_rejections(dev):
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(1, 1024, 1024, 128, seed=9)
    w = device_layer(layer, dev)
    bands, cpb = 4, 1024 // 32
    for plan in (stream_plan(5, 3, 16), stream_plan(8, 7, 16), dict(stream_plan(8, 3, 16), band_cols=512)):
        with pytest.raises(_lib.AnvilqError):
            ops.gemv_planned(T(x, dev), *w, 128, plan=plan)
    # more CTAs than chunks, or a CTA range longer than a band
    for ctas in (bands * cpb + 1, bands - 1, 0):
        with pytest.raises(_lib.AnvilqError):
            ops.gemv_planned(T(x, dev), *w, 128, plan=stream_plan(8, 3, ctas))


def cluster_plan(band_cols, cluster, kc, stages=4):
    return dict(kernel=_lib.GEMV_KERNEL_CLUSTER, band_cols=band_cols, cluster=cluster, kc=kc, warps=4,
                stages=stages, ctas=0)


@pytest.mark.parametrize("K,N", [(11008, 4096), (8192, 1024), (4864, 896)])
@pytest.mark.parametrize("band_cols,cluster,kc,stages", [(512, 8, 2, 4), (512, 8, 3, 3), (256, 4, 3, 4),
                                                          (128, 16, 2, 4), (512, 1, 8, 3)])
def test_cluster_split_k_fixup(dev, K, N, band_cols, cluster, kc, stages):
    """The cluster kernel's workspace fix-up (kc > 1 clusters per band, the last
    arriving cluster adds the partials in cluster order), forced through an
    explicit plan, twice on one workspace (tickets re-armed), whole output
    against the oracle."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(1, K, N, 128, seed=K + kc)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, None, 128,
                           threads=oracle.max_threads())
    w = device_layer(layer, dev)
    plan = cluster_plan(band_cols, cluster, kc, stages)
    y1 = ops.gemv_planned(T(x, dev), *w, 128, plan=plan)
    y2 = ops.gemv_planned(T(x, dev), *w, 128, plan=plan)
    ops.raise_device_errors(dev)
    assert torch.equal(y1, y2)
    err, cos = oracle.normalized_error(y1.float().cpu().numpy()[None], ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (K, N, plan, err, cos)


def test_cluster_plan_rejections(dev):
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(1, 1024, 1024, 128, seed=9)
    w = device_layer(layer, dev)
    for plan in (cluster_plan(384, 4, 1), cluster_plan(512, 3, 1), cluster_plan(512, 4, 9), cluster_plan(512, 32, 1),
                 dict(cluster_plan(512, 4, 1), warps=8), cluster_plan(512, 4, 1, stages=5)):
        with pytest.raises(_lib.AnvilqError):
            ops.gemv_planned(T(x, dev), *w, 128, plan=plan)


def test_default_and_planned_agree(dev):
    """anvilq_w4a16_gemm at M = 1 is the planned call under anvilq_w4a16_gemv_plan's plan."""
    from anvilq_b200 import ops
    for K, N in ((896, 4864), (4096, 11008)):
        x, layer = synthetic.gemv_case(1, K, N, 128, seed=1)
        w = device_layer(layer, dev)
        y = ops.gemm(T(x, dev), *w, 128)
        yp = ops.gemv_planned(T(x, dev), *w, 128, plan=ops.gemv_plan(K, N))
        ops.raise_device_errors(dev)
        assert torch.equal(y.view(-1), yp), (K, N)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_chain_plans_70b_slices(dev, world):
    """ops.chain_plans for one rank's slices of the 70B-class layer: one stream-K
    CTA shape for the whole chain (16 warps while a slice holds >= 40 MiB of int4),
    each slice correct under its plan, twice on one workspace."""
    from anvilq_b200 import ops
    shapes = [(K, N // world) for K, N in SHAPES_70B]
    plans = ops.chain_plans(shapes)
    assert all(p["kernel"] == _lib.GEMV_KERNEL_STREAM for p in plans), plans
    assert {p["warps"] for p in plans} == {16 if world <= 2 else 8}, plans
    for (K, N), plan in zip(SHAPES_70B, plans):
        x, layer = synthetic.gemv_case(1, K, N, 128, seed=5 * K + N + world)
        part = slice_layer(layer, 0, world)
        w = device_layer(part, dev)
        y1 = ops.gemv_planned(T(x, dev), *w, 128, plan=plan)
        y2 = ops.gemv_planned(T(x, dev), *w, 128, plan=plan)
        ops.raise_device_errors(dev)
        assert torch.equal(y1, y2)
        check_sampled(y1.float().cpu().numpy(), x, part, (K, N, world, plan))


def test_chain_plans_fallback(dev):
    """Groups of 16 rows fit the cluster kernel but not the stream-K kernel's
    32-row chunks: the chain keeps each projection's per-shape plan."""
    from anvilq_b200 import ops
    shapes = [(4096, 4096), (8192, 8192)]
    plans = ops.chain_plans(shapes, group=16)
    assert plans == [ops.gemv_plan(K, N, 16) for K, N in shapes]
    assert all(p["kernel"] == _lib.GEMV_KERNEL_CLUSTER for p in plans), plans
