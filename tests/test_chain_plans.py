"""Host logic of the rank-chain plans and of the deferred fused call's arguments
(no GPU: the library's per-shape plan query is replaced by a fake)."""
import types

import pytest
import torch

from anvilq_b200 import _lib, ops, tp


def _fake_stream_plans(monkeypatch, reject=()):
    """ops.gemv_plan answering like the library: the stream-K kernel's plan
    (16 warps from 8192 columns, 8 below; 148 CTAs) or ESHAPE for shapes in `reject`;
    without `kernel`, a cluster plan for rejected shapes."""
    calls = []

    def fake(K, N, group=128, kernel=None):
        calls.append((K, N, group, kernel))
        if (K, N) in reject:
            if kernel == _lib.GEMV_KERNEL_STREAM:
                raise _lib.AnvilqError("shape not supported")
            return dict(kernel=_lib.GEMV_KERNEL_CLUSTER, band_cols=128, cluster=16, kc=1, warps=4, stages=4, ctas=128)
        return dict(kernel=_lib.GEMV_KERNEL_STREAM, band_cols=256, cluster=1, kc=1,
                    warps=16 if N >= 8192 else 8, stages=2, ctas=148)

    monkeypatch.setattr(ops, "gemv_plan", fake)
    return calls


@pytest.mark.parametrize("world,warps", [(1, 16), (2, 16), (4, 8), (8, 8)])
def test_chain_plans_one_cta_shape(monkeypatch, world, warps):
    """Every slice of the 70B-class chain gets the same stream-K CTA shape: 16 warps while
    the largest slice holds at least 40 MiB of int4 (W = 1, 2), 8 below (W = 4, 8)."""
    _fake_stream_plans(monkeypatch)
    shapes = [(8192, 8192 // world), (8192, 28672 // world), (28672, 8192 // world)]
    plans = ops.chain_plans(shapes)
    assert len(plans) == 3
    assert all(p["kernel"] == _lib.GEMV_KERNEL_STREAM and p["stages"] == 2 for p in plans)
    assert {p["warps"] for p in plans} == {warps}


def test_chain_plans_threshold(monkeypatch):
    _fake_stream_plans(monkeypatch)
    K = 8192
    n_at = ops.CHAIN_WIDE_BYTES * 2 // K          # exactly CHAIN_WIDE_BYTES of int4
    assert ops.chain_plans([(K, n_at)])[0]["warps"] == 16
    assert ops.chain_plans([(K, n_at - 256)])[0]["warps"] == 8


def test_chain_plans_fallback_keeps_per_shape_plans(monkeypatch):
    """One projection the stream-K kernel rejects: every projection keeps its own plan."""
    calls = _fake_stream_plans(monkeypatch, reject={(4096, 4104)})
    shapes = [(8192, 8192), (4096, 4104)]
    plans = ops.chain_plans(shapes, group=64)
    assert plans[0]["warps"] == 16 and plans[1]["kernel"] == _lib.GEMV_KERNEL_CLUSTER
    assert (8192, 8192, 64, None) in calls and (4096, 4104, 64, None) in calls


def test_deferred_fused_call_needs_a_plan():
    """A deferred fused call runs under an explicit stream-K plan only."""
    outs = types.SimpleNamespace(world=2, rank=0, n_full=4096)
    qw = torch.zeros((4096, 256), dtype=torch.int32)      # this rank's 2048 columns
    qz = torch.zeros((32, 256), dtype=torch.int32)
    sc = torch.zeros((32, 2048), dtype=torch.float16)
    with pytest.raises(ValueError, match="stream-K plan"):
        tp.FusedTPLinear(qw, qz, sc, None, 128, outs, 0, sharded=True, deferred=True)
    lin = tp.FusedTPLinear(qw, qz, sc, None, 128, outs, 0, sharded=True)
    assert lin.plan is None and not lin.deferred and lin.N == 4096 and lin.col_base == 0
