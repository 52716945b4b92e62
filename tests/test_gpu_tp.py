"""Tensor-parallel N-split on 2 GPUs over NCCL (skipped with fewer than 2 GPUs).

Each rank computes its column slice with the W4A16 kernels and one all-gather
assembles y.  The result must equal, bit for bit, single-GPU calls on the same
column slices (no cross-rank partial sums), and the reference within the
per-operator tolerance.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from anvilq_b200 import synthetic

pytestmark = pytest.mark.gpu

TOL_ERR, TOL_COS = 2e-3, 0.9999


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, M, K, N, out_path):
    import datetime
    from anvilq_b200 import ops, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, layer = synthetic.gemv_case(M, K, N, 128, 31, bias=True)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        lin = tp.TPLinear(to(layer.qweight), to(layer.qzeros), to(layer.scales), to(layer.bias), 128)
        y = lin(to(x))
        ops.raise_device_errors(dev)
        torch.cuda.synchronize(dev)
        if rank == 0:
            np.save(out_path, y.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 16])
def test_tp2_matches_single_gpu_slices(tmp_path, M):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from anvilq_b200 import ops, tp
    K, N = 4096, 11008
    out = tmp_path / "y.npy"
    mp.spawn(_rank_main, args=(2, _free_port(), M, K, N, str(out)), nprocs=2, join=True)
    y_tp = np.load(out)
    dev = torch.device("cuda", 0)
    x, layer = synthetic.gemv_case(M, K, N, 128, 31, bias=True)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    full = (to(layer.qweight), to(layer.qzeros), to(layer.scales), to(layer.bias))
    slices = [ops.gemm(to(x), *tp.shard_awq(*full, r, 2), 128) for r in range(2)]
    ops.raise_device_errors(dev)
    assert np.array_equal(y_tp, torch.cat(slices, 1).cpu().numpy())
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits,
                           128, threads=oracle.max_threads())
    err, cos = oracle.normalized_error(y_tp.astype(np.float32), ref)
    assert err <= TOL_ERR and cos >= TOL_COS


def _fused_rank_main(rank, world, port, K, N, out_path):
    import datetime
    from anvilq_b200 import ops, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, layer = synthetic.gemv_case(1, K, N, 128, 37, bias=True)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        full = (to(layer.qweight), to(layer.qzeros), to(layer.scales), to(layer.bias))
        outs = tp.PeerOutputs(N, slots=2, device=dev)
        fused = [tp.FusedTPLinear(*full, 128, outs, s) for s in (0, 1)]
        nccl = tp.TPLinear(*full, 128)
        same = []
        for i in range(5):   # alternating slots, a different x every call
            xi = to((x[0].astype(np.float32) * (1.0 + 0.25 * i)).astype(np.float16))
            y = fused[i % 2](xi).clone()
            same.append(bool(torch.equal(y, nccl(xi))))
        ops.raise_device_errors(dev)
        torch.cuda.synchronize(dev)
        outs.close()
        if rank == 0:
            np.save(out_path, np.array(same))
    finally:
        dist.destroy_process_group()


def test_tp2_fused_allgather_matches_nccl(tmp_path):
    """The GEMV with the all-gather fused into its epilogue (peer stores over
    NVLink, flag exchange) returns the same full row, bit for bit, as the
    GEMV + NCCL all-gather, call after call."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "same.npy"
    mp.spawn(_fused_rank_main, args=(2, _free_port(), 4096, 11008, str(out)), nprocs=2, join=True)
    assert np.load(out).all()


def _timeout_rank_main(rank, world, port, K, N, out_path):
    import datetime
    import time
    from anvilq_b200 import ops, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, layer = synthetic.gemv_case(1, K, N, 128, 41)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        outs = tp.PeerOutputs(N, slots=2, device=dev)
        fused = tp.FusedTPLinear(to(layer.qweight), to(layer.qzeros), to(layer.scales), None, 128, outs, 0)
        err = ops.device_error_word(dev)
        err.zero_()
        torch.cuda.synchronize(dev)
        dist.barrier()
        if rank == 0:   # rank 1 never enters the fused call
            t0 = time.monotonic()
            fused(to(x[0]))
            torch.cuda.synchronize(dev)
            dt = time.monotonic() - t0
            bits = int(err.item())
            err.zero_()
            np.save(out_path, np.array([bits, dt]))
        dist.barrier()   # both ranks, between steps, with no kernel of theirs in flight
        torch.cuda.synchronize(dev)
        outs.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("K,N", [(4096, 11008), (896, 1152)])
def test_tp2_fused_allgather_wait_expires_when_a_rank_is_missing(tmp_path, K, N):
    """The fused all-gather's flag wait is bounded: with rank 1 never entering
    the call, rank 0's kernel gives up after about a second, sets
    ANVILQ_DEV_ERR_TIMEOUT and returns, and the context stays usable (the
    ranks then meet at a barrier and release their buffers).  Both the
    stream-K kernel (7B-class slice) and the cluster kernel (decode-size
    slice) are covered.  No multicast object; plain peer stores and flags."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "timeout.npy"
    mp.spawn(_timeout_rank_main, args=(2, _free_port(), K, N, str(out)), nprocs=2, join=True)
    bits, dt = np.load(out)
    assert int(bits) & 4, bits          # ANVILQ_DEV_ERR_TIMEOUT
    assert 0.5 <= dt <= 10.0, dt


CHAIN = [(4096, 4096), (4096, 11008), (11008, 4096)]   # each output row is the next input


def _deferred_rank_main(rank, world, port, out_path):
    import datetime
    from anvilq_b200 import ops, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        layers = []
        for i, (K, N) in enumerate(CHAIN):
            _, layer = synthetic.gemv_case(1, K, N, 128, 43 + i, bias=(i == 1))
            layers.append(tuple(None if a is None else to(a)
                                for a in (layer.qweight, layer.qzeros, layer.scales, layer.bias)))
        plans = ops.chain_plans([(K, N // world) for K, N in CHAIN])
        # two sets of three output slots, alternating by step: a row is read back
        # after the step's last call, so it must survive the other ranks' next step
        outs = tp.PeerOutputs(max(N for _, N in CHAIN), slots=6, device=dev)
        fused = [[tp.FusedTPLinear(*w, 128, outs, 3 * k + i, plan=plans[i], deferred=True)
                  for i, w in enumerate(layers)] for k in range(2)]
        nccl = [tp.TPLinear(*w, 128, compute=lambda x, qw, qz, sc, b, g, pl=pl:
                            ops.gemv_planned(x, qw, qz, sc, b, g, plan=pl).view(1, -1))
                for w, pl in zip(layers, plans)]
        x0, _ = synthetic.gemv_case(1, CHAIN[0][0], CHAIN[0][1], 128, 47)
        same = []
        for step in range(4):   # every slot is reused
            x = to((x0[0].astype(np.float32) * (1.0 + 0.5 * step)).astype(np.float16))
            y, ys = x, []
            for lin in fused[step % 2]:   # deferred: each call waits for the others before reading its x
                y = lin(y)
                ys.append(y)
            outs.wait()         # the last row is complete after this
            got = [t.clone() for t in ys]
            y = x
            for i, lin in enumerate(nccl):
                y = lin(y)
                same.append(bool(torch.equal(got[i], y)))
        ops.raise_device_errors(dev)
        torch.cuda.synchronize(dev)
        outs.close()
        if rank == 0:
            np.save(out_path, np.array(same))
    finally:
        dist.destroy_process_group()


def test_tp2_deferred_chain_matches_nccl(tmp_path):
    """Three column-split projections chained through their gathered rows with
    the deferred exchange (each call raises its flag and moves on; the next call
    waits for every rank before reading x; outputs.wait() ends the chain) give
    the same rows, bit for bit, as the same plans followed by NCCL all-gathers,
    step after step on reused output slots."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "same.npy"
    mp.spawn(_deferred_rank_main, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    same = np.load(out)
    assert same.size == 12 and same.all(), same


def _deferred_timeout_rank_main(rank, world, port, out_path):
    import datetime
    import time
    from anvilq_b200 import ops, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        K, N = 4096, 11008
        x, layer = synthetic.gemv_case(1, K, N, 128, 53)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        outs = tp.PeerOutputs(N, slots=2, device=dev)
        plan = ops.chain_plans([(K, N // world)])[0]
        fused = tp.FusedTPLinear(to(layer.qweight), to(layer.qzeros), to(layer.scales), None, 128, outs, 0,
                                 plan=plan, deferred=True)
        err = ops.device_error_word(dev)
        err.zero_()
        torch.cuda.synchronize(dev)
        dist.barrier()
        if rank == 0:   # rank 1 never enters the fused call
            t0 = time.monotonic()
            fused(to(x[0]))
            torch.cuda.synchronize(dev)
            bits_call = int(err.item())
            outs.wait()
            torch.cuda.synchronize(dev)
            dt = time.monotonic() - t0
            bits = int(err.item())
            err.zero_()
            np.save(out_path, np.array([bits_call, bits, dt]))
        dist.barrier()   # both ranks, between steps, with no kernel of theirs in flight
        torch.cuda.synchronize(dev)
        outs.close()
    finally:
        dist.destroy_process_group()


def test_tp2_deferred_wait_expires_when_a_rank_is_missing(tmp_path):
    """A deferred call does not wait for the other ranks (no error with rank 1
    absent); the wait that ends the chain is bounded: it gives up after about
    a second with ANVILQ_DEV_ERR_TIMEOUT and the context stays usable."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "timeout.npy"
    mp.spawn(_deferred_timeout_rank_main, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    bits_call, bits, dt = np.load(out)
    assert int(bits_call) == 0, bits_call
    assert int(bits) & 4, bits          # ANVILQ_DEV_ERR_TIMEOUT
    assert 0.5 <= dt <= 10.0, dt
