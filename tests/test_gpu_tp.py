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
