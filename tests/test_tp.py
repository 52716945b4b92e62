"""Tensor-parallel N-split host logic on CPU ranks (gloo, world size 2 and 4).

Each rank computes its column slice with the oracle's C restatement of
FP32Model.linear (anvil-q1/tests/official_weights.py:418-437) standing in for
the GPU kernel, and the all-gather must reassemble exactly the single-rank
result: the split has no cross-rank partial sums, so equality is bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from anvilq_b200 import synthetic, tp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_compute(x, qweight, qzeros, scales, bias, group):
    y = oracle.gemv_fp32(x.numpy().astype(np.float32), qweight.numpy(), qzeros.numpy(),
                         scales.numpy().view(np.uint16), None if bias is None else bias.numpy().view(np.uint16),
                         group)
    return torch.from_numpy(y)


def _rank_main(rank, world, port, M, K, N, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, layer = synthetic.gemv_case(M, K, N, 128, 23, bias=True)
        lin = tp.TPLinear(torch.from_numpy(layer.qweight), torch.from_numpy(layer.qzeros),
                          torch.from_numpy(layer.scales), torch.from_numpy(layer.bias), 128,
                          compute=_oracle_compute)
        y = lin(torch.from_numpy(x))
        if rank == 0:
            np.save(out_path, y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_split_gathers_the_full_projection(tmp_path, world):
    M, K, N = 3, 256, 512
    out = tmp_path / "y.npy"
    mp.spawn(_rank_main, args=(world, _free_port(), M, K, N, str(out)), nprocs=world, join=True)
    x, layer = synthetic.gemv_case(M, K, N, 128, 23, bias=True)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits, layer.bias_bits,
                           128)
    assert np.array_equal(np.load(out), ref)


def test_column_ranges():
    assert tp.column_range(4096, 0, 8) == (0, 512)
    assert tp.column_range(4096, 7, 8) == (3584, 4096)
    with pytest.raises(ValueError):
        tp.column_range(4100, 0, 8)
    qw = torch.arange(8 * 16, dtype=torch.int32).view(8, 16)
    qz = torch.arange(2 * 16, dtype=torch.int32).view(2, 16)
    sc = torch.zeros(2, 128, dtype=torch.float16)
    parts = [tp.shard_awq(qw, qz, sc, None, r, 4) for r in range(4)]
    assert torch.equal(torch.cat([p[0] for p in parts], 1), qw)
    assert all(p[2].shape == (2, 32) for p in parts)


def _skip_rank_main(rank, world, port, skipper, out_dir):
    """Every rank builds the split; rank `skipper` never enters the all-gather
    (it stays alive past the others' process-group timeout)."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    x, layer = synthetic.gemv_case(1, 256, 768, 128, 23)   # 768 columns split over 2 or 3 ranks
    lin = tp.TPLinear(torch.from_numpy(layer.qweight), torch.from_numpy(layer.qzeros),
                      torch.from_numpy(layer.scales), None, 128, compute=_oracle_compute)
    if rank == skipper:
        time.sleep(9)
        outcome = "skipped"
    else:
        t0 = time.monotonic()
        try:
            lin(torch.from_numpy(x))
            outcome = "returned"
        except RuntimeError:
            outcome = f"raised {time.monotonic() - t0:.2f}"
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)   # the group is broken by design; leave without a collective teardown


@pytest.mark.parametrize("world", [2, 3])
def test_rank_that_skips_the_gather_fails_the_others_on_timeout(tmp_path, world):
    """Failure detection on the host: a rank that never joins the column
    all-gather makes every other rank's call raise within the process-group
    timeout -- no rank returns a partial row."""
    mp.spawn(_skip_rank_main, args=(world, _free_port(), world - 1, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        outcome = (tmp_path / f"rank{r}.txt").read_text()
        if r == world - 1:
            assert outcome == "skipped"
        else:
            assert outcome.startswith("raised"), outcome
            assert float(outcome.split()[1]) < 8.0
