"""Tensor-parallel N-split of a W4A16 AWQ projection across ranks.

Reference analog: the column interleave of the Anvil-Q2 GEMV banks
(anvil-q2/rtl/anvil_q2_gemv_lane.sv:117,187) -- every bank owns a slice of the
output columns and sees the whole activation vector.  Here rank r of W owns the
contiguous output columns [r N/W, (r+1) N/W): qweight[:, r W8/W : (r+1) W8/W]
(W8 = N/8 packed words per row), the same words of qzeros, scales[:, cols] and
bias[cols].  x is replicated; each rank computes its slice with the single-GPU
kernels, and one all-gather (NCCL on GPUs) assembles y.

The exchange is the only collective: ranks share no partial sums (the K
reduction is complete inside each rank), so results are bit-identical to the
single-GPU call on the same slice of columns.

At M = 1 the all-gather can be fused into the GEMV itself
(``FusedTPLinear``): each rank's kernel stores its slice straight into every
rank's full-width output over NVLink (CUDA IPC buffers, ``PeerOutputs``) and
the ranks exchange completion flags, so one kernel per projection replaces the
GEMV + NCCL all-gather pair.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def column_range(N: int, rank: int, world: int):
    """Output columns owned by `rank`; N / world must be a multiple of 8 (whole packed words)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside the process group")
    if N % (8 * world):
        raise ValueError(f"N={N} does not split into {world} slices of whole 8-column words")
    n = N // world
    return rank * n, (rank + 1) * n


def shard_awq(qweight, qzeros, scales, bias, rank: int, world: int):
    """The rank's column slice of one AWQ projection (views, made contiguous)."""
    W8 = qweight.shape[1]
    c0, c1 = column_range(W8 * 8, rank, world)
    w0, w1 = c0 // 8, c1 // 8
    part = (qweight[:, w0:w1].contiguous(), qzeros[:, w0:w1].contiguous(), scales[:, c0:c1].contiguous(),
            None if bias is None else bias[c0:c1].contiguous())
    return part


def gather_columns(y_local, world: int, group=None):
    """[M, N/W] on every rank -> [M, N] on every rank, columns in rank order (all-gather)."""
    M, n = y_local.shape
    stacked = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(stacked, y_local.contiguous(), group=group)
    return stacked.view(world, M, n).permute(1, 0, 2).reshape(M, world * n)


class TPLinear:
    """One projection split across the ranks of a process group.

    ``compute(x, qweight, qzeros, scales, bias, group) -> y`` is the per-rank
    kernel (``ops.gemm`` by default; tests on CPU ranks substitute the oracle).
    """

    def __init__(self, qweight, qzeros, scales, bias=None, group_size: int = 128, process_group=None,
                 compute=None):
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.N = qweight.shape[1] * 8
        self.group_size = group_size
        self.shard = shard_awq(qweight, qzeros, scales, bias, self.rank, self.world)
        if compute is None:
            from . import ops
            compute = ops.gemm
        self.compute = compute

    def local(self, x):
        """This rank's [M, N/W] slice of y = x W (+ bias)."""
        return self.compute(x, *self.shard, self.group_size)

    def __call__(self, x):
        x2 = x.unsqueeze(0) if x.dim() == 1 else x
        y = gather_columns(self.local(x2), self.world, self.pg)
        return y.view(self.N) if x.dim() == 1 else y


class PeerOutputs:
    """Full-width fp16 outputs that every rank of the group writes directly
    (peer stores over NVLink into CUDA IPC buffers), ``slots`` of them, plus the
    flag array and the call counter of the fused all-gather.  Collective: every
    rank constructs it with the same arguments, and closes it."""

    _FLAGS = 256   # bytes reserved for the 8 flags at the start of the buffer

    def __init__(self, n_full: int, slots: int = 2, device=None, process_group=None):
        from . import _lib
        self.lib = _lib.load()
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        if not 1 <= self.world <= 8:
            raise ValueError("the fused all-gather spans 1 to 8 ranks")
        self.n_full, self.slots = n_full, slots
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.slot_bytes = -(-n_full * 2 // 256) * 256
        self.buf = torch.zeros(self._FLAGS + slots * self.slot_bytes, dtype=torch.uint8, device=self.device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        handle = (ctypes.c_char * self.lib.anvilq_peer_handle_size())()
        offset = ctypes.c_size_t()
        _lib.check(self.lib.anvilq_peer_export(self.buf.data_ptr(), handle, ctypes.byref(offset)),
                   "anvilq_peer_export")
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (bytes(handle), offset.value), group=process_group)
        self._opened, ptrs = [], []
        for r, (h, off) in enumerate(everyone):
            if r == self.rank:
                ptrs.append(self.buf.data_ptr())
                continue
            base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(self.lib.anvilq_peer_import(h, off, ctypes.byref(base), ctypes.byref(ptr)),
                       "anvilq_peer_import")
            self._opened.append(base.value)
            ptrs.append(ptr.value)
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.y_ptrs = [(ctypes.c_void_p * self.world)(*[q + self._FLAGS + s * self.slot_bytes for q in ptrs])
                       for s in range(slots)]
        dist.barrier(group=process_group)   # every rank holds every buffer before anyone writes

    def wait(self, stream=None):
        """Enqueue on ``stream`` (default: the current stream) a wait until every
        rank's flag reached this rank's count of fused calls: the last deferred
        call's row is complete here after it (anvilq_peer_wait)."""
        from . import _lib, ops
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        err = ops.device_error_word(self.device)
        _lib.check(self.lib.anvilq_peer_wait(ctypes.c_void_p(self.flag_ptrs[self.rank]), self.world,
                                             self.epoch.data_ptr(), err.data_ptr(), s.cuda_stream),
                   "anvilq_peer_wait")

    def output(self, slot: int, n: int | None = None):
        """This rank's full-width output of one slot (a view, fp16 [n_full])."""
        off = self._FLAGS + slot * self.slot_bytes
        return self.buf[off:off + 2 * (n or self.n_full)].view(torch.float16)

    def close(self):
        """Collective: release the imported peer buffers (after all fused calls completed)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.pg)
        for base in self._opened:
            self.lib.anvilq_peer_close(base)
        self._opened = []


class FusedTPLinear:
    """``TPLinear`` at M = 1 with the all-gather fused into the GEMV: one kernel
    per call computes this rank's slice and stores it in every rank's output
    slot, then waits for every rank's completion flag.  Returns the full row
    (a view of ``outputs.output(slot)``); slots must alternate between calls
    (see anvilq_w4a16_gemv_allgather).

    With ``plan`` (a stream-K plan, e.g. from ``ops.chain_plans``) the slice
    runs under it (anvilq_w4a16_gemv_allgather_planned); with ``deferred`` too
    the call does not wait for the other ranks at its end: the next deferred
    call waits for them before reading x, so x may be the previous call's row
    and the exchange overlaps the next weight stream.  A deferred call's row is
    complete only after the next deferred call or ``outputs.wait()``."""

    DEFERRED = 2   # ANVILQ_GATHER_DEFERRED

    def __init__(self, qweight, qzeros, scales, bias, group_size: int, outputs: PeerOutputs, slot: int,
                 sharded: bool = False, plan: dict | None = None, deferred: bool = False):
        """Full AWQ tensors of the projection, or (``sharded``) this rank's slice already."""
        self.out = outputs
        self.slot = slot
        self.N = qweight.shape[1] * 8 * (outputs.world if sharded else 1)
        if self.N > outputs.n_full:
            raise ValueError("projection wider than the peer outputs")
        self.col_base = column_range(self.N, outputs.rank, outputs.world)[0]
        self.shard = ((qweight, qzeros, scales, bias) if sharded
                      else shard_awq(qweight, qzeros, scales, bias, outputs.rank, outputs.world))
        self.group_size = group_size
        self.K = qweight.shape[0]
        if deferred and plan is None:
            raise ValueError("a deferred fused call takes an explicit stream-K plan")
        self.plan = None if plan is None else _plan_struct(plan)
        self.deferred = deferred

    def __call__(self, x, flags: int = 0):
        from . import _lib, ops
        lib = self.out.lib
        qw, qz, sc, b = self.shard
        n = qw.shape[1] * 8
        need = (lib.anvilq_w4a16_gemm_workspace_size(1, self.K, n, self.group_size) if self.plan is None else
                lib.anvilq_w4a16_gemv_plan_workspace_size(self.K, n, self.group_size, ctypes.byref(self.plan)))
        if need == 0:
            raise ValueError(f"the plan does not fit K={self.K}, N={n}")
        ws = ops.workspace(x.device, need)
        err = ops.device_error_word(x.device)
        if self.plan is not None:
            _lib.check(lib.anvilq_w4a16_gemv_allgather_planned(
                x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), None if b is None else b.data_ptr(),
                self.K, n, self.group_size, self.out.rank, self.out.world, self.col_base, self.N,
                ctypes.cast(self.out.y_ptrs[self.slot], ctypes.c_void_p),
                ctypes.cast(self.out.flag_ptrs, ctypes.c_void_p), self.out.epoch.data_ptr(),
                ctypes.byref(self.plan), ws.data_ptr(), ws.numel(), err.data_ptr(),
                flags | (self.DEFERRED if self.deferred else 0), torch.cuda.current_stream(x.device).cuda_stream),
                "anvilq_w4a16_gemv_allgather_planned")
            return self.out.output(self.slot, self.N)
        _lib.check(lib.anvilq_w4a16_gemv_allgather(
            x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), None if b is None else b.data_ptr(),
            self.K, n, self.group_size, self.out.rank, self.out.world, self.col_base, self.N,
            ctypes.cast(self.out.y_ptrs[self.slot], ctypes.c_void_p), ctypes.cast(self.out.flag_ptrs, ctypes.c_void_p),
            self.out.epoch.data_ptr(), ws.data_ptr(), ws.numel(), err.data_ptr(), flags,
            torch.cuda.current_stream(x.device).cuda_stream), "anvilq_w4a16_gemv_allgather")
        return self.out.output(self.slot, self.N)


def _plan_struct(plan: dict):
    from . import _lib
    return _lib.GemvPlan(**plan)
