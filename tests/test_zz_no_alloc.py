"""The no-allocation attention entry point against the workspace one, through the C ABI.

anvilq_gqa_decode_noalloc serves callers that cannot give the library device
memory (their allocator owns HBM, their binding only forwards the tensors it
was given, or their loop must not pay cudaMalloc's implicit synchronisation).
It keeps its split-KV scratch in a fixed array inside the library, so this test
checks two consecutive calls -- the second one finding the first call's
leftovers in that array -- against anvilq_gqa_decode with a fresh workspace.
This file is collected last so that a failure here leaves every other test run.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import _lib, synthetic

pytestmark = pytest.mark.gpu

# the attention tests' tolerance (anvil-q1-fp/design/SPEC.md:311-317)
TOL_ERR, TOL_COS = 2e-3, 0.9999


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _case(dev, B, Hq, Hkv, D, Tmax, seed):
    q, k, v = synthetic.kv_case(B, Hq, Hkv, D, Tmax, seed=seed)
    rng = np.random.default_rng(seed)
    seqlens = np.array([Tmax] + list(rng.integers(1, Tmax + 1, size=B - 1)), np.int32)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return to(q), to(k), to(v), to(seqlens)


def test_noalloc_matches_workspace_entry_point(dev):
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    cases = [(4, 32, 8, 128, 4096, 17), (3, 14, 2, 64, 1024, 43)]   # two calls in a row
    for B, Hq, Hkv, D, Tmax, seed in cases:
        q, k, v, seqlens = _case(dev, B, Hq, Hkv, D, Tmax, seed)
        scale = 1.0 / np.sqrt(D)

        need = lib.anvilq_gqa_decode_workspace_size(B, Hq, Hkv, D, Tmax)
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        err_ref = torch.zeros(1, dtype=torch.int32, device=dev)
        out_ref = torch.empty_like(q)
        rc = lib.anvilq_gqa_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(seqlens), _ptr(out_ref), B, Hq, Hkv, D,
                                   Tmax, scale, _ptr(ws), need, _ptr(err_ref), ctypes.c_void_p(stream))
        assert rc == 0, lib.anvilq_strerror(rc)

        err = torch.zeros(1, dtype=torch.int32, device=dev)
        out = torch.full_like(q, float("nan"))
        rc = lib.anvilq_gqa_decode_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(seqlens), _ptr(out), B, Hq, Hkv, D,
                                           Tmax, scale, _ptr(err), ctypes.c_void_p(stream))
        assert rc == 0, lib.anvilq_strerror(rc)
        torch.cuda.synchronize(dev)
        assert int(err_ref.item()) == 0 and int(err.item()) == 0

        e, cos = oracle.normalized_error(out.float().cpu().numpy(), out_ref.float().cpu().numpy())
        assert e <= TOL_ERR and cos >= TOL_COS, ((B, Hq, Hkv, D, Tmax), e, cos)


def test_noalloc_rejects_bad_arguments_before_launch(dev):
    lib = _lib.load()
    q, k, v, seqlens = _case(dev, 1, 8, 2, 64, 64, 5)
    out = torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    # head_dim 96 is outside the supported sizes
    assert lib.anvilq_gqa_decode_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(seqlens), _ptr(out), 1, 8, 2, 96, 64,
                                         0.0, _ptr(err), s) == -5
    assert lib.anvilq_gqa_decode_noalloc(None, _ptr(k), _ptr(v), _ptr(seqlens), _ptr(out), 1, 8, 2, 64, 64,
                                         0.0, _ptr(err), s) == -1
    assert b"fixed no-allocation" in lib.anvilq_strerror(-6)


def test_noalloc_scratch_holds_every_plan_on_this_device(dev):
    """ANVILQ_ENOSCRATCH guards the fixed 4 MiB array.  The split plan's scratch
    is bounded by the resident CTA slots (pairs x splits <= 2 x SMs), so on a
    148-SM B200 no valid shape reaches the limit: every extreme of the
    supported range (largest batch x kv heads, largest group, both head dims,
    long and short contexts) needs at most a few hundred KiB, and the
    no-allocation entry point accepts it."""
    lib = _lib.load()
    limit = 4 << 20
    worst = 0
    for D in (64, 128):
        for B, Hkv, group in ((1, 1, 8), (1, 8, 8), (2, 4, 8), (16, 8, 4), (2048, 8, 1), (4096, 4, 8)):
            for Tmax in (16, 1024, 32768, 1 << 20):
                need = lib.anvilq_gqa_decode_workspace_size(B, Hkv * group, Hkv, D, Tmax)
                assert 0 < need <= limit, (B, Hkv, group, D, Tmax, need)
                worst = max(worst, need)
    assert worst <= limit // 4
    # the largest-scratch case runs through the no-allocation entry point
    q, k, v, seqlens = _case(dev, 1, 64, 8, 128, 32768, 7)
    out = torch.full_like(q, float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    assert lib.anvilq_gqa_decode_noalloc(_ptr(q), _ptr(k), _ptr(v), _ptr(seqlens), _ptr(out), 1, 64, 8, 128,
                                         32768, 0.0, _ptr(err), s) == 0
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0 and not torch.isnan(out).any()
