"""GPU parity of the INT8 KV cache (Anvil-Q4 per-head encoding with FP32 escape)
and of decode attention over it.

The encoder is bit-exact against the oracle, itself pinned to the reference's
rational model (anvil-q4/tests/cache_reference.py:54-83, tests/golden/kv_int8.npz).
Attention over the INT8 cache is compared with the fp64 attention of
fp64_reference.py:164-170 applied to the decoded fp32 K/V, at the per-operator
tolerance (anvil-q1-fp/design/SPEC.md:311-317)."""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import synthetic

pytestmark = pytest.mark.gpu
TOL_ERR, TOL_COS = 2e-3, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _encode_gpu(dev, src, Tmax, start=None):
    from anvilq_b200 import ops
    B, Tn, H, D = src.shape
    codes = torch.full((B, Tmax, H, D), 77, dtype=torch.int8, device=dev)
    meta = torch.full((B, H, Tmax), 0x1234, dtype=torch.int32, device=dev)
    esc = torch.full((B, Tmax, H, D), 3.0, dtype=torch.float32, device=dev)
    st = None if start is None else T(np.asarray(start, np.int32), dev)
    ops.kv_int8_store(T(src, dev), codes, meta, esc, start=st)
    ops.raise_device_errors(dev)
    return codes.cpu().numpy(), meta.cpu().numpy().view(np.uint32), esc.cpu().numpy().view(np.uint32)


def test_store_reference_fixture_heads(dev, golden_dir):
    g = np.load(golden_dir / "kv_int8.npz")
    for i in range(int(g["count"])):
        h = g[f"h{i}_in"]
        codes, meta, esc = _encode_gpu(dev, h.view(np.float32)[None, None, None, :], 1)
        assert int(meta[0, 0, 0]) == int(g[f"h{i}_scale"]), i
        assert np.array_equal(codes[0, 0, 0].view(np.uint8), g[f"h{i}_codes"]), i
        expect = g[f"h{i}_recon"] if int(g[f"h{i}_scale"]) == oracle.KV_ESCAPE_MARKER else np.zeros_like(h)
        assert np.array_equal(esc[0, 0, 0], expect), i


@pytest.mark.parametrize("half", [True, False])
def test_store_matches_oracle(dev, half):
    rng = np.random.default_rng(5 + half)
    B, Tn, H, D, Tmax = 2, 37, 8, 128, 96
    x = (rng.standard_normal((B, Tn, H, D)) * 10.0 ** rng.integers(-3, 3, size=(B, Tn, H, 1))).astype(np.float32)
    x[0, 3, 2, 7] = -0.0
    x[1, 5, 0, 0] = np.inf
    x[1, 9, 4, 100] = np.nan
    x[0, 11, 1] = 1e-44                         # scale underflows: escape
    src = x.astype(np.float16) if half else x
    start = [5, 59]
    codes, meta, esc = _encode_gpu(dev, src, Tmax, start)
    sc, oc, _, oe = oracle.kv_int8_encode(src.astype(np.float32).view(np.uint32))
    for b in range(B):
        rows = slice(start[b], start[b] + Tn)
        assert np.array_equal(codes[b, rows], oc[b]), b
        assert np.array_equal(meta[b, :, rows], sc[b].T), b
        assert np.array_equal(esc[b, rows], oe[b]), b
    assert (meta == oracle.KV_ESCAPE_MARKER).sum() >= 3 if not half else True


def _attention_case(dev, B, Hq, Hkv, D, Tmax, seqlens, seed, specials=False):
    from anvilq_b200 import ops
    q, k, v = synthetic.kv_case(B, Hq, Hkv, D, Tmax, seed=seed)
    if specials:
        k[0, 1, 0, 3] = -0.0                     # escaped rows with finite values
        v[0, 2, 1, 0] = -0.0
        k[0, 7, 0] = 6e-8                        # fp16's smallest values: an ordinary row with a tiny scale
    kc = torch.zeros((B, Tmax, Hkv, D), dtype=torch.int8, device=dev)
    vc = torch.zeros_like(kc)
    km = torch.zeros((B, Hkv, Tmax), dtype=torch.int32, device=dev)
    vm = torch.zeros_like(km)
    ke = torch.zeros((B, Tmax, Hkv, D), dtype=torch.float32, device=dev)
    ve = torch.zeros_like(ke)
    ops.kv_int8_store(T(k, dev), kc, km, ke)
    ops.kv_int8_store(T(v, dev), vc, vm, ve)
    y = ops.gqa_decode_int8(T(q, dev), kc, km, vc, vm, T(np.asarray(seqlens, np.int32), dev), ke, ve)
    y2 = ops.gqa_decode_int8(T(q, dev), kc, km, vc, vm, T(np.asarray(seqlens, np.int32), dev), ke, ve)
    ops.raise_device_errors(dev)
    assert torch.equal(y, y2), "not run-to-run deterministic"
    # metadata [B][Hkv][Tmax] -> per-row scales [B][Tmax][Hkv], as the codes are laid out
    rows = lambda m: m.cpu().numpy().view(np.uint32).transpose(0, 2, 1)
    kd = oracle.kv_int8_decode(rows(km), kc.cpu().numpy(), ke.cpu().numpy().view(np.uint32))
    vd = oracle.kv_int8_decode(rows(vm), vc.cpu().numpy(), ve.cpu().numpy().view(np.uint32))
    ref = oracle.decode_attention_f64(q.astype(np.float64), kd.astype(np.float64), vd.astype(np.float64), seqlens)
    y = y.float().cpu().numpy()
    for b in range(B):
        err, cos = oracle.normalized_error(y[b], ref[b])
        assert err <= TOL_ERR and cos >= TOL_COS, (b, seqlens[b], err, cos)
    return km, vm


@pytest.mark.parametrize("B,Hq,Hkv,D,Tmax,seqlens", [
    (2, 32, 8, 128, 4096, [4096, 1000]),       # 32/8 heads of 128, clusters of 2
    (1, 14, 2, 64, 1088, [1050]),              # 0.5B heads, clusters of 8
    (1, 14, 2, 64, 8192, [8000]),              # several clusters per pair (global merge)
    (3, 8, 2, 128, 512, [1, 17, 512]),         # ragged, partial tiles
])
def test_attention_int8_matches_reference(dev, B, Hq, Hkv, D, Tmax, seqlens):
    _attention_case(dev, B, Hq, Hkv, D, Tmax, seqlens, seed=Tmax + B)


def test_attention_int8_escaped_rows(dev):
    km, vm = _attention_case(dev, 1, 8, 2, 128, 256, [200], seed=3, specials=True)
    marker = np.int32(np.uint32(oracle.KV_ESCAPE_MARKER).view(np.int32))
    assert int((km == int(marker)).sum()) == 1 and int((vm == int(marker)).sum()) == 1


def test_attention_int8_escape_without_payload_flags_error(dev):
    from anvilq_b200 import ops, AnvilqError
    q, k, v = synthetic.kv_case(1, 8, 2, 64, 64, seed=9)
    k[0, 3, 1, 0] = -0.0
    kc = torch.zeros((1, 64, 2, 64), dtype=torch.int8, device=dev)
    vc = torch.zeros_like(kc)
    km = torch.zeros((1, 2, 64), dtype=torch.int32, device=dev)
    vm = torch.zeros_like(km)
    ke = torch.zeros((1, 64, 2, 64), dtype=torch.float32, device=dev)
    ops.kv_int8_store(T(k, dev), kc, km, ke)
    ops.kv_int8_store(T(v, dev), vc, vm)
    ops.raise_device_errors(dev)
    ops.gqa_decode_int8(T(q, dev), kc, km, vc, vm, T(np.array([64], np.int32), dev))   # no escape buffers
    with pytest.raises(AnvilqError):
        ops.raise_device_errors(dev)


def test_golden_api_encode_head_matches_reference(dev, golden_dir):
    """golden_api.encode_head (the reference's signature, GPU encoder) returns the
    reference's own (scale, codes, reconstructed) for every fixture head."""
    from anvilq_b200 import golden_api
    g = np.load(golden_dir / "kv_int8.npz")
    for i in range(int(g["count"])):
        scale, codes, recon = golden_api.encode_head([int(b) for b in g[f"h{i}_in"]])
        assert scale == int(g[f"h{i}_scale"]), i
        assert codes == [int(c) for c in g[f"h{i}_codes"]], i
        assert recon == [int(r) for r in g[f"h{i}_recon"]], i
