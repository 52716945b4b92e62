"""GPU parity of the GQA decode attention kernel against the oracle, through the C ABI."""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import synthetic

pytestmark = pytest.mark.gpu

# Per-operator tolerance of anvil-q1-fp/design/SPEC.md:311-317 (cosine >= 0.9999,
# max|y - ref| / max(1, max|ref|) <= 0.002).  The kernel computes scores and the
# softmax in fp32 and rounds probabilities to fp16 for the P.V tensor-core product.
TOL_ERR, TOL_COS = 2e-3, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run(dev, q, k, v, seqlens):
    from anvilq_b200 import ops
    out = ops.gqa_decode(T(q, dev), T(k, dev), T(v, dev), T(np.asarray(seqlens, np.int32), dev))
    ops.raise_device_errors(dev)
    return out.float().cpu().numpy()


def check(y, ref, what):
    err, cos = oracle.normalized_error(y, ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (what, err, cos)


def test_reference_fixtures(dev, golden_dir):
    """fp64_reference.attention outputs on the fixture cases (head_dim 64/128)."""
    g = np.load(golden_dir / "attention.npz")
    n = 0
    for key in [str(s) for s in g["case_names"]]:
        q, k, v, ref = g[key + "_q"], g[key + "_k"], g[key + "_v"], g[key + "_y"]
        if q.shape[1] not in (64, 128):
            continue
        y = run(dev, q[None], k[None], v[None], [k.shape[0]])
        check(y[0], ref, key)
        n += 1
    assert n >= 4


@pytest.mark.parametrize("B,Tmax", [(1, 512), (8, 512), (1, 4096), (8, 4096), (2, 32768)])
def test_config_shapes(dev, B, Tmax):
    """32 q heads / 8 kv heads, head_dim 128 (the decode-attention benchmark configuration)."""
    q, k, v = synthetic.kv_case(B, 32, 8, 128, Tmax, seed=17 + B)
    rng = np.random.default_rng(Tmax + B)
    seqlens = [Tmax] + list(rng.integers(1, Tmax + 1, size=B - 1))
    y = run(dev, q, k, v, seqlens)
    ref = oracle.decode_attention_f64(q, k, v, seqlens)
    for b in range(B):
        check(y[b], ref[b], (B, Tmax, b, seqlens[b]))


@pytest.mark.parametrize("B", [32, 64])
@pytest.mark.parametrize("Tmax", [512, 4096, 32768])
def test_config_large_batches(dev, B, Tmax):
    """Batches of 32 and 64 sequences (32 / 8 heads of 128) at every context of
    the decode-attention configuration, with ragged lengths (the first sequence
    full).  The caches are drawn on the device from a seeded generator; a sample
    of sequences (first, middle, last, and the shortest) is checked against the
    binary64 attention() restatement."""
    from anvilq_b200 import ops
    Hq, Hkv, D = 32, 8, 128
    g = torch.Generator(device=dev)
    g.manual_seed(B * 100003 + Tmax)
    k = torch.randn((B, Tmax, Hkv, D), generator=g, device=dev, dtype=torch.float16)
    v = torch.randn((B, Tmax, Hkv, D), generator=g, device=dev, dtype=torch.float16)
    q = torch.randn((B, Hq, D), generator=g, device=dev, dtype=torch.float16)
    rng = np.random.default_rng(B + Tmax)
    seqlens = np.concatenate([[Tmax], rng.integers(1, Tmax + 1, size=B - 1)]).astype(np.int32)
    sl = T(seqlens, dev)
    y1 = ops.gqa_decode(q, k, v, sl).clone()
    y2 = ops.gqa_decode(q, k, v, sl)
    ops.raise_device_errors(dev)
    assert torch.equal(y1, y2)
    y = y1.float().cpu().numpy()
    for b in sorted({0, B // 2, B - 1, int(np.argmin(seqlens))}):
        L = int(seqlens[b])
        ref = oracle.attention_f64(q[b].cpu().numpy(), k[b, :L].cpu().numpy(), v[b, :L].cpu().numpy())
        check(y[b], ref, (B, Tmax, b, L))
    del k, v
    torch.cuda.empty_cache()


def test_qwen05b_shape(dev):
    """14 q heads / 2 kv heads (group of 7), head_dim 64, context 1024."""
    q, k, v = synthetic.kv_case(3, 14, 2, 64, 1024, seed=43)
    seqlens = [1024, 1, 513]
    y = run(dev, q, k, v, seqlens)
    ref = oracle.decode_attention_f64(q, k, v, seqlens)
    for b in range(3):
        check(y[b], ref[b], seqlens[b])


@pytest.mark.parametrize("L", [1, 2, 15, 16, 17, 63, 64, 65, 127, 129, 1000])
def test_ragged_lengths(dev, L):
    q, k, v = synthetic.kv_case(1, 8, 2, 128, 1024, seed=L)
    y = run(dev, q, k, v, [L])
    ref = oracle.decode_attention_f64(q, k, v, [L])
    check(y[0], ref[0], L)


# Each shape reaches one way of merging a pair's KV splits on a 148-SM B200:
# one CTA per pair (no merge), one cluster (distributed shared memory), and
# several clusters (cluster merge, then the global merge of their partials).
@pytest.mark.parametrize("B,Hq,Hkv,D,Tmax,seqlens", [
    (40, 16, 4, 64, 256, None),                 # 160 pairs: one CTA each
    (1, 14, 2, 64, 300, [300]),                 # clusters of 2
    (1, 14, 2, 64, 1090, [1050]),               # clusters of 8 (the 0.5B decode step)
    (1, 14, 2, 64, 8192, [8192]),               # 8 clusters of 8
    (2, 14, 2, 64, 8192, [40, 8191]),           # as above, most clusters of sequence 0 empty
    (1, 8, 1, 128, 16384, [16384]),             # 16 clusters of 8, head_dim 128
    (3, 12, 3, 128, 5000, [1, 4999, 2500]),     # group of 4
])
def test_split_merge_paths(dev, B, Hq, Hkv, D, Tmax, seqlens):
    from anvilq_b200 import ops
    q, k, v = synthetic.kv_case(B, Hq, Hkv, D, Tmax, seed=Tmax + B)
    if seqlens is None:
        seqlens = list(np.random.default_rng(B).integers(1, Tmax + 1, size=B))
    args = (T(q, dev), T(k, dev), T(v, dev), T(np.asarray(seqlens, np.int32), dev))
    a = ops.gqa_decode(*args).clone()
    y = ops.gqa_decode(*args)
    ops.raise_device_errors(dev)
    assert torch.equal(a, y), "split merge is not run-to-run deterministic"
    ref = oracle.decode_attention_f64(q, k, v, seqlens)
    y = y.float().cpu().numpy()
    for b in range(B):
        check(y[b], ref[b], (B, Hq, Hkv, D, Tmax, b, seqlens[b]))


def test_fp32_loop_agreement(dev):
    """Against the FP32 sequential loop of official_weights.py:471-486 as well."""
    q, k, v = synthetic.kv_case(1, 14, 2, 64, 300, seed=89)
    y = run(dev, q, k, v, [300])
    ref32 = oracle.attention_fp32(q[0].view(np.uint16), k[0].view(np.uint16), v[0].view(np.uint16))
    check(y[0], ref32, "fp32 loop")


def test_repeat_is_deterministic(dev):
    from anvilq_b200 import ops
    q, k, v = synthetic.kv_case(4, 32, 8, 128, 4096, seed=5)
    args = (T(q, dev), T(k, dev), T(v, dev), T(np.array([4096, 3000, 17, 2048], np.int32), dev))
    a = ops.gqa_decode(*args).clone()
    b = ops.gqa_decode(*args)
    ops.raise_device_errors(dev)
    assert torch.equal(a, b)


def test_bad_seqlen_flags_error(dev):
    from anvilq_b200 import ops, AnvilqError
    q, k, v = synthetic.kv_case(2, 8, 2, 64, 64, seed=3)
    for bad in (0, 65, -1):
        ops.gqa_decode(T(q, dev), T(k, dev), T(v, dev), T(np.array([64, bad], np.int32), dev))
        with pytest.raises(AnvilqError):
            ops.raise_device_errors(dev)


def test_unsupported_shape_rejected_on_host(dev):
    from anvilq_b200 import ops
    q, k, v = synthetic.kv_case(1, 8, 2, 32, 16, seed=3)   # head_dim 32 is not a supported size
    with pytest.raises(ValueError):
        ops.gqa_decode(T(q, dev), T(k, dev), T(v, dev), T(np.array([16], np.int32), dev))


def test_programmatic_launch_matches_plain(dev):
    """anvilq_gqa_decode_ex with ANVILQ_GEMM_OVERLAP_PRIOR, right after a kernel
    that writes q and the lengths, gives the bits of the plain launch; unknown
    flags are rejected."""
    from anvilq_b200 import _lib
    lib = _lib.load()
    B, Hq, Hkv, D, Tmax = 1, 14, 2, 64, 1100
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    k = torch.randn((B, Tmax, Hkv, D), generator=g, device=dev).half()
    v = torch.randn((B, Tmax, Hkv, D), generator=g, device=dev).half()
    q_src = torch.randn((B, Hq, D), generator=g, device=dev).half()
    q = torch.zeros_like(q_src)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(lib.anvilq_gqa_decode_workspace_size(B, Hq, Hkv, D, Tmax), dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    outs = []
    for flags in (0, 1, 1):
        q.zero_()
        lens.zero_()
        out = torch.empty((B, Hq, D), dtype=torch.float16, device=dev)
        q.copy_(q_src)          # the preceding kernels write q and the length
        lens.fill_(1025)
        rc = lib.anvilq_gqa_decode_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), out.data_ptr(),
                                      B, Hq, Hkv, D, Tmax, 0.0, ws.data_ptr(), ws.numel(), err.data_ptr(), flags, s)
        assert rc == 0, lib.anvilq_strerror(rc)
        outs.append(out)
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert lib.anvilq_gqa_decode_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), q.data_ptr(),
                                    B, Hq, Hkv, D, Tmax, 0.0, ws.data_ptr(), ws.numel(), err.data_ptr(), 4, s) != 0
