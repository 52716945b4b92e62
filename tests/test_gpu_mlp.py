"""GPU parity of the one-launch decode MLP (anvilq_w4a16_mlp) against the oracle
and against the two fused GEMVs it replaces (FP32Model.token's feed-forward
block, anvil-q1/tests/official_weights.py:491-503)."""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import _lib, ops, synthetic

pytestmark = pytest.mark.gpu

TOL_OP = (2e-3, 0.9999)   # per-operator tolerance, anvil-q1-fp/design/SPEC.md:311-317
SHAPES = [(896, 4864), (1024, 2816), (2048, 5632), (896, 384)]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _case(H, I, seed):
    rng = np.random.default_rng(seed)
    r = (rng.standard_normal(H) * 3).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(H)).astype(np.float16)
    gu = synthetic.awq_layer(H, 2 * I, 128, rng=rng)     # gate columns first, then up
    down = synthetic.awq_layer(I, H, 128, rng=rng)
    return r, gamma, gu, down


def _oracle_delta(r, gamma, gu, down, I):
    h = r.astype(np.float64) * gamma / np.sqrt(np.mean(r.astype(np.float64) ** 2) + 1e-6)
    h = h.astype(np.float16).astype(np.float32)
    y = oracle.gemv_fp32(h[None], gu.qweight, gu.qzeros, gu.scales_bits, None, 128,
                         threads=oracle.max_threads())[0].astype(np.float16)
    g, u = y[:I].astype(np.float64), y[I:].astype(np.float64)
    a = (g / (1 + np.exp(-g)) * u).astype(np.float16).astype(np.float32)
    return oracle.gemv_fp32(a[None], down.qweight, down.qzeros, down.scales_bits, None, 128,
                           threads=oracle.max_threads())[0]


def _run_mlp(dev, r, gamma, gu, down):
    gq, gz, gs = ops.mlp_interleave(T(gu.qweight, dev), T(gu.qzeros, dev), T(gu.scales, dev))
    rt = T(r, dev)
    ops.mlp(rt, T(gamma, dev), (gq, gz, gs), (T(down.qweight, dev), T(down.qzeros, dev), T(down.scales, dev)))
    torch.cuda.synchronize(dev)
    return rt


@pytest.mark.parametrize("H,I", SHAPES)
def test_mlp_matches_oracle(dev, H, I):
    r, gamma, gu, down = _case(H, I, H + I)
    rt = _run_mlp(dev, r, gamma, gu, down)
    ops.raise_device_errors(dev)
    delta = rt.cpu().numpy().astype(np.float64) - r
    err, cos = oracle.normalized_error(delta.astype(np.float32), _oracle_delta(r, gamma, gu, down, I))
    assert err <= TOL_OP[0] and cos >= TOL_OP[1], (H, I, err, cos)


@pytest.mark.parametrize("H,I", SHAPES[:3])
def test_mlp_matches_the_two_gemvs_and_repeats(dev, H, I):
    """Against anvilq_w4a16_gemv_fused (RMSNorm in, fp16 out) on [gate | up] and
    (SiLU-mul in, residual out) on down; two calls on one workspace give the
    same bits (the tickets re-arm)."""
    lib = _lib.load()
    r, gamma, gu, down = _case(H, I, 7 * H + I)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(max(lib.anvilq_w4a16_gemm_workspace_size(1, H, 2 * I, 128),
                         lib.anvilq_w4a16_gemm_workspace_size(1, I, H, 128)), dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    rr, gm = T(r, dev), T(gamma, dev)
    y = torch.empty(2 * I, dtype=torch.float16, device=dev)
    g = [T(a, dev) for a in (gu.qweight, gu.qzeros, gu.scales)]
    d = [T(a, dev) for a in (down.qweight, down.qzeros, down.scales)]
    assert lib.anvilq_w4a16_gemv_fused(rr.data_ptr(), 1, gm.data_ptr(), 1e-6, g[0].data_ptr(), g[1].data_ptr(),
                                       g[2].data_ptr(), None, y.data_ptr(), 0, H, 2 * I, 128, ws.data_ptr(),
                                       ws.numel(), err.data_ptr(), 0, s) == 0
    assert lib.anvilq_w4a16_gemv_fused(y.data_ptr(), 2, None, 1e-6, d[0].data_ptr(), d[1].data_ptr(),
                                       d[2].data_ptr(), None, rr.data_ptr(), 1, I, H, 128, ws.data_ptr(),
                                       ws.numel(), err.data_ptr(), 0, s) == 0
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    r1 = _run_mlp(dev, r, gamma, gu, down)
    r2 = _run_mlp(dev, r, gamma, gu, down)
    ops.raise_device_errors(dev)
    assert torch.equal(r1, r2)
    ref = rr.cpu().numpy().astype(np.float64) - r
    got = r1.cpu().numpy().astype(np.float64) - r
    # only the order of the down projection's fp32 sums differs
    assert np.abs(got - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max()), (H, I)


def test_mlp_invalid_down_scale_fails_operation(dev):
    r, gamma, gu, down = _case(896, 4864, 3)
    sc = down.scales_bits.copy()
    sc[5, 100] = 0x7C00   # +inf
    down = synthetic.AwqLayer(down.qweight, down.qzeros, sc.view(np.float16), None, 128)
    _run_mlp(dev, r, gamma, gu, down)
    with pytest.raises(_lib.AnvilqError):
        ops.raise_device_errors(dev)


def test_mlp_rejections(dev):
    lib = _lib.load()
    r = torch.zeros(896, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    p = r.data_ptr()
    # null pointers, I not a multiple of 32, unknown flags
    assert lib.anvilq_w4a16_mlp(None, p, 1e-6, p, p, p, p, p, p, 896, 4864, 128, p, 1 << 20, None, 0, s) != 0
    assert lib.anvilq_w4a16_mlp(p, p, 1e-6, p, p, p, p, p, p, 896, 4848, 128, p, 1 << 20, None, 0, s) != 0
    assert lib.anvilq_w4a16_mlp(p, p, 1e-6, p, p, p, p, p, p, 896, 4864, 128, p, 1 << 20, None, 8, s) != 0
    assert lib.anvilq_w4a16_mlp_workspace_size(896, 4864, 128) > 0


# -- the decoder with its MLP in one launch ------------------------------------
TOL_DECODE = (1e-2, 0.999)   # 24-layer integration tolerance, anvil-q1-fp/design/SPEC.md:313-314


def test_decoder_mlp_matches_reference_token(dev, golden_dir):
    """Greedy decode against FP32Model.token itself (tests/golden/decode_small.npz)."""
    from anvilq_b200 import decoder
    g = np.load(golden_dir / "decode_small.npz")
    shape = tuple(int(v) for v in g["shape"])
    w = decoder.synthetic_weights(shape, seed=29)
    d = decoder.Decoder(w, dev, max_seq=shape[-1], keep_logits=True, mlp=True)
    assert d.mlp and d.kernels_per_step() == 1 + 4 * shape[0] + 2
    tokens = [int(t) for t in g["tokens"]]
    d.reset(tokens[0])
    for pos in range(len(g["logits"])):
        d.step()
        d.stream.synchronize()
        d.check_errors()
        err, cos = oracle.normalized_error(d.logits.cpu().numpy(), g["logits"][pos])
        assert err <= TOL_DECODE[0] and cos >= TOL_DECODE[1], (pos, err, cos)
        assert int(d.token.item()) == tokens[pos + 1]


def test_decoder_mlp_qwen05b_shape_and_graph(dev):
    """The 0.5B shape against the binary16-rounding oracle, then the CUDA graph
    against eager steps."""
    from anvilq_b200 import decoder
    w = decoder.synthetic_weights(decoder.QWEN05B_SHAPE, seed=17)
    d = decoder.Decoder(w, dev, max_seq=64, keep_logits=True, mlp=True)
    o = oracle.DecodeOracle(w, act16=True)
    token = 1000
    d.reset(token)
    for pos in range(3):
        ref = o.step(token, pos)
        d.step()
        d.stream.synchronize()
        d.check_errors()
        err, cos = oracle.normalized_error(d.logits.cpu().numpy(), ref)
        assert err <= TOL_DECODE[0] and cos >= TOL_DECODE[1], (pos, err, cos)
        token = int(d.token.item())
    eager = decoder.Decoder(w, dev, max_seq=16, mlp=True).generate(7, 6)
    g = decoder.Decoder(w, dev, max_seq=16, mlp=True)
    g.reset(7)
    g.capture()
    g.reset(7)
    out = []
    for _ in range(6):
        g.step()
        g.stream.synchronize()
        out.append(int(g.token.item()))
    g.check_errors()
    assert out == eager


# -- the gate/up GEMV with the SiLU product in its epilogue --------------------
@pytest.mark.parametrize("x_mode", [0, 1])
@pytest.mark.parametrize("H,I", [(896, 4864), (4096, 11008), (896, 384)])
def test_gate_up_silu_epilogue_bit_identical(dev, H, I, x_mode):
    """ANVILQ_GEMV_Y_SILU_MUL on unit-interleaved gate/up columns against the
    stored [gate | up] output followed by the SiLU product of the down GEMV's
    prologue (anvilq_silu_mul_rows restates it): identical bits; and the down
    GEMV on those activations (HALF in) against its SILU_MUL-in form."""
    lib = _lib.load()
    rng = np.random.default_rng(H + I + x_mode)
    gu = synthetic.awq_layer(H, 2 * I, 128, rng=rng)
    down = synthetic.awq_layer(I, H, 128, rng=rng)
    s = torch.cuda.current_stream(dev).cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(max(lib.anvilq_w4a16_gemm_workspace_size(1, H, 2 * I, 128),
                         lib.anvilq_w4a16_gemm_workspace_size(1, I, H, 128)), dtype=torch.uint8, device=dev)
    if x_mode == 1:
        x = T((rng.standard_normal(H) * 3).astype(np.float32), dev)
        gamma = T((1 + 0.1 * rng.standard_normal(H)).astype(np.float16), dev)
    else:
        x = T(rng.standard_normal(H).astype(np.float16), dev)
        gamma = None
    gp = None if gamma is None else gamma.data_ptr()

    def gemv(xin, xm, w, y, ym, K, N):
        rc = lib.anvilq_w4a16_gemv_fused(xin.data_ptr(), xm, gp if xm == 1 else None, 1e-6, w[0].data_ptr(),
                                         w[1].data_ptr(), w[2].data_ptr(), None, y.data_ptr(), ym, K, N, 128,
                                         ws.data_ptr(), ws.numel(), err.data_ptr(), 0, s)
        assert rc == 0, lib.anvilq_strerror(rc)

    g_cat = [T(a, dev) for a in (gu.qweight, gu.qzeros, gu.scales)]
    g_il = ops.mlp_interleave(*g_cat)
    d = [T(a, dev) for a in (down.qweight, down.qzeros, down.scales)]
    y_cat = torch.empty(2 * I, dtype=torch.float16, device=dev)
    act_ref = torch.empty(I, dtype=torch.float16, device=dev)
    act = torch.empty(I, dtype=torch.float16, device=dev)
    gemv(x, x_mode, g_cat, y_cat, 0, H, 2 * I)
    assert lib.anvilq_silu_mul_rows(y_cat.data_ptr(), act_ref.data_ptr(), 1, I, 0, s) == 0
    gemv(x, x_mode, g_il, act, 2, H, 2 * I)
    r0 = rng.standard_normal(H).astype(np.float32)
    r_ref, r_new = T(r0, dev), T(r0, dev)
    gemv(y_cat, 2, d, r_ref, 1, I, H)
    gemv(act, 0, d, r_new, 1, I, H)
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    assert torch.equal(act, act_ref), (H, I)
    assert torch.equal(r_new, r_ref), (H, I)


def test_decoder_gate_up_epilogue_matches_two_mode_path(dev):
    """The default decoder (gate/up with the SiLU epilogue) and the SiLU-prologue
    path give identical logits, step after step."""
    from anvilq_b200 import decoder
    w = decoder.synthetic_weights(decoder.QWEN05B_SHAPE, seed=41)
    a = decoder.Decoder(w, dev, max_seq=32, keep_logits=True)
    b = decoder.Decoder(w, dev, max_seq=32, keep_logits=True, gu_act=False)
    assert a.gu_act and not b.gu_act
    a.reset(11)
    b.reset(11)
    for _ in range(3):
        a.step()
        b.step()
        a.stream.synchronize()
        b.stream.synchronize()
        a.check_errors()
        b.check_errors()
        assert torch.equal(a.logits, b.logits)
        assert int(a.token.item()) == int(b.token.item())
