"""GPU parity of the W4A16 AWQ kernels against the oracle, through the C ABI."""
import json

import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import synthetic

pytestmark = pytest.mark.gpu

# Per-operator tolerance of the reference's FP datapath: cosine >= 0.9999 and
# max|y - ref| / max(1, max|ref|) <= 0.002 (anvil-q1-fp/design/SPEC.md:311-317).
# The fast kernels differ from FP32Model.linear by accumulation order (split-K,
# per-slot fp32 partial sums) and one fp16 output rounding.
TOL_ERR, TOL_COS = 2e-3, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_dequant_bit_exact_known_answers(dev, golden_dir):
    from anvilq_b200 import ops
    data = json.loads((golden_dir / "dequant_cases.json").read_text())
    for qw, qz, h, lane, w, invalid, w32 in data["cases"]:
        qweight = T(np.array([[qw]], np.uint32).view(np.int32), dev)
        qzeros = T(np.array([[qz]], np.uint32).view(np.int32), dev)
        sc = np.zeros((1, 8), np.uint16)
        sc[0, lane] = h
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        delta, wf = ops.dequant(qweight, qzeros, T(sc.view(np.float16), dev), 1, dev_err=err)
        exp_delta = ((qw >> oracle.SHIFTS[lane]) & 15) - ((qz >> oracle.SHIFTS[lane]) & 15)
        assert int(delta[0, lane]) == exp_delta
        assert int(err.item()) == invalid
        if not invalid:
            assert np.float32(wf[0, lane].item()) == np.float32(w32)


def test_dequant_matrix_bit_exact(dev):
    from anvilq_b200 import ops
    for K, N, G, seed in ((256, 512, 128, 17), (96, 64, 32, 43), (24, 48, 3, 89)):
        layer = synthetic.awq_layer(K, N, G, seed)
        d_ref, w_ref, _, _ = oracle.dequant(layer.qweight, layer.qzeros, layer.scales_bits, G)
        delta, w = ops.dequant(T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), G)
        assert (delta.cpu().numpy() == d_ref).all()
        assert (w.cpu().numpy().view(np.uint32) == w_ref.view(np.uint32)).all()


def test_pack_unpack(dev, golden_dir):
    from anvilq_b200 import ops
    g = np.load(golden_dir / "pack.npz")
    words = ops.pack_lanes(T(g["lanes_codes"], dev))
    assert (words.cpu().numpy().view(np.uint32) == g["lanes_words"]).all()
    assert (ops.unpack_lanes(words, 24).cpu().numpy() == g["lanes_codes"]).all()
    rng = np.random.default_rng(17)
    codes = rng.integers(0, 16, size=(64, 96)).astype(np.uint8)
    packed = ops.pack(T(codes, dev))
    assert (packed.cpu().numpy().view(np.uint32) == oracle.pack_rows(codes)).all()
    assert (ops.unpack(packed).cpu().numpy() == codes).all()


def _linear_cases(g):
    names = ["official_p0", "official_p1", "official_p4"] + [str(n) for n in g["case_names"]]
    for key in names:
        G = int(g[key + "_G"]) if key + "_G" in g else 128
        bias = g[key + "_bias"] if key + "_bias" in g else None
        yield key, g[key + "_x"], g[key + "_qweight"], g[key + "_qzeros"], g[key + "_scales"], bias, G


def test_exact_kernel_bit_identical_to_reference(dev, golden_dir):
    """The reference-order kernel reproduces FP32Model.linear bit for bit."""
    from anvilq_b200 import ops
    g = np.load(golden_dir / "linear.npz")
    for key, x, qw, qz, sc, bias, G in _linear_cases(g):
        y = ops.gemm_exact(T(x.astype(np.float16), dev), T(qw.view(np.int32), dev), T(qz.view(np.int32), dev),
                           T(sc.view(np.float16), dev), None if bias is None else T(bias.view(np.float16), dev), G)
        ops.raise_device_errors(dev)
        assert (y.cpu().numpy().view(np.uint32) == g[key + "_y"].view(np.uint32)).all(), key


def test_fast_kernel_golden_fixtures(dev, golden_dir):
    """Every fixture through the public GEMM (fast kernels where the shape allows)."""
    from anvilq_b200 import ops
    g = np.load(golden_dir / "linear.npz")
    for key, x, qw, qz, sc, bias, G in _linear_cases(g):
        y = ops.gemm(T(x.astype(np.float16), dev), T(qw.view(np.int32), dev), T(qz.view(np.int32), dev),
                     T(sc.view(np.float16), dev), None if bias is None else T(bias.view(np.float16), dev), G)
        ops.raise_device_errors(dev)
        err, cos = oracle.normalized_error(y.float().cpu().numpy(), g[key + "_y"])
        assert err <= TOL_ERR and (cos is None or cos >= TOL_COS), (key, err, cos)


def test_qwen05b_gate_proj_full_size(dev, golden_dir):
    """Qwen2.5-0.5B gate_proj (896 x 4864) against FP32Model.linear's own output."""
    from anvilq_b200 import ops
    g = np.load(golden_dir / "qwen05b_gate_proj_896x4864.npz")
    x, layer = synthetic.gemv_case(1, 896, 4864, 128, 17, False)
    y = ops.gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 128)
    ops.raise_device_errors(dev)
    err, cos = oracle.normalized_error(y.float().cpu().numpy(), g["y"])
    assert err <= TOL_ERR and cos >= TOL_COS, (err, cos)


SHAPES = [(896, 4864), (4864, 896), (896, 896), (896, 128), (4096, 4096), (4096, 11008), (11008, 4096)]


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_fast_kernel_shapes(dev, M, K, N):
    from anvilq_b200 import ops
    seed = {1: 17, 2: 43, 4: 89, 8: 17}[M]
    x, layer = synthetic.gemv_case(M, K, N, 128, seed, bias=(N == 128))
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                           layer.bias_bits, 128, threads=oracle.max_threads())
    args = (T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev),
            None if layer.bias is None else T(layer.bias, dev), 128)
    y1 = ops.gemm(*args)
    y2 = ops.gemm(*args)          # workspace reuse: tickets re-armed, deterministic
    ops.raise_device_errors(dev)
    assert torch.equal(y1, y2)
    err, cos = oracle.normalized_error(y1.float().cpu().numpy(), ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (M, K, N, err, cos)


@pytest.mark.parametrize("M", [2, 4, 8, 12])
def test_small_m_large_activations(dev, M):
    """Activations up to |x| = 1000 (past where 16-product binary16 partial sums
    overflow: 16 * 15 * 1000 > 65504) stay finite and within the tolerance: the
    small-M kernels sum x (q - z) in fp32."""
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(M, 4096, 4096, 128, 61)
    rng = np.random.default_rng(61)
    x = np.clip(rng.standard_normal((M, 4096)) * 300.0, -1000.0, 1000.0).astype(np.float16)
    x[:, 0] = 1000.0
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                           None, 128, threads=oracle.max_threads())
    assert np.isfinite(ref).all() and np.abs(ref).max() < 6e4
    y = ops.gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 128)
    ops.raise_device_errors(dev)
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    err, cos = oracle.normalized_error(got, ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (M, err, cos)


@pytest.mark.parametrize("M", [16, 64])
def test_verify_batch(dev, M):
    from anvilq_b200 import ops
    x, layer = synthetic.gemv_case(M, 4096, 4096, 128, 43)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                           None, 128, threads=oracle.max_threads())
    y = ops.gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(layer.scales, dev), None, 128)
    ops.raise_device_errors(dev)
    err, cos = oracle.normalized_error(y.float().cpu().numpy(), ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (M, err, cos)


def test_invalid_scale_fails_operation(dev):
    from anvilq_b200 import ops, AnvilqError
    for bad in (0x7C00, 0xFC00, 0x7E00, 0x8001, 0xBC00):
        x, layer = synthetic.gemv_case(1, 512, 256, 128, 17)
        sc = layer.scales_bits.copy()
        sc[2, 77] = bad
        args = (T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(sc.view(np.float16), dev), None, 128)
        ops.gemm(*args)
        with pytest.raises(AnvilqError):
            ops.raise_device_errors(dev)
        ops.gemm_exact(*args)
        with pytest.raises(AnvilqError):
            ops.raise_device_errors(dev)
    sc = layer.scales_bits.copy()
    sc[1, 5] = 0x8000           # negative zero is a valid scale
    ops.gemm(T(x, dev), T(layer.qweight, dev), T(layer.qzeros, dev), T(sc.view(np.float16), dev), None, 128)
    ops.raise_device_errors(dev)


def test_golden_api_linear(dev):
    """GpuLinear.linear has FP32Model.linear's signature and meaning."""
    from anvilq_b200.checkpoint import ArrayCheckpoint, gemv_shape
    from anvilq_b200.golden_api import GpuLinear
    x, layer = synthetic.gemv_case(1, 256, 64, 128, 43, bias=True)
    ckpt = ArrayCheckpoint({(0, 0): layer})
    shape = gemv_shape(256, 64, 128, 0)
    y = GpuLinear(ckpt, shape).linear([float(v) for v in x[0]], 0, 0)
    ref = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                           layer.bias_bits, 128)
    err, cos = oracle.normalized_error(np.asarray(y), ref)
    assert err <= TOL_ERR and cos >= TOL_COS
    y_exact = GpuLinear(ckpt, shape).linear([float(v) for v in x[0]], 0, 0, exact=True)
    assert np.asarray(y_exact, np.float32).view(np.uint32).tolist() == ref[0].view(np.uint32).tolist()


def test_golden_api_dequant(dev, golden_dir):
    from anvilq_b200.golden_api import dequant
    data = json.loads((golden_dir / "dequant_cases.json").read_text())
    for qw, qz, h, lane, w, invalid, _ in data["cases"][::7]:
        assert dequant(qw, qz, h, lane) == (w, invalid)
