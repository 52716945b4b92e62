"""Pins the CPU oracle to the reference's own golden outputs (tests/golden/*).

The fixtures were produced by tests/golden/make_golden.py, which imports the
reference's verify.py / official_weights.py / awq_prepare.py / fp64_reference.py.
"""
import json

import numpy as np
import pytest

import oracle


def test_dequant_known_answers(golden_dir):
    """verify.py:357-384 directed + official cases: Q16.16 value, invalid flag, f32 weight."""
    data = json.loads((golden_dir / "dequant_cases.json").read_text())
    cases = data["cases"]
    assert len(cases) == 18 * 8 * 7 + data["official_cases"]
    for qw, qz, h, lane, w, invalid, w32 in cases:
        got, bad = oracle.dequant_scalar(qw, qz, h, lane)
        assert bad == invalid, (qw, qz, h, lane)
        assert got == w, (qw, qz, h, lane)
        if not invalid:
            qweight = np.array([[qw]], np.uint32)
            qzeros = np.array([[qz]], np.uint32)
            scales = np.zeros((1, 8), np.uint16)
            scales[0, lane] = h
            _, wf, _, _ = oracle.dequant(qweight, qzeros, scales, 1)
            assert np.float32(wf[0, lane]) == np.float32(w32)


def test_spec_dequant_values():
    """anvil-q1/design/SPEC.md:193-198 known values."""
    def q16(h, delta):
        words = [0] * 8
        zeros = [0] * 8
        if delta >= 0:
            words[0] = delta
        else:
            zeros[0] = -delta
        return oracle.dequant_scalar(oracle.pack8(words), oracle.pack8(zeros), h, 0)
    assert q16(0x6C00, 15) == (4026531840, 0)
    assert q16(0x7BFF, 15) == (64393052160, 0)
    assert q16(0x6C00, 8) == (2147483648, 0)
    assert q16(0x6C00, -8) == (-2147483648, 0)
    assert q16(0x6C00, 7) == (1879048192, 0)
    assert q16(0x77FF, 1) == (2146435072, 0)
    assert q16(0x7800, -1) == (-2147483648, 0)
    assert q16(0x7C00, 3) == (0, 1)
    assert q16(0x8001, 3) == (0, 1)
    assert q16(0x8000, 3) == (0, 0)


def test_pack_order(golden_dir):
    g = np.load(golden_dir / "pack.npz")
    for vec, word in zip(g["pack_vectors"], g["pack_words"]):
        assert oracle.pack8(vec) == int(word)
        assert int(oracle.pack_rows(np.asarray(vec, np.uint8)[None, :])[0, 0]) == int(word)
    words = oracle.pack_lanes(g["lanes_codes"])
    assert (words == g["lanes_words"]).all()
    assert (oracle.unpack_lanes(words, 24) == g["lanes_codes"]).all()
    # row-major C restatement agrees with the reference's output-major numpy layout
    assert (oracle.pack_rows(g["lanes_codes"].T) == g["lanes_words"]).all()
    assert (oracle.unpack_rows(g["lanes_words"], 24) == g["lanes_codes"].T).all()


def _linear_cases(g):
    names = ["official_p0", "official_p1", "official_p4"] + [str(n) for n in g["case_names"]]
    for key in names:
        G = int(g[key + "_G"]) if key + "_G" in g else 128
        bias = g[key + "_bias"] if key + "_bias" in g else None
        yield key, g[key + "_x"], g[key + "_qweight"], g[key + "_qzeros"], g[key + "_scales"], bias, G


def test_fp32_linear_bit_exact(golden_dir):
    """C and numpy restatements equal FP32Model.linear bit for bit."""
    g = np.load(golden_dir / "linear.npz")
    n = 0
    for key, x, qw, qz, sc, bias, G in _linear_cases(g):
        ref = g[key + "_y"]
        for threads in (1, 3):
            y = oracle.gemv_fp32(x, qw, qz, sc, bias, G, threads=threads)
            assert y.view(np.uint32).tolist() == ref.view(np.uint32).tolist(), key
        y2 = oracle.gemv_fp32_numpy(x, qw, qz, sc, bias, G)
        assert y2.view(np.uint32).tolist() == ref.view(np.uint32).tolist(), key
        n += 1
    assert n >= 19


def test_q16_linear_bit_exact(golden_dir):
    g = np.load(golden_dir / "linear.npz")
    for key, x, qw, qz, sc, bias, G in _linear_cases(g):
        if key + "_yq16" not in g:
            continue
        y = oracle.gemv_q16(g[key + "_xq16"], qw, qz, sc, bias, G, threads=2)
        assert (y == g[key + "_yq16"]).all(), key


def test_q16_wide_cancellation():
    """verify.py:536-615 test_case 0: K=9216, N=8, G=8, scale 0x7bff.  Column 1 saturates
    positive, column 2 negative, and the second half cancels the others to zero."""
    K, G = 9216, 8
    x = np.where(np.arange(K) < 4608, 8388352, -8388352).astype(np.int32)[None, :]
    qweight = np.where(np.arange(K) < 4608, 0xFFFFFF0F, 0xFFF0FF0F).astype(np.uint32)[:, None]
    qzeros = np.where(np.arange(K // G) < 576, 0x000000F0, 0).astype(np.uint32)[:, None]
    scales = np.full((K // G, 8), 0x7BFF, np.uint16)
    y = oracle.gemv_q16(x, qweight, qzeros, scales, None, G, threads=2)
    expected = [0, 0x7FFFFFFF, -0x80000000, 0, 0, 0, 0, 0]
    assert y[0].tolist() == expected


def test_qwen05b_gate_proj_full_size(golden_dir):
    """Qwen2.5-0.5B gate_proj (K=896, N=4864): C restatement equals FP32Model.linear."""
    import hashlib
    from anvilq_b200 import synthetic
    g = np.load(golden_dir / "qwen05b_gate_proj_896x4864.npz")
    x, layer = synthetic.gemv_case(1, 896, 4864, 128, 17, False)
    digest = hashlib.sha256()
    for a in (x, layer.qweight, layer.qzeros, layer.scales):
        digest.update(np.ascontiguousarray(a).tobytes())
    assert digest.hexdigest() == str(g["input_sha256"]), "synthetic generator drifted"
    y = oracle.gemv_fp32(x.astype(np.float32), layer.qweight, layer.qzeros, layer.scales_bits,
                         None, 128, threads=oracle.max_threads())
    assert y.view(np.uint32).tolist() == g["y"].view(np.uint32).tolist()


def test_attention(golden_dir):
    g = np.load(golden_dir / "attention.npz")
    for key in [str(n) for n in g["case_names"]]:
        q, k, v, ref = g[key + "_q"], g[key + "_k"], g[key + "_v"], g[key + "_y"]
        y64 = oracle.attention_f64(q, k, v)
        np.testing.assert_allclose(y64, ref, rtol=1e-12, atol=1e-12)
        y32 = oracle.attention_fp32(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16))
        err, cos = oracle.normalized_error(y32, ref)
        assert err <= 1e-5 and cos >= 0.99999, key


def test_invalid_scale_raises():
    x = np.ones((1, 8), np.float32)
    qw = np.zeros((8, 1), np.uint32)
    qz = np.zeros((1, 1), np.uint32)
    for bad in (0x7C00, 0xFC00, 0x7E00, 0x8001, 0xBC00):
        sc = np.full((1, 8), 0x3C00, np.uint16)
        sc[0, 3] = bad
        with pytest.raises(oracle.OracleError):
            oracle.gemv_fp32(x, qw, qz, sc, None, 8)
    sc = np.full((1, 8), 0x8000, np.uint16)      # negative zero is valid
    assert (oracle.gemv_fp32(x, qw, qz, sc, None, 8) == 0).all()


def test_kv_int8_encoding_matches_reference(golden_dir):
    """oracle.kv_int8_encode reproduces anvil-q4's cache_reference.encode_head (rational
    model) on its own cases and on seeded heads, escapes included, bit for bit."""
    g = np.load(golden_dir / "kv_int8.npz")
    n = int(g["count"])
    assert n >= 30
    for i in range(n):
        scale, codes, recon, esc = oracle.kv_int8_encode(g[f"h{i}_in"][None])
        assert int(scale[0]) == int(g[f"h{i}_scale"]), i
        assert np.array_equal(codes[0].view(np.uint8), g[f"h{i}_codes"]), i
        assert np.array_equal(recon[0], g[f"h{i}_recon"]), i
        if int(scale[0]) == oracle.KV_ESCAPE_MARKER:
            assert np.array_equal(esc[0], g[f"h{i}_recon"]), i
