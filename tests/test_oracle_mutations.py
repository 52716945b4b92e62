"""Mutation tests: the reference's golden fixtures must catch planted mistakes.

The reference kills source mutations of its datapath with its functional checks
(anvil-q1/tests/verify.py:3019-3043: wrong AWQ lane shift, dropped bias, GQA
mapping, dequant truncated to 32 bits, 64-bit accumulator, ...).  Here the
mistakes are planted in the CPU oracle -- the checker every GPU parity test
compares against -- and each one must make the comparison with the fixtures
(tests/golden, produced by running the reference itself) fail.  Where a
mutant is a separate restatement, the unmutated restatement is checked to pass
first, so a mutant is only "killed" by the fixture, never by a broken harness.
"""
import json

import numpy as np

import oracle


def test_wrong_awq_lane_shift_is_caught(golden_dir, monkeypatch):
    """verify.py mutation "1: shift=4": lane 1 read from nibble 1 instead of nibble 4."""
    g = np.load(golden_dir / "pack.npz")
    assert (oracle.unpack_lanes(g["lanes_words"], 24) == g["lanes_codes"]).all()
    order = list(oracle.NIBBLE_ORDER)
    order[1], order[2] = order[2], order[1]
    monkeypatch.setattr(oracle, "NIBBLE_ORDER", tuple(order))
    assert not (oracle.unpack_lanes(g["lanes_words"], 24) == g["lanes_codes"]).all()
    assert not (oracle.pack_lanes(g["lanes_codes"]) == g["lanes_words"]).all()


def test_dropped_bias_is_caught(golden_dir):
    g = np.load(golden_dir / "linear.npz")
    key = "official_p0"                  # the q projection carries a bias
    args = (g[key + "_x"], g[key + "_qweight"], g[key + "_qzeros"], g[key + "_scales"])
    ref = g[key + "_y"].view(np.uint32)
    assert (oracle.gemv_fp32_numpy(*args, g[key + "_bias"], 128).view(np.uint32) == ref).all()
    assert not (oracle.gemv_fp32_numpy(*args, None, 128).view(np.uint32) == ref).all()


def test_dequant_truncated_to_32_bits_is_caught(golden_dir):
    """The Q16.16 weight delta * S needs more than 32 bits (up to 15 * 65504 * 2^16)."""
    cases = json.loads((golden_dir / "dequant_cases.json").read_text())["cases"]
    wrap32 = lambda v: ((v + (1 << 31)) % (1 << 32)) - (1 << 31)
    killed = 0
    for qw, qz, h, lane, w, invalid, _ in cases:
        got, bad = oracle.dequant_scalar(qw, qz, h, lane)
        assert (got, bad) == (w, invalid)
        killed += wrap32(got) != w
    assert killed > 0


def _q16_linear(x, w_q16, wrap64):
    """FixedModel.linear's accumulation (official_weights.py:592-612, SPEC.md:151-158):
    sum x * w in wide integers, round half away from zero >> 16, saturate to int32;
    wrap64 narrows the running sum to a signed 64-bit register (the mutation)."""
    out = []
    for c in range(w_q16.shape[1]):
        acc = 0
        for k in range(w_q16.shape[0]):
            acc += int(x[k]) * int(w_q16[k, c])
            if wrap64:
                acc = ((acc + (1 << 63)) % (1 << 64)) - (1 << 63)
        m = (abs(acc) + (1 << 15)) >> 16
        v = -m if acc < 0 else m
        out.append(max(-(1 << 31), min((1 << 31) - 1, v)))
    return out


def test_64_bit_accumulator_is_caught():
    """verify.py:536-615 wide cancellation: the exact sum passes through values past
    2^63 before cancelling; a 64-bit accumulator wraps and gets it wrong."""
    K, G = 9216, 8
    x = np.where(np.arange(K) < 4608, 8388352, -8388352).astype(np.int64)
    qweight = np.where(np.arange(K) < 4608, 0xFFFFFF0F, 0xFFF0FF0F).astype(np.uint32)[:, None]
    qzeros = np.where(np.arange(K // G) < 576, 0x000000F0, 0).astype(np.uint32)[:, None]
    scales = np.full((K // G, 8), 0x7BFF, np.uint16)
    _, _, w_q16, bad = oracle.dequant(qweight, qzeros, scales, G)
    assert not bad.any()
    expected = [0, 0x7FFFFFFF, -0x80000000, 0, 0, 0, 0, 0]
    assert oracle.gemv_q16(x[None].astype(np.int32), qweight, qzeros, scales, None, G)[0].tolist() == expected
    cols = w_q16[:, :3]
    assert _q16_linear(x, cols, wrap64=False) == expected[:3]
    assert _q16_linear(x, cols, wrap64=True) != expected[:3]


def _attention_mapping(q, keys, values, contiguous):
    """attention() with kv head j // group (contiguous groups, fp64_reference.py:164-170)
    or, mutated, j % Hkv (interleaved)."""
    hq, d = q.shape
    hkv = keys.shape[1]
    group = hq // hkv
    out = np.empty((hq, d))
    for j in range(hq):
        h = j // group if contiguous else j % hkv
        s = keys[:, h].astype(np.float64) @ q[j].astype(np.float64) / np.sqrt(d)
        p = np.exp(s - s.max())
        out[j] = (p / p.sum()) @ values[:, h].astype(np.float64)
    return out


def test_gqa_mapping_is_caught(golden_dir):
    g = np.load(golden_dir / "attention.npz")
    key = "attn_H14_2_D64_T37_s43"       # 14 query heads over 2 kv heads
    q, k, v, ref = g[key + "_q"], g[key + "_k"], g[key + "_v"], g[key + "_y"]
    np.testing.assert_allclose(_attention_mapping(q, k, v, True), ref, rtol=1e-10, atol=1e-12)
    assert not np.allclose(_attention_mapping(q, k, v, False), ref, rtol=1e-3, atol=1e-3)


def test_legacy_codec_mutations_are_caught(golden_dir, monkeypatch):
    """Rounding half to even instead of half away from zero, and the symmetric
    exponent taken from the ROUNDED magnitude (the SPEC requires the unrounded
    one, anvil-q4/design/SPEC.md:254-258) -- each changes some fixture block."""
    g = np.load(golden_dir / "legacy_kv.npz")
    blocks = [[int(v) for v in g[f"b{i}_in"]] for i in range(int(g["count"]))]

    def mismatches():
        bad = 0
        for i, b in enumerate(blocks):
            for fmt in (1, 2, 3):
                meta, codes, decoded = oracle.legacy_kv_block(b, fmt)
                bad += (meta != int(g[f"b{i}_f{fmt}_meta"]) or codes != [int(c) for c in g[f"b{i}_f{fmt}_codes"]]
                        or decoded != [int(d) for d in g[f"b{i}_f{fmt}_decoded"]])
        return bad

    assert mismatches() == 0
    exact = oracle._round_away_shift

    def half_even(v, e):
        if e == 0:
            return v
        q, r = divmod(v, 1 << e)           # floor division
        half = 1 << (e - 1)
        return q + (1 if r > half or (r == half and q % 2) else 0)

    monkeypatch.setattr(oracle, "_round_away_shift", half_even)
    assert mismatches() > 0
    monkeypatch.setattr(oracle, "_round_away_shift", exact)

    def rounded_exponent(values, fmt):
        if fmt == 3:
            return real(values, fmt)
        limit, emax = oracle.LEGACY_LIMITS[fmt]
        e = next(k for k in range(emax + 1) if max(abs(exact(v, k)) for v in values) <= limit)
        codes = [min(limit, max(-limit, exact(int(v), e))) for v in values]
        return e, codes, [oracle._sat32(c << e) for c in codes]

    real = oracle.legacy_kv_block
    monkeypatch.setattr(oracle, "legacy_kv_block", rounded_exponent)
    assert mismatches() > 0


def test_int8_cache_without_negative_zero_escape_is_caught(golden_dir):
    """A head holding -0.0 must escape (anvil-q4/design/SPEC.md:218-221); treating it
    as +0 encodes it as an ordinary head, which the fixtures reject."""
    g = np.load(golden_dir / "kv_int8.npz")
    killed = 0
    for i in range(int(g["count"])):
        h = g[f"h{i}_in"].copy()
        if not (h == 0x80000000).any():
            continue
        scale, codes, _, _ = oracle.kv_int8_encode(h[None])
        assert int(scale[0]) == int(g[f"h{i}_scale"])
        h[h == 0x80000000] = 0
        scale_m, codes_m, _, _ = oracle.kv_int8_encode(h[None])
        killed += int(scale_m[0]) != int(g[f"h{i}_scale"]) or not np.array_equal(
            codes_m[0].view(np.uint8), g[f"h{i}_codes"])
    assert killed > 0
