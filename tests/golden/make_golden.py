#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ by running the reference itself.

This script imports the reference's own Python golden models read-only from a
checkout of aHappend/anvil-q, named by --reference or $ANVILQ_REFERENCE:

* anvil-q1/tests/verify.py         dequant_cases / dequant / pack / rounded / sat / half_fixed
* anvil-q1/tests/official_weights.py  FP32Model.linear, FP32Model.token, f32
* anvil-q1-fp/tests/awq_prepare.py    pack_lanes / unpack_lanes
* anvil-q1-fp/tests/fp64_reference.py attention
* anvil-q4/tests/cache_reference.py  encode_head (per-head INT8 KV cache with FP32 escape)
* anvil-q4/tests/legacy_reference.py cache_block (legacy symmetric INT8/INT4 and asymmetric INT4
                                     KV-cache codecs over Q16.16 values)

and writes their outputs on seeded inputs.  The tests only read the fixtures;
nothing at test time needs the reference.  Run from the repository root:

    python tests/golden/make_golden.py --reference <checkout of aHappend/anvil-q>
"""
from __future__ import annotations

import json
import os
import struct
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _reference_root() -> Path:
    import argparse
    ap = argparse.ArgumentParser(description="regenerate tests/golden from the reference's own golden models")
    ap.add_argument("--reference", default=os.environ.get("ANVILQ_REFERENCE"),
                    help="checkout of aHappend/anvil-q (default: $ANVILQ_REFERENCE)")
    args, _ = ap.parse_known_args()
    if not args.reference:
        raise SystemExit("name the reference checkout: --reference <path> or $ANVILQ_REFERENCE")
    root = Path(args.reference)
    if not (root / "anvil-q1" / "tests" / "official_weights.py").exists():
        raise SystemExit(f"{root} does not hold anvil-q1/tests/official_weights.py")
    return root


REF = _reference_root()
sys.path.insert(0, str(REPO))


def _load(name, path):
    """Import one reference module by file path under a unique name (anvil-q1 and
    anvil-q1-fp both ship a tests/verify.py)."""
    import importlib.util
    sys.path.insert(0, str(path.parent))
    try:
        spec = importlib.util.spec_from_file_location(name, path)
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
        return module
    finally:
        sys.path.remove(str(path.parent))


ow = _load("official_weights", REF / "anvil-q1" / "tests" / "official_weights.py")
verify = _load("anvil_q1_verify", REF / "anvil-q1" / "tests" / "verify.py")
sys.path.insert(0, str(REF / "anvil-q1-fp" / "tests"))
import fp64_reference  # noqa: E402
import awq_prepare  # noqa: E402

from anvilq_b200.checkpoint import ArrayCheckpoint, gemv_shape  # noqa: E402
from anvilq_b200 import synthetic  # noqa: E402

SLICE = REF / "anvil-q1" / "hf_qwen25_05b_awq_spec" / "official_layer0_awq_slice.json"


def f16_bits(values):
    return np.asarray(values, np.float16).view(np.uint16)


def dequant_fixture():
    slices = json.loads(SLICE.read_text())
    cases, official = verify.dequant_cases(slices)
    rows = []
    for qw, qz, h, lane, w, invalid in cases:
        if invalid:
            w32 = None
        else:
            delta = ((qw >> verify.SHIFTS[lane]) & 15) - ((qz >> verify.SHIFTS[lane]) & 15)
            scale = struct.unpack("<e", struct.pack("<H", h))[0]
            w32 = ow.f32(delta * scale)
        rows.append([qw, qz, h, lane, w, invalid, w32])
    return dict(source="anvil-q1/tests/verify.py:357-384 dequant_cases + official_weights.py:428-431",
                official_cases=official, cases=rows)


def pack_fixture():
    rng = np.random.default_rng(17)
    vectors = rng.integers(0, 16, size=(64, 8))
    packed = [verify.pack([int(v) for v in vec]) for vec in vectors]
    awq_prepare.numerics()
    codes = rng.integers(0, 16, size=(24, 16)).astype(np.uint8)   # [N outputs, K inputs]
    lanes = awq_prepare.pack_lanes(codes)
    back = awq_prepare.unpack_lanes(lanes, 24)
    assert (back == codes).all()
    return dict(pack_vectors=vectors, pack_words=np.asarray(packed, np.uint64),
                lanes_codes=codes, lanes_words=lanes.astype(np.uint32))


def official_layers():
    """Official layer-0 Q/K/gate 8x8 words, G=128 group 0 (verify.py:618-660)."""
    t = json.loads(SLICE.read_text())["tensors"]
    out = {}
    for p, name in ((0, "self_attn.q_proj"), (1, "self_attn.k_proj"), (4, "mlp.gate_proj")):
        prefix = "model.layers.0." + name + "."
        hexes = [t[prefix + s]["raw_hex"] for s in ("qweight", "qzeros", "scales")]
        qweight = np.array([[int(hexes[0][r][0], 16)] for r in range(8)], np.uint32)
        qzeros = np.array([[int(hexes[1][0][0], 16)]], np.uint32)
        scales = np.array([[int(hexes[2][0][c], 16) for c in range(8)]], np.uint16)
        bias = (np.array([int(h, 16) for h in t[prefix + "bias"]["raw_hex"][:8]], np.uint16)
                if p < 3 else None)
        out[p] = (qweight, qzeros, scales, bias)
    return out


def fp32_linear(x, qweight, qzeros, scales_bits, bias_bits, G, projection):
    """Run the reference FP32Model.linear on an ArrayCheckpoint."""
    layer = synthetic.AwqLayer(qweight.view(np.int32), qzeros.view(np.int32),
                               scales_bits.view(np.float16),
                               None if bias_bits is None else bias_bits.view(np.float16), G)
    K, N = layer.K, layer.N
    shape = gemv_shape(K, N, G, projection)
    model = ow.FP32Model(ArrayCheckpoint({(0, projection): layer}), shape)
    return np.asarray([model.linear([float(v) for v in row], 0, projection) for row in x], np.float32)


def q16_linear(x_q16, qweight, qzeros, scales_bits, bias_bits, G):
    """The integer GEMV golden composed from verify.py (dequant, rounded, sat, half_fixed)
    exactly as verify.py:618-660 builds its official GEMV expectations."""
    K, N = qweight.shape[0], qweight.shape[1] * 8
    y = np.zeros((x_q16.shape[0], N), np.int64)
    for m, row in enumerate(x_q16):
        for c in range(N):
            total = 0
            for k in range(K):
                value, invalid = verify.dequant(int(qweight[k, c // 8]), int(qzeros[k // G, c // 8]),
                                                int(scales_bits[k // G, c]), c % 8)
                assert not invalid
                total += int(row[k]) * value
            if bias_bits is not None:
                total += verify.sat(verify.half_fixed(int(bias_bits[c]))) * 65536
            y[m, c] = verify.sat(verify.rounded(total, 65536))
    return y.astype(np.int32)


def linear_fixture():
    out = {}
    # (1) official 8x8 submatrices, activations of verify.py:621
    act = np.array([-769, 511, -257, 127, -31, 17, -1, 3], np.float64) / 256
    for p, (qw, qz, sc, bias) in official_layers().items():
        x = act[None, :].astype(np.float32)
        out[f"official_p{p}_x"] = x
        out[f"official_p{p}_qweight"] = qw
        out[f"official_p{p}_qzeros"] = qz
        out[f"official_p{p}_scales"] = sc
        if bias is not None:
            out[f"official_p{p}_bias"] = bias
        out[f"official_p{p}_y"] = fp32_linear(x, qw, qz, sc, bias, 128, p)
        xq = np.array([[-769, 511, -257, 127, -31, 17, -1, 3]], np.int64) * 256
        out[f"official_p{p}_xq16"] = xq.astype(np.int32)
        out[f"official_p{p}_yq16"] = q16_linear(xq, qw, qz, sc, bias, 128)
    # (2) reduced shapes with the reference's integrated() stimulus
    #     (verify.py:2039-2100: q 5..11, z 7..9, scales {1/128,1/64,3/128})
    names = []
    for label, (K, N, G) in (("A", (16, 32, 8)), ("B", (112, 128, 16)), ("C", (24, 48, 3)),
                             ("D", (8, 8, 8))):
        for seed in (17, 43, 89):
            rng = np.random.default_rng(seed)
            codes = rng.integers(5, 12, size=(K, N)).astype(np.uint8)
            zcodes = rng.integers(7, 10, size=(K // G, N)).astype(np.uint8)
            qw = awq_prepare.pack_lanes(codes.T).astype(np.uint32)
            qz = awq_prepare.pack_lanes(zcodes.T).astype(np.uint32)
            sc = f16_bits(rng.choice([1 / 128, 1 / 64, 3 / 128], size=(K // G, N)))
            bias = f16_bits(rng.standard_normal(N)) if label in ("A", "C") else None
            x = rng.standard_normal((2, K)).astype(np.float16).astype(np.float32)
            key = f"matrix{label}_s{seed}"
            names.append(key)
            out[key + "_x"], out[key + "_qweight"], out[key + "_qzeros"] = x, qw, qz
            out[key + "_scales"] = sc
            if bias is not None:
                out[key + "_bias"] = bias
            out[key + "_G"] = np.array(G)
            out[key + "_y"] = fp32_linear(x, qw, qz, sc, bias, G, 0 if bias is not None else 4)
            xq = np.round(x.astype(np.float64) * 65536).astype(np.int64)
            out[key + "_xq16"] = xq.astype(np.int32)
            out[key + "_yq16"] = q16_linear(xq, qw, qz, sc, bias, G)
    # (3) the benchmark value distributions at small sizes (x ~ N(0,1), u4 uniform, scales |N|*.01+1e-3)
    for (M, K, N, seed, bias) in ((1, 256, 64, 17, False), (1, 256, 64, 43, True),
                                  (4, 384, 128, 89, False), (2, 128, 256, 17, True)):
        x, layer = synthetic.gemv_case(M, K, N, 128, seed, bias)
        key = f"dist_M{M}_K{K}_N{N}_s{seed}{'_bias' if bias else ''}"
        names.append(key)
        xf = x.astype(np.float32)
        out[key + "_x"] = xf
        out[key + "_qweight"] = layer.qweight.view(np.uint32)
        out[key + "_qzeros"] = layer.qzeros.view(np.uint32)
        out[key + "_scales"] = layer.scales_bits
        if bias:
            out[key + "_bias"] = layer.bias_bits
        out[key + "_G"] = np.array(128)
        out[key + "_y"] = fp32_linear(xf, layer.qweight.view(np.uint32), layer.qzeros.view(np.uint32),
                                      layer.scales_bits, layer.bias_bits, 128, 0 if bias else 4)
    out["case_names"] = np.array(names)
    return out


def qwen05b_gate_proj_fixture():
    """Qwen2.5-0.5B gate_proj shape, the reference's CPU-runnable case: K=896, N=4864, G=128,
    seed 17.  Inputs are regenerated from anvilq_b200.synthetic.gemv_case; their digests
    are stored to catch generator drift."""
    import hashlib
    x, layer = synthetic.gemv_case(1, 896, 4864, 128, 17, False)
    t0 = time.time()
    y = fp32_linear(x.astype(np.float32), layer.qweight.view(np.uint32), layer.qzeros.view(np.uint32),
                    layer.scales_bits, None, 128, 4)
    dt = time.time() - t0
    digest = hashlib.sha256()
    for a in (x, layer.qweight, layer.qzeros, layer.scales):
        digest.update(np.ascontiguousarray(a).tobytes())
    return dict(y=y, input_sha256=np.array(digest.hexdigest()), reference_seconds=np.array(dt))


def attention_fixture():
    out = {}
    names = []
    for (Hq, Hkv, D, T, seed) in ((14, 2, 64, 1, 17), (14, 2, 64, 37, 43), (32, 8, 128, 20, 89),
                                  (8, 2, 128, 130, 17), (4, 4, 16, 7, 43)):
        rng = np.random.default_rng(seed)
        q = rng.standard_normal((Hq, D)).astype(np.float16)
        k = rng.standard_normal((T, Hkv, D)).astype(np.float16)
        v = rng.standard_normal((T, Hkv, D)).astype(np.float16)
        y = fp64_reference.attention(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64))
        key = f"attn_H{Hq}_{Hkv}_D{D}_T{T}_s{seed}"
        names.append(key)
        out[key + "_q"], out[key + "_k"], out[key + "_v"] = q, k, v
        out[key + "_y"] = y
    out["case_names"] = np.array(names)
    return out


DECODE_SHAPE = (2, 128, 256, 2, 1, 64, 128, 64, 8)   # (L,H,I,QH,KVH,D,G,V,SEQ)


def decode_fixture():
    """FP32Model.token (official_weights.py:451-509) greedy-decoding 4 tokens on a
    small Qwen2-shaped model with synthetic weights (anvilq_b200.decoder.synthetic_weights,
    seed 29), starting from token 5."""
    import hashlib
    from anvilq_b200 import decoder
    w = decoder.synthetic_weights(DECODE_SHAPE, seed=29)
    model = ow.FP32Model(w.checkpoint(), DECODE_SHAPE)
    tokens, logits = [5], []
    for pos in range(4):
        out = model.token(tokens[-1], pos, new_sequence=(pos == 0))
        logits.append(np.asarray(out, np.float32))
        best = max(range(len(out)), key=lambda i: (out[i], -i))
        tokens.append(best)
    digest = hashlib.sha256()
    for projs in w.layers:
        for p in range(7):
            digest.update(np.ascontiguousarray(projs[p].qweight).tobytes())
    digest.update(w.embedding.tobytes())
    return dict(shape=np.array(DECODE_SHAPE), tokens=np.array(tokens), logits=np.stack(logits),
                weights_sha256=np.array(digest.hexdigest()))


def kv_int8_fixture():
    """cache_reference.encode_head on its own CASES and on seeded heads (ordinary
    N(0,1)-scaled values, tiny magnitudes near the scale underflow, -0.0 / inf / NaN
    escapes), D = 2..128."""
    cr = _load("anvilq_q4_cache_reference", REF / "anvil-q4" / "tests" / "cache_reference.py")
    heads = [list(v) for v in cr.CASES.values()]
    rng = np.random.default_rng(170043)
    for d in (2, 8, 64, 128):
        for kind in range(6):
            v = (rng.standard_normal(d) * (10.0 ** rng.integers(-4, 4))).astype(np.float32).view(np.uint32)
            if kind == 1:
                v = rng.integers(0, 80, size=d).astype(np.uint32)            # subnormal units around 63/64
            if kind == 2:
                v[rng.integers(0, d)] = 0x80000000                           # negative zero
            if kind == 3:
                v[rng.integers(0, d)] = (0x7F800000, 0xFF800000)[int(rng.integers(0, 2))]
            if kind == 4:
                v[rng.integers(0, d)] = 0x7F800000 | int(rng.integers(1, 1 << 23)) | (int(rng.integers(0, 2)) << 31)
            if kind == 5:
                v = np.zeros(d, np.uint32)
            heads.append([int(b) for b in v])
    out = {"count": np.array(len(heads))}
    for i, h in enumerate(heads):
        scale, codes, recon = cr.encode_head(h)
        out[f"h{i}_in"] = np.array(h, np.uint32)
        out[f"h{i}_scale"] = np.array(scale, np.uint32)
        out[f"h{i}_codes"] = np.array(codes, np.uint8)
        out[f"h{i}_recon"] = np.array(recon, np.uint32)
    return out


def legacy_kv_fixture():
    """legacy_reference.cache_block for the three legacy cache formats (1: INT8
    symmetric, 2: INT4 symmetric, 3: INT4 asymmetric) on the SPEC's worked
    values, int32 extremes, zero and one-sided blocks, and seeded Q16.16 blocks
    of lengths 1..64 over magnitudes 2^0..2^31."""
    sys.path.insert(0, str(REF / "anvil-q4" / "tests"))
    lr = _load("anvilq_q4_legacy_reference", REF / "anvil-q4" / "tests" / "legacy_reference.py")
    lo, hi = -(1 << 31), (1 << 31) - 1
    blocks = [[509, -509, 3, 0], [29, -29, 1], [0] * 8, [lo, hi, 0, 1], [lo] * 5, [hi] * 3, [-1, -2, -3],
              [1, 2, 3, 4, 5, 6, 7, 8], [-7, 7, 8, -8], [hi, -hi], [(1 << 30) + 12345, -5], [127, -127, 128],
              [7, -7, 8], [254, 255, 256, -1]]
    rng = np.random.default_rng(20250417)
    for n in (1, 2, 7, 8, 24, 32, 63, 64):
        for _ in range(6):
            mag = 1 << int(rng.integers(0, 32))
            v = rng.integers(-mag, mag, size=n, dtype=np.int64)
            if rng.integers(0, 4) == 0:
                v = np.abs(v) + int(rng.integers(0, 1000))      # one-sided (asymmetric zero point)
            blocks.append([int(min(hi, max(lo, x))) for x in v])
    out = {"count": np.array(len(blocks))}
    for i, b in enumerate(blocks):
        out[f"b{i}_in"] = np.array(b, np.int32)
        for fmt in (1, 2, 3):
            meta, codes, decoded = lr.cache_block(b, fmt)
            out[f"b{i}_f{fmt}_meta"] = np.array(meta, np.int32)
            out[f"b{i}_f{fmt}_codes"] = np.array(codes, np.int8)
            out[f"b{i}_f{fmt}_decoded"] = np.array(decoded, np.int32)
    return out


def main():
    t0 = time.time()
    only = set(sys.argv[1:])
    if only:
        if "attention" in only:
            np.savez_compressed(HERE / "attention.npz", **attention_fixture())
        if "decode" in only:
            np.savez_compressed(HERE / "decode_small.npz", **decode_fixture())
        if "kv_int8" in only:
            np.savez_compressed(HERE / "kv_int8.npz", **kv_int8_fixture())
        if "legacy_kv" in only:
            np.savez_compressed(HERE / "legacy_kv.npz", **legacy_kv_fixture())
        return
    (HERE / "dequant_cases.json").write_text(json.dumps(dequant_fixture()))
    np.savez_compressed(HERE / "pack.npz", **pack_fixture())
    np.savez_compressed(HERE / "linear.npz", **linear_fixture())
    np.savez_compressed(HERE / "attention.npz", **attention_fixture())
    np.savez_compressed(HERE / "qwen05b_gate_proj_896x4864.npz", **qwen05b_gate_proj_fixture())
    np.savez_compressed(HERE / "decode_small.npz", **decode_fixture())
    np.savez_compressed(HERE / "kv_int8.npz", **kv_int8_fixture())
    np.savez_compressed(HERE / "legacy_kv.npz", **legacy_kv_fixture())
    print(f"golden fixtures written in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
