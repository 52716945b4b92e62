"""CPU oracle for the W4A16 AWQ decode path -- TEST INFRASTRUCTURE ONLY.

This module is the checker.  Only the tests, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference arm of ``bench.py`` import it; the product package
(``anvilq_b200``) never does.  It restates the reference's golden models:

* ``pack_lanes`` / ``unpack_lanes``: anvil-q1-fp/tests/awq_prepare.py:84-99
  (nibble order (0, 4, 1, 5, 2, 6, 3, 7), i.e. bit shifts
  (0, 16, 4, 20, 8, 24, 12, 28) of anvil-q1/tests/verify.py:38).
* ``dequant``: anvil-q1/tests/verify.py:241-250 (Q16.16 integer) and
  anvil-q1/tests/official_weights.py:428-431 (binary32 ``f32(delta*scale)``).
* ``gemv_fp32``: FP32Model.linear, anvil-q1/tests/official_weights.py:418-437,
  in C (oracle/awq_oracle.c) and, vectorised over columns, in numpy
  (``gemv_fp32_numpy``); both sum in increasing k with every binary32 operation
  rounded separately, so both are bit-exact against the reference.
* ``gemv_q16``: FixedModel.linear, official_weights.py:592-612.
* ``attention_f64``: anvil-q1-fp/tests/fp64_reference.py:164-170.
* ``attention_fp32``: the FP32 loop of official_weights.py:471-486.

Parity of these restatements is pinned by tests/test_oracle_golden.py against
fixtures that tests/golden/make_golden.py produced by importing the reference.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

NIBBLE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)   # awq_prepare.py:18
SHIFTS = (0, 16, 4, 20, 8, 24, 12, 28)     # verify.py:38

_lib = None


def build(force: bool = False) -> Path:
    """Compile oracle/awq_oracle.c into oracle/liboracle.so with make."""
    src = HERE / "awq_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        I = ctypes.c_int
        L.anvilq_oracle_pack.argtypes = [P, P, I, I]
        L.anvilq_oracle_unpack.argtypes = [P, P, I, I]
        L.anvilq_oracle_dequant.argtypes = [P, P, P, I, I, I, P, P, P, P]
        L.anvilq_oracle_dequant.restype = ctypes.c_int64
        L.anvilq_oracle_gemv_fp32.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, I]
        L.anvilq_oracle_gemv_q16.argtypes = [P, P, P, P, P, P, I, I, I, I, I]
        L.anvilq_oracle_attention_fp32.argtypes = [P, P, P, P, I, I, I, I, P, I]
        L.anvilq_oracle_max_threads.restype = I
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


def max_threads() -> int:
    return int(lib().anvilq_oracle_max_threads())


class OracleError(ValueError):
    """Raised where the reference raises CheckpointError (official_weights.py:37)."""


_STATUS = {-1: "invalid argument", -2: "invalid AWQ scale (negative nonzero or nonfinite)",
           -3: "FP32 nonfinite result"}


def _check(status):
    if status != 0:
        raise OracleError(_STATUS.get(status, f"oracle status {status}"))


# ---------------------------------------------------------------- packing
def pack_lanes(codes):
    """awq_prepare.py:84-91: codes uint8 [N, K] (output-major) -> uint32 [K, N/8]."""
    codes = np.asarray(codes)
    if codes.ndim != 2 or codes.shape[0] % 8 or codes.min(initial=0) < 0 or codes.max(initial=0) > 15:
        raise OracleError("invalid nibble array")
    out = np.zeros((codes.shape[1], codes.shape[0] // 8), dtype="<u4")
    for lane, nib in enumerate(NIBBLE_ORDER):
        out |= codes[lane::8].T.astype("<u4") << (4 * nib)
    return out


def unpack_lanes(words, outputs):
    """awq_prepare.py:94-99: uint32 [K, N/8] -> uint8 [N, K]."""
    words = np.asarray(words, dtype="<u4")
    if words.ndim != 2 or words.shape[1] * 8 != outputs:
        raise OracleError("invalid packed output shape")
    out = np.empty((outputs, words.shape[0]), dtype=np.uint8)
    for lane, nib in enumerate(NIBBLE_ORDER):
        out[lane::8] = ((words >> (4 * nib)) & 15).T
    return out


def pack_rows(codes):
    """Row-major codes uint8 [K, N] -> qweight uint32 [K, N/8] (C restatement)."""
    codes = _c(codes, np.uint8)
    K, N = codes.shape
    out = np.empty((K, N // 8), dtype=np.uint32)
    _check(lib().anvilq_oracle_pack(_ptr(codes), _ptr(out), K, N))
    return out


def unpack_rows(packed, n):
    packed = _c(packed, np.uint32)
    out = np.empty((packed.shape[0], n), dtype=np.uint8)
    _check(lib().anvilq_oracle_unpack(_ptr(packed), _ptr(out), packed.shape[0], n))
    return out


def pack8(values):
    """verify.py:252-253."""
    return sum((int(v) & 15) << s for v, s in zip(values, SHIFTS))


# ---------------------------------------------------------------- dequant
def dequant(qweight, qzeros, scales_bits, G):
    """Element-wise dequantisation of a [K, N] AWQ matrix.

    Returns (delta int8 [K,N], w_f32 float32 [K,N], w_q16 int64 [K,N], invalid uint8 [K,N]).
    """
    qweight = _c(qweight, np.uint32)
    qzeros = _c(qzeros, np.uint32)
    scales_bits = _c(scales_bits, np.uint16)
    K, N = qweight.shape[0], qweight.shape[1] * 8
    delta = np.empty((K, N), np.int8)
    w = np.empty((K, N), np.float32)
    q16 = np.empty((K, N), np.int64)
    bad = np.empty((K, N), np.uint8)
    r = lib().anvilq_oracle_dequant(_ptr(qweight), _ptr(qzeros), _ptr(scales_bits), K, N, G,
                                    _ptr(delta), _ptr(w), _ptr(q16), _ptr(bad))
    if r < 0:
        _check(int(r))
    return delta, w, q16, bad


def dequant_scalar(qw, qz, h, lane):
    """verify.py:241-250 signature: (w_q16, invalid) for one lane of one word."""
    qweight = np.array([[qw & 0xFFFFFFFF]], np.uint32)
    qzeros = np.array([[qz & 0xFFFFFFFF]], np.uint32)
    scales = np.zeros((1, 8), np.uint16)
    scales[0, lane] = h
    _, _, q16, bad = dequant(qweight, qzeros, scales, 1)
    return int(q16[0, lane]), int(bad[0, lane])


# ---------------------------------------------------------------- GEMV
def gemv_fp32(x, qweight, qzeros, scales_bits, bias_bits=None, G=128, threads=1,
              n_range=None):
    """FP32Model.linear over M rows (C restatement, bit-exact).

    x: float32-representable [M, K] (fp16 inputs are exact); returns float32 [M, N].
    """
    x = _c(np.atleast_2d(x), np.float32)
    qweight = _c(qweight, np.uint32)
    qzeros = _c(qzeros, np.uint32)
    scales_bits = _c(scales_bits, np.uint16)
    bias_bits = _c(bias_bits, np.uint16)
    M, K = x.shape
    N = qweight.shape[1] * 8
    if qweight.shape[0] != K:
        raise OracleError("activation width differs from qweight rows")
    y = np.zeros((M, N), np.float32)
    a, b = (0, N) if n_range is None else n_range
    _check(lib().anvilq_oracle_gemv_fp32(_ptr(x), _ptr(qweight), _ptr(qzeros), _ptr(scales_bits),
                                         _ptr(bias_bits), _ptr(y), M, K, N, G, a, b, threads))
    return y


def gemv_fp32_numpy(x, qweight, qzeros, scales_bits, bias_bits=None, G=128):
    """Same arithmetic as ``gemv_fp32`` vectorised over columns with numpy float32.

    numpy float32 multiply and add each round to binary32 (no fusion), and the
    k loop runs in increasing order from +0.0, so this matches FP32Model.linear.
    """
    x = np.atleast_2d(np.asarray(x, np.float32))
    _, w, _, bad = dequant(qweight, qzeros, scales_bits, G)
    if bad.any():
        raise OracleError(_STATUS[-2])
    M, K = x.shape
    y = np.zeros((M, w.shape[1]), np.float32)
    for k in range(K):
        y = y + (x[:, k:k + 1] * w[k][None, :])
    if bias_bits is not None:
        y = y + np.asarray(bias_bits, np.uint16).view(np.float16).astype(np.float32)[None, :]
    if not np.isfinite(y).all():
        raise OracleError(_STATUS[-3])
    return y


def gemv_q16(x_q16, qweight, qzeros, scales_bits, bias_bits=None, G=128, threads=1):
    """FixedModel.linear (Q16.16 in, Q16.16 out, round-away, sat32)."""
    x_q16 = _c(np.atleast_2d(x_q16), np.int32)
    qweight = _c(qweight, np.uint32)
    qzeros = _c(qzeros, np.uint32)
    scales_bits = _c(scales_bits, np.uint16)
    bias_bits = _c(bias_bits, np.uint16)
    M, K = x_q16.shape
    N = qweight.shape[1] * 8
    y = np.zeros((M, N), np.int32)
    _check(lib().anvilq_oracle_gemv_q16(_ptr(x_q16), _ptr(qweight), _ptr(qzeros), _ptr(scales_bits),
                                        _ptr(bias_bits), _ptr(y), M, K, N, G, threads))
    return y


# ---------------------------------------------------------------- attention
def attention_f64(q, keys, values):
    """fp64_reference.py:164-170: q [Hq, D], keys/values [T, Hkv, D]."""
    q = np.asarray(q, np.float64)
    keys = np.asarray(keys, np.float64)
    values = np.asarray(values, np.float64)
    hq, d = q.shape
    hkv = keys.shape[1]
    grouping = hq // hkv
    # query head j uses kv head j // grouping (the reference's np.repeat expansion),
    # evaluated per kv head without materialising the repeated caches
    qg = q.reshape(hkv, grouping, d)
    scores = np.einsum("kgd,tkd->kgt", qg, keys) / np.sqrt(d)
    e = np.exp(scores - scores.max(axis=2, keepdims=True))
    p = e / e.sum(axis=2, keepdims=True)
    return np.einsum("kgt,tkd->kgd", p, values).reshape(hq, d)


# ---- legacy symmetric / asymmetric KV-cache codecs over Q16.16 values --------
# anvil-q4/tests/legacy_reference.py:71-97 (cache_block) and the payload layout
# of :186-203 / anvil-q4/design/SPEC.md:250-262.  Formats: 1 INT8 symmetric,
# 2 INT4 symmetric, 3 INT4 asymmetric.

LEGACY_LIMITS = {1: (127, 25), 2: (7, 29)}    # (largest code, largest exponent)
LEGACY_EMAX = {1: 25, 2: 29, 3: 32}


def _round_away_shift(v: int, e: int) -> int:
    """v / 2^e rounded half away from zero (signed magnitude)."""
    if e == 0:
        return v
    m = (abs(v) + (1 << (e - 1))) >> e
    return -m if v < 0 else m


def _sat32(v: int) -> int:
    return max(-(1 << 31), min((1 << 31) - 1, v))


def legacy_kv_block(values, fmt):
    """One block of Q16.16 values -> (metadata, codes, decoded).

    Symmetric (fmt 1/2): the exponent is the smallest e <= Emax with
    max|v| <= L 2^e (on the unrounded magnitude), codes round v / 2^e half away
    from zero and clamp to [-L, L].  Asymmetric (fmt 3): the first e in 0..32 for
    which the rounded extrema plus a zero point z in [-8, 7] fit [-8, 7]; z is
    the fitting value closest to 0.  Metadata = e | (z & 15) << 8; decoded =
    sat32((code - z) 2^e)."""
    vals = [int(v) for v in values]
    if fmt == 3:
        for e in range(33):
            r = [_round_away_shift(v, e) for v in vals]
            low, high = max(-8, -8 - min(r)), min(7, 7 - max(r))
            if low <= high:
                z = low if low > 0 else (high if high < 0 else 0)
                codes = [x + z for x in r]
                break
        else:
            raise AssertionError("no exponent fits the asymmetric range")
    else:
        limit, emax = LEGACY_LIMITS[fmt]
        a = max(abs(v) for v in vals)
        e = next(k for k in range(emax + 1) if a <= limit << k)
        z = 0
        codes = [min(limit, max(-limit, _round_away_shift(v, e))) for v in vals]
    return e | ((z & 15) << 8), codes, [_sat32((c - z) << e) for c in codes]


def legacy_kv_encode(values, H, D, block, fmt):
    """Rows of H heads x D Q16.16 values [R, H*D] -> payload uint32 [R, H*B*W],
    metadata uint32 [R, H*B], decoded int32 [R, H*D]; B = ceil(D / block) blocks
    per head, W = ceil(block * bits / 32) words per block, codes in ascending
    bytes (INT8) or nibbles (INT4) of each word, padding zero."""
    values = np.asarray(values, np.int64)
    R = values.shape[0]
    bits = 8 if fmt == 1 else 4
    per = 32 // bits
    B = (D + block - 1) // block
    W = (block * bits + 31) // 32
    payload = np.zeros((R, H * B * W), np.uint32)
    meta = np.zeros((R, H * B), np.uint32)
    decoded = np.zeros((R, H * D), np.int32)
    for r in range(R):
        for h in range(H):
            for b in range(B):
                lo, hi = h * D + b * block, h * D + min(D, (b + 1) * block)
                m, codes, dec = legacy_kv_block(values[r, lo:hi], fmt)
                meta[r, h * B + b] = m
                decoded[r, lo:hi] = dec
                padded = codes + [0] * (W * per - len(codes))
                for w in range(W):
                    word = 0
                    for k in range(per):
                        word |= (padded[w * per + k] & ((1 << bits) - 1)) << (k * bits)
                    payload[r, (h * B + b) * W + w] = word
    return payload, meta, decoded


def tree_attention_f64(q, k_cache, v_cache, ancestors, prefix_len):
    """Per-node tree attention: node m attends to rows [0, prefix_len) and the
    rows prefix_len + j of its ancestors j (bit j of ancestors[m]), prefix
    first, then the nodes in ascending order (anvil-q1-ht3/design/SPEC.md:528-538),
    each through attention() of fp64_reference.py:164-170.
    q [M, Hq, D], caches [Tmax, Hkv, D]."""
    out = []
    for m in range(len(q)):
        rows = list(range(prefix_len)) + [prefix_len + j for j in range(32) if (int(ancestors[m]) >> j) & 1]
        out.append(attention_f64(q[m], k_cache[rows], v_cache[rows]))
    return np.stack(out)


def tree_is_valid(ancestors):
    """The ancestor contract of anvil-q1-ht3/design/SPEC.md:528-533: node m sees
    itself, no later node, and the ancestors of each of its ancestors."""
    a = [int(x) & 0xFFFFFFFF for x in ancestors]
    for m, mask in enumerate(a):
        if not (mask >> m) & 1 or mask >> (m + 1):
            return False
        if any((mask >> j) & 1 and a[j] & ~mask for j in range(m)):
            return False
    return True


def attention_fp32(q_bits, k_bits, v_bits):
    """official_weights.py:471-486 FP32 loop for one sequence; inputs are binary16 bits."""
    q_bits = _c(q_bits, np.uint16)
    k_bits = _c(k_bits, np.uint16)
    v_bits = _c(v_bits, np.uint16)
    Hq, D = q_bits.shape
    T, Hkv, _ = k_bits.shape
    out = np.empty((Hq, D), np.float32)
    scratch = np.empty(T, np.float32)
    _check(lib().anvilq_oracle_attention_fp32(_ptr(q_bits), _ptr(k_bits), _ptr(v_bits), _ptr(out),
                                              Hq, Hkv, D, T, _ptr(scratch), 1))
    return out


def decode_attention_f64(q, k_cache, v_cache, seqlens):
    """Batched GQA decode: q [B,Hq,D], caches [B,Tmax,Hkv,D]; sequence b uses positions < seqlens[b]."""
    out = np.empty(q.shape, np.float64)
    for b in range(q.shape[0]):
        T = int(seqlens[b])
        out[b] = attention_f64(q[b], k_cache[b, :T], v_cache[b, :T])
    return out


# ---------------------------------------------------------------- metrics
KV_ESCAPE_MARKER = 0x7FC00000


def kv_int8_encode(bits):
    """Per-head INT8 KV-cache encoding with FP32 escape, restating
    anvil-q4/tests/cache_reference.py:54-83 (format anvil-q4/design/SPEC.md:209-235)
    on float32 bit patterns [..., D] (one head per last axis).

    Ordinary head: scale = fp32(maxabs / 127) (1.0 for an all-+0 head), code =
    clamp(round-half-even(|fp32(v / scale)|), 127) with v's sign, reconstruction
    fp32(code * scale).  A head holding NaN, +-inf or -0.0, or whose scale
    underflows to 0, escapes: metadata 0x7FC00000, codes 0, payload = the values
    with every NaN made 0x7FC00000.  Every step is one IEEE binary32 operation
    (division, round to integer, product), which numpy float32 performs exactly.
    Returns (scale_bits uint32 [...], codes int8 [..., D], recon_bits uint32 [..., D],
    escape_bits uint32 [..., D] (zero for ordinary heads))."""
    bits = np.ascontiguousarray(bits, np.uint32)
    nonfinite = (bits & 0x7F800000) == 0x7F800000
    esc = np.any(nonfinite | (bits == 0x80000000), axis=-1)
    with np.errstate(all="ignore"):
        v = bits.view(np.float32)
        maxabs = np.where(esc[..., None], np.float32(0), np.abs(v)).max(axis=-1).astype(np.float32)
        scale = np.where(maxabs > 0, maxabs / np.float32(127), np.float32(1)).astype(np.float32)
        esc = esc | (scale == 0)
        safe = np.where(esc, np.float32(1), scale).astype(np.float32)
        ratio = (np.where(esc[..., None], np.float32(0), v) / safe[..., None]).astype(np.float32)
        mag = np.minimum(np.rint(np.abs(ratio)), np.float32(127))
        code = np.where(ratio < 0, -mag, mag).astype(np.int8)
        recon = (code.astype(np.float32) * safe[..., None]).astype(np.float32)
    canon = np.where(nonfinite & ((bits & 0x7FFFFF) != 0), np.uint32(KV_ESCAPE_MARKER), bits)
    scale_bits = np.where(esc, np.uint32(KV_ESCAPE_MARKER), scale.view(np.uint32)).astype(np.uint32)
    codes = np.where(esc[..., None], np.int8(0), code).astype(np.int8)
    recon_bits = np.where(esc[..., None], canon, recon.view(np.uint32)).astype(np.uint32)
    escape_bits = np.where(esc[..., None], canon, np.uint32(0)).astype(np.uint32)
    return scale_bits, codes, recon_bits, escape_bits


def kv_int8_decode(scale_bits, codes, escape_bits):
    """Reconstruction of kv_int8_encode's output as float32: fp32(code * scale),
    or the escape payload for marker heads (SPEC.md:221-229)."""
    scale_bits = np.asarray(scale_bits, np.uint32)
    esc = scale_bits == KV_ESCAPE_MARKER
    scale = np.where(esc, np.uint32(0x3F800000), scale_bits).view(np.float32)
    recon = (np.asarray(codes, np.int8).astype(np.float32) * scale[..., None]).astype(np.float32)
    return np.where(esc[..., None], np.asarray(escape_bits, np.uint32).view(np.float32), recon)


def normalized_error(actual, reference):
    """anvil-q1-fp/design/SPEC.md:311-317: max|a-r| / max(1, max|r|) and cosine."""
    a = np.asarray(actual, np.float64).ravel()
    r = np.asarray(reference, np.float64).ravel()
    err = float(np.max(np.abs(a - r))) if a.size else 0.0
    norm = max(1.0, float(np.max(np.abs(r)))) if r.size else 1.0
    na, nr = float(np.linalg.norm(a)), float(np.linalg.norm(r))
    cos = float(a @ r / (na * nr)) if na and nr else None
    return err / norm, cos


# ---------------------------------------------------------------- decode step
class DecodeOracle:
    """Greedy decode in binary64, restating FP32Model.token
    (anvil-q1/tests/official_weights.py:451-509) and QwenFP64.step
    (anvil-q1-fp/tests/fp64_reference.py:210-246) for any model shape
    (L, H, I, QH, KVH, D, G, V, SEQ).

    weights: an object with .shape, .layers[l][p] (AWQ layers, p = 0..6 =
    q,k,v,o,gate,up,down), .norms[("input"|"post", l)], .norms[("final", 0)]
    and .embedding (fp16 [V, H], tied lm_head).  W4 weights are dequantised
    exactly (delta * scale) per layer when used.
    """

    def __init__(self, weights, theta=1e6, eps=1e-6, act16=False):
        """act16: round to binary16 where a W4A16 datapath stores activations in
        binary16 (GEMV inputs, q/k/v, rotated q/k, attention output, gate/up
        outputs); the residual stream and all arithmetic stay binary64."""
        self.w = weights
        self.shape = weights.shape
        self.theta, self.eps = theta, eps
        self.act16 = act16
        self.cache = {}
        self.E = np.asarray(weights.embedding)   # fp16; rows widened to binary64 when used

    def _w(self, l, p):
        lay = self.w.layers[l][p]
        _, wf, _, bad = dequant(lay.qweight, lay.qzeros, lay.scales_bits, lay.group)
        if bad.any():
            raise OracleError(_STATUS[-2])
        b = None if lay.bias is None else np.asarray(lay.bias, np.float64)
        return wf.astype(np.float64), b

    def _linear(self, x, l, p):
        w, b = self._w(l, p)
        y = x @ w
        return y + b if b is not None else y

    def _norm(self, x, gamma):
        return x * np.asarray(gamma, np.float64) / np.sqrt(np.mean(x * x) + self.eps)

    def _rope(self, x, heads, pos):
        _, _, _, _, _, D, _, _, _ = self.shape
        x = x.reshape(heads, D).copy()
        half = D // 2
        ang = pos * np.power(self.theta, -2.0 * np.arange(half) / D)
        c, s = np.cos(ang), np.sin(ang)
        a, b = x[:, :half].copy(), x[:, half:].copy()
        x[:, :half] = a * c - b * s
        x[:, half:] = b * c + a * s
        return x.reshape(-1)

    def _r(self, a):
        return a.astype(np.float16).astype(np.float64) if self.act16 else a

    def step(self, token, pos):
        L, H, I, QH, KVH, D, G, V, SEQ = self.shape
        r = self._r
        x = self.E[token].astype(np.float64)
        for l in range(L):
            h = r(self._norm(x, self.w.norms["input", l]))
            q = r(self._rope(r(self._linear(h, l, 0)), QH, pos))
            k = r(self._rope(r(self._linear(h, l, 1)), KVH, pos))
            v = r(self._linear(h, l, 2))
            self.cache[l, pos] = (k.reshape(KVH, D), v.reshape(KVH, D))
            keys = np.stack([self.cache[l, t][0] for t in range(pos + 1)])
            vals = np.stack([self.cache[l, t][1] for t in range(pos + 1)])
            ctx = r(attention_f64(q.reshape(QH, D), keys, vals).reshape(-1))
            x = x + self._linear(ctx, l, 3)
            h = r(self._norm(x, self.w.norms["post", l]))
            g, u = r(self._linear(h, l, 4)), r(self._linear(h, l, 5))
            silu = g / (1.0 + np.exp(-g))
            x = x + self._linear(r(silu * u), l, 6)
        h = self._norm(x, self.w.norms["final", 0])
        # vocabulary in chunks, as fp64_reference.py:238-242 does, so the binary64
        # embedding never exists in full
        logits = np.empty(self.E.shape[0], np.float64)
        for r in range(0, self.E.shape[0], 8192):
            logits[r:r + 8192] = self.E[r:r + 8192].astype(np.float64) @ h
        return logits


def greedy(logits):
    """Lowest index among the maxima (anvil-q4/tests/transformer_reference.py:212-217)."""
    logits = np.asarray(logits)
    return int(np.flatnonzero(logits == logits.max())[0])
