"""GPU drop-ins with the call signatures of the reference's Python golden models.

* ``GpuLinear(checkpoint, shape).linear(x, layer, projection)`` mirrors
  ``FP32Model(checkpoint, shape).linear`` (anvil-q1/tests/official_weights.py:400-437):
  same checkpoint object, same model shape tuple (L,H,I,QH,KVH,D,G,V,SEQ), same
  projection numbering (0..6 = q,k,v,o,gate,up,down), bias added for q/k/v,
  list of floats out, and a CheckpointError-style exception on an invalid
  scale.  Activations are rounded to binary16 (the W4A16 contract).
* ``GpuLinear(...).linear_q16(x_q16, layer, projection)`` is the integer model's
  projection (the ``linear`` inside FixedModel.token, official_weights.py:592-612):
  Q16.16 ints in and out, bit-identical.
* ``dequant(qw, qz, h, lane)`` mirrors verify.dequant (anvil-q1/tests/verify.py:241-250)
  for one lane of one word, computed on the GPU by the GEMM kernels' unpack.
* ``pack(values)`` mirrors verify.pack (verify.py:252-253).
* ``encode_head(values)`` mirrors cache_reference.encode_head
  (anvil-q4/tests/cache_reference.py:54-71): the per-head INT8 KV encoding with
  FP32 escape, encoded on the GPU by the cache-store kernel.
* ``cache_block(values, cache_format)`` mirrors legacy_reference.cache_block
  (anvil-q4/tests/legacy_reference.py:71-92): the legacy INT8/INT4 codecs of
  the Q16.16 datapath, encoded and decoded on the GPU.
* ``attention(q, keys, values)`` mirrors fp64_reference.attention
  (anvil-q1-fp/tests/fp64_reference.py:164-170): numpy in, numpy out, on the
  decode-attention kernel.
* ``pack_lanes(codes)`` / ``unpack_lanes(words, outputs)`` mirror
  awq_prepare.pack_lanes / unpack_lanes (anvil-q1-fp/tests/awq_prepare.py:84-99)
  on numpy arrays, packed and unpacked on the GPU.
* ``GpuModel(checkpoint, shape).token(token, position, new_sequence)`` mirrors
  FP32Model.token (anvil-q1/tests/official_weights.py:451-509): one decode step
  of the device-resident decoder, the logits returned as a list.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops, synthetic
from ._lib import AnvilqError
from .checkpoint import CheckpointError, output_width


def _layer_arrays(checkpoint, layer, projection, shape):
    """Whole AWQ tensors of one projection from a checkpoint object.

    Accepts ArrayCheckpoint (``arrays``) or the reference's safetensors-backed
    Checkpoint (``data``/``base``/``tensors`` descriptors, official_weights.py:141-200).
    """
    if hasattr(checkpoint, "arrays"):
        t = checkpoint.arrays(layer, projection)
        return t.qweight, t.qzeros, t.scales, t.bias
    if all(hasattr(checkpoint, a) for a in ("data", "base", "tensors", "resolve")):
        out = []
        for kind in (1, 2, 3, 4):
            if kind == 4 and projection >= 3:
                out.append(None)
                continue
            name, _ = checkpoint.resolve(kind, layer, projection, 0, 0)
            d = checkpoint.tensors[name]
            dtype = np.int32 if d["dtype"] == "I32" else np.float16
            count = (d["end"] - d["start"]) // d["width"]
            a = np.frombuffer(checkpoint.data, dtype=dtype, count=count,
                              offset=checkpoint.base + d["start"]).reshape(d["shape"])
            out.append(a)
        return tuple(out)
    raise CheckpointError("checkpoint exposes neither arrays() nor safetensors descriptors")


class GpuLinear:
    """``FP32Model.linear`` on the GPU, over the same checkpoint object."""

    def __init__(self, checkpoint, shape, device="cuda"):
        self.checkpoint, self.shape = checkpoint, shape
        self.device = torch.device(device)
        self._cache = {}

    def weights(self, layer, projection):
        key = (layer, projection)
        w = self._cache.get(key)
        if w is None:
            qweight, qzeros, scales, bias = _layer_arrays(self.checkpoint, layer, projection, self.shape)
            to = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(self.device)
            w = (to(qweight), to(qzeros), to(scales), to(bias) if projection < 3 else None)
            no = output_width(self.shape, projection)
            if w[0].shape[1] * 8 != no:
                raise CheckpointError("projection width differs from the model shape")
            self._cache[key] = w
        return w

    def linear(self, x, layer, projection, exact=False):
        qweight, qzeros, scales, bias = self.weights(layer, projection)
        group = self.shape[6]
        xt = torch.tensor(np.asarray(x, np.float32).astype(np.float16), device=self.device)
        try:
            if exact:
                y = ops.gemm_exact(xt, qweight, qzeros, scales, bias, group)
            else:
                y = ops.gemm(xt, qweight, qzeros, scales, bias, group)
            ops.raise_device_errors(self.device)
        except AnvilqError as exc:
            raise CheckpointError(str(exc)) from exc
        return [float(v) for v in y.float().cpu().numpy()]

    def linear_q16(self, x_q16, layer, projection):
        """The integer model's projection (the ``linear`` of FixedModel.token,
        official_weights.py:592-612): Q16.16 int activations in, Q16.16 ints out,
        exact sum of x * (q - z) * round_away(scale * 2^16), bias * 2^16 added for
        q/k/v, round-half-away >> 16, saturated to int32; bit-identical."""
        qweight, qzeros, scales, bias = self.weights(layer, projection)
        xt = torch.tensor(np.asarray(x_q16, np.int64).astype(np.int32), device=self.device)
        try:
            y = ops.gemm_q16(xt, qweight, qzeros, scales, bias, self.shape[6])
            ops.raise_device_errors(self.device)
        except AnvilqError as exc:
            raise CheckpointError(str(exc)) from exc
        return [int(v) for v in y.cpu().numpy().reshape(-1)]


SHIFTS = (0, 16, 4, 20, 8, 24, 12, 28)


def pack(values):
    """verify.pack: value i -> bit shift SHIFTS[i] (host-side, exact integer)."""
    return sum((int(v) & 15) << s for v, s in zip(values, SHIFTS))


def dequant(qw, qz, h, lane, device="cuda"):
    """verify.dequant signature -> (Q16.16 weight, invalid).

    The signed delta q - z comes from the GPU dequantiser (the GEMM kernels'
    in-register unpack); the Q16.16 scale round_away(scale * 2^16) is formed on
    the host from the binary16 fields with integer arithmetic, and the result
    is their product, as in verify.py:241-250.
    """
    dev = torch.device(device)
    qweight = torch.from_numpy(np.array([[qw & 0xFFFFFFFF]], np.uint32).view(np.int32)).to(dev)
    qzeros = torch.from_numpy(np.array([[qz & 0xFFFFFFFF]], np.uint32).view(np.int32)).to(dev)
    sc = np.zeros((1, 8), np.uint16)
    sc[0, lane] = h
    scales = torch.from_numpy(sc.view(np.float16)).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    delta, _ = ops.dequant(qweight, qzeros, scales, 1, dev_err=err)
    # invalid is per lane; recompute the lane's flag exactly as the kernel does
    e = (h >> 10) & 31
    invalid = int(e == 31 or ((h & 0x8000) and (h & 0x7FFF)))
    if invalid:
        return 0, 1
    d = int(delta[0, lane].item())
    # exact Q16.16 scale: round_away(scale * 2^16) from the binary16 fields
    sign = -1 if h & 0x8000 else 1
    significand = (h & 1023) if e == 0 else (h & 1023) + 1024
    power = -24 if e == 0 else e - 25
    num, den = significand << max(power + 16, 0), 1 << max(-(power + 16), 0)
    s16 = (2 * num + den) // (2 * den)
    return d * sign * s16, 0


ESCAPE_MARKER = 0x7FC00000


def encode_head(values, device="cuda"):
    """cache_reference.encode_head signature: binary32 bit patterns of one
    (token, kv head) row -> (scale bits or the escape marker, codes as unsigned
    bytes, reconstructed binary32 bit patterns).  Codes and scale come from the
    GPU encoder (anvilq_kv_int8_store); an ordinary row reconstructs as
    fp32(code * scale), an escaped row as its canonical payload."""
    bits = np.array([int(v) & 0xFFFFFFFF for v in values], np.uint32)
    D = bits.size
    dev = torch.device(device)
    src = torch.from_numpy(bits.view(np.float32).reshape(1, 1, 1, D).copy()).to(dev)
    codes = torch.zeros((1, 1, 1, D), dtype=torch.int8, device=dev)
    meta = torch.zeros((1, 1, 1), dtype=torch.int32, device=dev)
    escape = torch.zeros((1, 1, 1, D), dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.kv_int8_store(src, codes, meta, escape=escape, dev_err=err)
    if int(err.item()):
        raise AnvilqError(f"kv_int8_store device error bits 0x{int(err.item()):x}")
    scale = int(meta.cpu().numpy().view(np.uint32)[0, 0, 0])
    c = codes.cpu().numpy().reshape(D)
    if scale == ESCAPE_MARKER:
        payload = escape.cpu().numpy().reshape(D).view(np.uint32)
        return scale, [int(x) & 255 for x in c], [int(x) for x in payload]
    s32 = np.array([scale], np.uint32).view(np.float32)[0]
    recon = (c.astype(np.float32) * s32).astype(np.float32).view(np.uint32)
    return scale, [int(x) & 255 for x in c], [int(x) for x in recon]


def cache_block(values, cache_format, device="cuda"):
    """legacy_reference.cache_block signature: one block of Q16.16 ints and the
    cache format (1 INT8 symmetric, 2 INT4 symmetric, 3 INT4 asymmetric) ->
    (metadata, codes, decoded), encoded and decoded on the GPU
    (anvilq_legacy_kv_encode / anvilq_legacy_kv_decode)."""
    if cache_format not in (1, 2, 3):
        raise ValueError("cache_format must be 1, 2 or 3")
    n = len(values)
    if not 1 <= n <= 64:
        raise ValueError("a block holds 1..64 values")
    dev = torch.device(device)
    x = torch.tensor([[int(v) for v in values]], dtype=torch.int32, device=dev)
    payload, meta = ops.legacy_kv_encode(x, 1, n, n, cache_format)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    decoded = ops.legacy_kv_decode(payload, meta, 1, n, n, cache_format, dev_err=err)
    if int(err.item()):
        raise AnvilqError(f"legacy cache decode device error bits 0x{int(err.item()):x}")
    bits = 8 if cache_format == 1 else 4
    words = payload.cpu().numpy().view(np.uint32).reshape(-1)
    per = 32 // bits
    codes = []
    for i in range(n):
        raw = (int(words[i // per]) >> ((i % per) * bits)) & ((1 << bits) - 1)
        codes.append(raw - (1 << bits) if raw >= 1 << (bits - 1) else raw)
    return int(meta.cpu().numpy().view(np.uint32)[0, 0]), codes, [int(v) for v in decoded.cpu().numpy()[0]]


def attention(q, keys, values, device="cuda"):
    """fp64_reference.attention(q, keys, values): q [Hq, D], keys / values
    [T, Hkv, D] -> [Hq, D] as a float64 numpy array, query head j attending
    with kv head j // (Hq / Hkv).  Computed by the decode-attention kernel
    (anvilq_gqa_decode) over the inputs rounded to binary16, the fp16 KV
    cache of the W4A16 datapath; scores and softmax in fp32.  Head dims 64
    and 128 are supported; others raise ValueError."""
    q = np.asarray(q)
    keys = np.asarray(keys)
    values = np.asarray(values)
    if q.ndim != 2 or keys.ndim != 3 or values.shape != keys.shape:
        raise ValueError("q [Hq, D] and keys / values [T, Hkv, D] expected")
    hq, d = q.shape
    t, hkv, dk = keys.shape
    if dk != d or t < 1 or hkv < 1 or hq % hkv:
        raise ValueError("q, keys and values disagree on head dim, kv heads or length")
    dev = torch.device(device)
    f16 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float16)).to(dev)
    out = ops.gqa_decode(f16(q)[None], f16(keys)[None], f16(values)[None],
                         torch.tensor([t], dtype=torch.int32, device=dev))
    ops.raise_device_errors(dev)
    return out[0].double().cpu().numpy()


def pack_lanes(codes, device="cuda"):
    """awq_prepare.pack_lanes(codes): output-major nibbles uint8 [N, K], N % 8 == 0,
    -> little-endian uint32 [K, N / 8] with lane i of word w holding column 8 w + i
    at bit shift (0, 16, 4, 20, 8, 24, 12, 28)[i]."""
    codes = np.asarray(codes)
    if codes.ndim != 2 or codes.shape[0] % 8 or codes.size == 0 or (codes < 0).any() or (codes > 15).any():
        raise ValueError("invalid nibble array")
    t = torch.from_numpy(np.ascontiguousarray(codes, np.uint8)).to(torch.device(device))
    return ops.pack_lanes(t).cpu().numpy().view("<u4")


def unpack_lanes(words, outputs, device="cuda"):
    """awq_prepare.unpack_lanes(words, outputs): uint32 [K, N / 8] with N == outputs
    -> uint8 [N, K]."""
    words = np.asarray(words)
    if words.ndim != 2 or words.shape[1] * 8 != outputs or words.size == 0:
        raise ValueError("invalid packed output shape")
    t = torch.from_numpy(np.ascontiguousarray(words).astype(np.uint32).view(np.int32)).to(torch.device(device))
    return ops.unpack_lanes(t, int(outputs)).cpu().numpy()


def _f16_tensor(checkpoint, kind, layer):
    """A whole fp16 tensor (embedding, kind 0; norms, kinds 5-7) of a checkpoint."""
    if hasattr(checkpoint, "embedding") and hasattr(checkpoint, "norms"):
        if kind == 0:
            return checkpoint.embedding
        return checkpoint.norms[{5: ("input", layer), 6: ("post", layer), 7: ("final", 0)}[kind]]
    name, _ = checkpoint.resolve(kind, layer if kind != 7 else 0, 0, 0, 0)
    d = checkpoint.tensors[name]
    count = (d["end"] - d["start"]) // d["width"]
    return np.frombuffer(checkpoint.data, dtype=np.float16, count=count,
                         offset=checkpoint.base + d["start"]).reshape(d["shape"])


class GpuModel:
    """``FP32Model(checkpoint, shape)`` for the decode step: ``token(token,
    position, new_sequence)`` returns the logits after the token, as
    FP32Model.token does, computed by one step of the device-resident decoder
    (W4A16 projections with binary16 activations, fp16 KV cache, tied fp16
    lm_head).  Positions must follow one another from 0 (a new sequence
    restarts at 0); a violated bound or a device error raises CheckpointError,
    as the reference's demand() does."""

    def __init__(self, checkpoint, shape, device="cuda"):
        from .decoder import Decoder, DecoderWeights
        self.shape = tuple(int(v) for v in shape)
        L, H, I, QH, KVH, D, G, V, SEQ = self.shape
        layers = []
        for l in range(L):
            projs = {}
            for p in range(7):
                qweight, qzeros, scales, bias = _layer_arrays(checkpoint, l, p, self.shape)
                projs[p] = synthetic.AwqLayer(np.asarray(qweight), np.asarray(qzeros), np.asarray(scales),
                                              None if bias is None else np.asarray(bias), G)
            layers.append(projs)
        norms = {("input", l): _f16_tensor(checkpoint, 5, l) for l in range(L)}
        norms.update({("post", l): _f16_tensor(checkpoint, 6, l) for l in range(L)})
        norms["final", 0] = _f16_tensor(checkpoint, 7, 0)
        weights = DecoderWeights(self.shape, layers, norms, _f16_tensor(checkpoint, 0, 0))
        self.decoder = Decoder(weights, device, max_seq=SEQ, keep_logits=True)
        self.next_position = 0

    def token(self, token, position, new_sequence=False):
        L, H, I, QH, KVH, D, G, V, SEQ = self.shape
        token, position = int(token), int(position)
        if not (0 <= token < V and 0 <= position < min(SEQ, self.decoder.max_seq)):
            raise CheckpointError("token or position outside the model shape")
        if new_sequence:
            if position != 0:
                raise CheckpointError("a new sequence starts at position 0")
            self.next_position = 0
        if position != self.next_position:
            raise CheckpointError("positions must follow one another")
        d = self.decoder
        try:
            d.set_position(token, position)
            d.step()
            d.stream.synchronize()
            d.check_errors()
        except AnvilqError as exc:
            raise CheckpointError(str(exc)) from exc
        self.next_position += 1
        return [float(v) for v in d.logits.cpu().numpy()]
