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
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
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
