"""Array-backed checkpoint with the reference's duck-typed checkpoint interface.

The reference's golden models read weights one scalar at a time through a
checkpoint object exposing ``resolve``, ``half`` and ``bus``
(anvil-q1/tests/official_weights.py:320-356).  ``ArrayCheckpoint`` offers the
same three methods over in-memory AWQ arrays, so the reference's
``FP32Model(checkpoint, shape).linear(x, layer, projection)`` and this
package's ``GpuLinear(checkpoint, shape).linear(...)`` consume identical bytes.
It also exposes whole tensors (``arrays``) for the GPU path, which cannot
afford scalar access.

Model kinds follow the reference's public address map
(official_weights.py:332-353): 1 qweight, 2 qzeros, 3 scales, 4 bias.
"""
from __future__ import annotations

import struct

import numpy as np

from .synthetic import AwqLayer

PROJECTIONS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
               "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


class CheckpointError(ValueError):
    """Mirrors the reference's CheckpointError (official_weights.py:37)."""


class ArrayCheckpoint:
    def __init__(self, layers: dict, embedding=None, norms=None):
        """layers: {(layer, projection): AwqLayer}; embedding fp16 [V, H] (kind 0,
        also the tied lm_head); norms: {("input", layer) | ("post", layer) | ("final", 0): fp16 [H]}
        (kinds 5, 6, 7)."""
        self.layers = dict(layers)
        self.embedding = embedding
        self.norms = dict(norms or {})

    # -- reference interface (official_weights.py:320-356) --------------------
    @staticmethod
    def resolve(kind, layer, projection, row, col):
        if not all(type(v) is int and v >= 0 for v in (kind, layer, projection, row, col)):
            raise CheckpointError("invalid public model address")
        if kind == 0:
            if layer or projection:
                raise CheckpointError("embedding unused address fields")
            return (0, 0, 0), (row, col)
        if kind in (5, 6, 7):
            if projection or row or (kind == 7 and layer):
                raise CheckpointError("norm unused address fields")
            return (kind, layer, 0), (col,)
        if kind not in (1, 2, 3, 4):
            raise CheckpointError(f"not an array checkpoint model kind: {kind}")
        if kind == 4:
            if row != 0:
                raise CheckpointError("bias unused row")
            return (4, layer, projection), (col,)
        return (kind, layer, projection), (row, col)

    def _array(self, name):
        kind, layer, projection = name
        if kind == 0:
            if self.embedding is None:
                raise CheckpointError("checkpoint has no embedding")
            return self.embedding
        if kind in (5, 6, 7):
            key = {5: ("input", layer), 6: ("post", layer), 7: ("final", 0)}[kind]
            try:
                return self.norms[key]
            except KeyError as exc:
                raise CheckpointError(f"no norm {key}") from exc
        try:
            t = self.layers[layer, projection]
        except KeyError as exc:
            raise CheckpointError(f"no tensor for layer {layer} projection {projection}") from exc
        a = (t.qweight, t.qzeros, t.scales, t.bias)[kind - 1]
        if a is None:
            raise CheckpointError("projection has no bias")
        return a

    def raw(self, name, coordinate):
        a = self._array(name)
        coordinate = tuple(int(c) for c in coordinate)
        # whole-element coordinates inside the tensor only (numpy would wrap negatives)
        if len(coordinate) != a.ndim or any(not 0 <= c < n for c, n in zip(coordinate, a.shape)):
            raise CheckpointError("tensor coordinate out of bounds")
        v = a[coordinate]
        return int(v.view(np.uint32)) if a.dtype == np.int32 else int(v.view(np.uint16))

    def half(self, name, coordinate):
        # official_weights.py half(): the tensor must be F16
        if self._array(name).dtype != np.float16:
            raise CheckpointError(f"{name} is not an F16 tensor")
        value = struct.unpack("<e", struct.pack("<H", self.raw(name, coordinate)))[0]
        if not np.isfinite(value):
            raise CheckpointError(f"nonfinite F16 {name}{tuple(coordinate)}")
        return value

    def bus(self, kind, layer, projection, row, col):
        return self.raw(*self.resolve(kind, layer, projection, row, col))

    # -- whole-tensor access for the GPU path --------------------------------
    def arrays(self, layer, projection) -> AwqLayer:
        try:
            return self.layers[layer, projection]
        except KeyError as exc:
            raise CheckpointError(f"no tensor for layer {layer} projection {projection}") from exc


def output_width(shape, projection):
    """official_weights.py:419-421: output count of a projection for a model shape."""
    _, h, intermediate, _, kvheads, d, _, _, _ = shape
    return kvheads * d if projection in (1, 2) else intermediate if projection in (4, 5) else h


def gemv_shape(K, N, G, projection=4):
    """A model shape tuple (L,H,I,QH,KVH,D,G,V,SEQ) under which `projection` maps K -> N."""
    if projection in (4, 5):
        return (1, K, N, 1, 1, 1, G, 1, 1)
    if projection in (0, 3):
        return (1, N, 8, 1, 1, 1, G, 1, 1)
    if projection == 6:
        return (1, N, K, 1, 1, 1, G, 1, 1)
    return (1, K, 8, 1, 1, N, G, 1, 1)  # k/v: kvheads * d = N
