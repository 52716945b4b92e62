"""Batch-1 greedy decode of a Qwen2-architecture W4A16 AWQ model on B200.

The step follows FP32Model.token (anvil-q1/tests/official_weights.py:451-509)
and QwenFP64.step (anvil-q1-fp/tests/fp64_reference.py:210-246):

    x = E[token]                                   fp32 residual stream
    per layer:  h = rmsnorm(x); q,k,v = h W_qkv + b; rope(q, k); cache k, v
                a = attention(q, K, V); x += a W_o
                h = rmsnorm(x); g, u = h W_gate, h W_up; x += (silu(g) u) W_down
    logits = rmsnorm(x) E^T;  token = argmax (lowest index on ties)

Kernels per token, fused step (fused=True, where the shape allows): one
persistent kernel runs every layer (anvilq_decode_layers: the five phases of a
layer as roles of one CTA per SM, synchronised by producer counters, each CTA's
next-layer weights streamed into shared memory ahead of use), then the
lm_head/argmax and the token commit -- 3 launches.  Per-kernel step (the
default): 1 embedding + per layer 5 (QKV GEMV with RMSNorm
prologue, bias and a RoPE + KV-append epilogue, attention, O GEMV with residual
epilogue, gate/up GEMV with RMSNorm prologue, down GEMV with SiLU-product
prologue and residual epilogue) + the lm_head/argmax + the token commit.  q/k/v and gate/up are each one GEMV
over weights concatenated along N at load time (AWQ packs 8 columns per word,
so concatenating N-blocks of multiples of 8 keeps the layout).  Token, position
and caches live on the device, so one CUDA graph replays every step.

Weights here are synthetic (seeded) with the reference's value distributions;
no checkpoint is available offline.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, ops, synthetic
from .checkpoint import ArrayCheckpoint

# (L, H, I, QH, KVH, D, G, V, SEQ) as in official_weights.py:21 DEFAULT_SHAPE
QWEN05B_SHAPE = (24, 896, 4864, 14, 2, 64, 128, 151936, 32768)
# a Llama-7B-class decoder in the same tuple: 32 layers, hidden 4096, intermediate
# 11008, 32 heads of 128 (no grouping), vocabulary 32000; no q/k/v bias
LLAMA7B_SHAPE = (32, 4096, 11008, 32, 32, 128, 128, 32000, 4096)
ROPE_THETA = 1_000_000.0
RMS_EPS = 1e-6
FLAG_OVERLAP = 1   # ANVILQ_GEMM_OVERLAP_PRIOR


@dataclass
class DecoderWeights:
    """Per-layer AWQ projections in the reference's numbering (0..6 = q,k,v,o,gate,up,down)."""
    shape: tuple
    layers: list                      # [L] of dict projection -> AwqLayer
    norms: dict = field(default_factory=dict)   # ("input", l) / ("post", l) / ("final", 0) -> fp16 [H]
    embedding: np.ndarray | None = None         # fp16 [V, H], tied lm_head

    def checkpoint(self) -> ArrayCheckpoint:
        flat = {(l, p): lay for l, projs in enumerate(self.layers) for p, lay in projs.items()}
        return ArrayCheckpoint(flat, embedding=self.embedding, norms=self.norms)


def synthetic_weights(shape=QWEN05B_SHAPE, seed: int = 17, qkv_bias: bool = True) -> DecoderWeights:
    """Random-init weights of the given shape.  W4 tensors use the benchmark
    value distributions (u4 uniform, scales |N(0,1)|*0.01+1e-3); biases N(0,1)
    (q/k/v only, and only with qkv_bias); norm weights 1 + 0.1 N(0,1);
    embedding 0.5 N(0,1); all fp16."""
    L, H, I, QH, KVH, D, G, V, _ = shape
    rng = np.random.default_rng(seed)
    b = qkv_bias
    dims = ((H, QH * D, b), (H, KVH * D, b), (H, KVH * D, b), (QH * D, H, False),
            (H, I, False), (H, I, False), (I, H, False))
    layers = []
    norms = {}
    for l in range(L):
        layers.append({p: synthetic.awq_layer(K, N, G, rng=rng, bias=b) for p, (K, N, b) in enumerate(dims)})
        for which in ("input", "post"):
            norms[which, l] = (1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32)).astype(np.float16)
    norms["final", 0] = (1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32)).astype(np.float16)
    embedding = (0.5 * rng.standard_normal((V, H), dtype=np.float32)).astype(np.float16)
    return DecoderWeights(shape, layers, norms, embedding)


def device_synthetic_weights(shape, device, seed: int = 17, qkv_bias: bool = True) -> DecoderWeights:
    """``synthetic_weights`` drawn on the device (a seeded torch generator, the
    same value distributions): the tensors are torch tensors, for model sizes
    whose host-side generation would take minutes (7B-class)."""
    L, H, I, QH, KVH, D, G, V, _ = shape
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    dims = ((H, QH * D, qkv_bias), (H, KVH * D, qkv_bias), (H, KVH * D, qkv_bias), (QH * D, H, False),
            (H, I, False), (H, I, False), (I, H, False))
    layers = []
    norms = {}
    gamma = lambda: (1.0 + 0.1 * torch.randn(H, generator=gen, device=dev)).half()
    for l in range(L):
        layers.append({p: synthetic.AwqLayer(*synthetic.device_awq_layer(K, N, G, gen, dev, bias=b), G)
                       for p, (K, N, b) in enumerate(dims)})
        norms["input", l] = gamma()
        norms["post", l] = gamma()
    norms["final", 0] = gamma()
    embedding = (0.5 * torch.randn((V, H), generator=gen, device=dev)).half()
    return DecoderWeights(shape, layers, norms, embedding)


def _concat(layers):
    """AWQ layers with equal K and G concatenated along N (numpy arrays or torch tensors)."""
    if isinstance(layers[0].qweight, torch.Tensor):
        cat = lambda name: torch.cat([getattr(l, name) for l in layers], dim=1)
        bias = None if layers[0].bias is None else torch.cat([l.bias for l in layers])
        return synthetic.AwqLayer(cat("qweight"), cat("qzeros"), cat("scales"), bias, layers[0].group)
    cat = lambda name: np.concatenate([getattr(l, name) for l in layers], axis=1)
    bias = None
    if layers[0].bias is not None:
        bias = np.concatenate([l.bias for l in layers])
    return synthetic.AwqLayer(cat("qweight"), cat("qzeros"), cat("scales"), bias, layers[0].group)


class Decoder:
    """Device-resident greedy decoder; ``step`` enqueues one token, ``capture``
    records it as a CUDA graph that every later step replays."""

    def __init__(self, weights: DecoderWeights, device="cuda", max_seq: int = 2048, keep_logits: bool = False,
                 fused: bool | None = False, mlp: bool = False, gu_act: bool = True):
        """fused: run the layers as one persistent kernel (True: require it;
        None: when the shape allows it; False, the default: one kernel per
        operation, the faster path on B200 at the 0.5B shape).
        mlp: on the per-operation path, run each layer's MLP (gate/up and down)
        as one launch (anvilq_w4a16_mlp) instead of two fused GEMVs.
        gu_act: the gate/up GEMV stores fp16(silu(g) u) itself (its columns
        interleaved at load time) and the down GEMV reads it as fp16 input --
        bit-identical to the gate/up output followed by the SiLU prologue, and
        faster (the prologue's per-row exp left the down GEMV's tile loop)."""
        self.shape = weights.shape
        L, H, I, QH, KVH, D, G, V, SEQ = self.shape
        self.max_seq = min(max_seq, SEQ)
        self.device = torch.device(device)
        dev = self.device
        t = lambda a: (None if a is None else a.to(dev).contiguous() if isinstance(a, torch.Tensor)
                       else torch.from_numpy(np.ascontiguousarray(a)).to(dev))
        self.layers = []
        for projs in weights.layers:
            qkv = _concat([projs[0], projs[1], projs[2]])
            gu = _concat([projs[4], projs[5]])
            self.layers.append({
                "qkv": tuple(t(a) for a in (qkv.qweight, qkv.qzeros, qkv.scales, qkv.bias)),
                "o": tuple(t(a) for a in (projs[3].qweight, projs[3].qzeros, projs[3].scales)) + (None,),
                "gu": tuple(t(a) for a in (gu.qweight, gu.qzeros, gu.scales)) + (None,),
                "down": tuple(t(a) for a in (projs[6].qweight, projs[6].qzeros, projs[6].scales)) + (None,),
            })
        self.gamma_in = [t(weights.norms["input", l]) for l in range(L)]
        self.gamma_post = [t(weights.norms["post", l]) for l in range(L)]
        self.gamma_final = t(weights.norms["final", 0])
        self.embedding = t(weights.embedding)
        self.k_cache = torch.zeros((L, self.max_seq, KVH, D), dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.x = torch.zeros(H, dtype=torch.float32, device=dev)
        self.q = torch.empty((1, QH, D), dtype=torch.float16, device=dev)
        self.attn = torch.empty((1, QH, D), dtype=torch.float16, device=dev)
        self.gu = torch.empty(2 * I, dtype=torch.float16, device=dev)
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.seqlen = torch.ones(1, dtype=torch.int32, device=dev)
        self.key = torch.zeros(1, dtype=torch.int64, device=dev)
        self.logits = torch.empty(V, dtype=torch.float32, device=dev) if keep_logits else None
        self.dev_err = torch.zeros(1, dtype=torch.int32, device=dev)
        lib = _lib.load()
        ws_bytes = max(lib.anvilq_w4a16_gemm_workspace_size(1, K, N, G)
                       for K, N in ((H, (QH + 2 * KVH) * D), (QH * D, H), (H, 2 * I), (I, H)))
        ws_bytes = max(ws_bytes, lib.anvilq_gqa_decode_workspace_size(1, QH, KVH, D, self.max_seq))
        self.workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        fused_ws = lib.anvilq_decode_layers_workspace_size(L, H, I, QH, KVH, D, G, self.max_seq)
        if fused and fused_ws == 0:
            raise ValueError("the fused decode step does not support this model shape")
        self.fused = fused is not False and fused_ws > 0
        if self.fused:
            self.fused_ws = torch.zeros(fused_ws, dtype=torch.uint8, device=dev)
            s = torch.cuda.current_stream(dev).cuda_stream

            def blocked(t, block):
                """The tensor's column blocks of `block` elements one after another (anvilq_block_columns)."""
                out = torch.empty_like(t)
                _lib.check(lib.anvilq_block_columns(t.data_ptr(), out.data_ptr(), t.shape[0], t.shape[1], block,
                                                    t.element_size(), s), "anvilq_block_columns")
                return out

            def blocked_awq(w, words):   # qweight, qzeros in blocks of `words` words, scales of 8 words
                return (blocked(w[0], words), blocked(w[1], words), blocked(w[2], 8 * words), w[3])

            def interleaved_gu(w):
                """gate|up ([.., 2 I / 8] words, [.., 2 I] scales) as 32-column units u, each
                row holding the gate's 4 words then the up's 4 (whole AWQ words move)."""
                qw, qz, sc = w[0], w[1], w[2]
                unit = lambda t, per: t.view(t.shape[0], 2, I // 32, per).permute(2, 0, 1, 3).contiguous()
                return (unit(qw, 4), unit(qz, 4), unit(sc, 32), None)

            p = lambda t: 0 if t is None else t.data_ptr()
            rows = []
            self.blocked_layers = []
            for l, w in enumerate(self.layers):   # anvilq_decode_layer, field by field
                b = {"qkv": blocked_awq(w["qkv"], D // 8), "o": blocked_awq(w["o"], 4),
                     "gu": interleaved_gu(w["gu"]), "down": blocked_awq(w["down"], 4)}
                self.blocked_layers.append(b)
                rows.append([p(a) for a in b["qkv"]] + [p(a) for a in b["o"][:3]] + [p(a) for a in b["gu"][:3]]
                            + [p(a) for a in b["down"][:3]] + [p(self.gamma_in[l]), p(self.gamma_post[l]),
                                                               p(self.k_cache[l]), p(self.v_cache[l])])
            self.layer_table = torch.tensor(rows, dtype=torch.int64, device=dev)
            torch.cuda.synchronize(dev)
        self.mlp = bool(mlp) and not self.fused
        self.gu_act = bool(gu_act) and not self.fused and not self.mlp
        if self.mlp or self.gu_act:   # gate/up columns unit-interleaved (anvilq_w4a16_mlp's order)
            self.mlp_gu = [ops.mlp_interleave(*w["gu"][:3]) for w in self.layers]
        if self.mlp:
            self.mlp_ws = torch.zeros(lib.anvilq_w4a16_mlp_workspace_size(H, I, G), dtype=torch.uint8, device=dev)
        if self.gu_act:
            self.act = torch.empty(I, dtype=torch.float16, device=dev)
        self.stream = torch.cuda.Stream(dev)
        self.graph = None
        # host staging for the end-to-end path
        self.token_in = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.token_out = torch.zeros(1, dtype=torch.int32).pin_memory()

    # -- one token -----------------------------------------------------------
    def _gemv(self, w, x, x_mode, gamma, y, y_mode, K, N):
        lib = _lib.load()
        qweight, qzeros, scales, bias = w
        _lib.check(lib.anvilq_w4a16_gemv_fused(
            x.data_ptr(), x_mode, None if gamma is None else gamma.data_ptr(), RMS_EPS,
            qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(), None if bias is None else bias.data_ptr(),
            y.data_ptr(), y_mode, K, N, self.shape[6], self.workspace.data_ptr(), self.workspace.numel(),
            self.dev_err.data_ptr(), FLAG_OVERLAP, self.stream.cuda_stream), "anvilq_w4a16_gemv_fused")

    def _qkv_rope(self, l, w):
        """QKV projection of layer l with RoPE and the KV-cache append in its epilogue."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        lib = _lib.load()
        qweight, qzeros, scales, bias = w["qkv"]
        _lib.check(lib.anvilq_w4a16_gemv_qkv_rope(
            self.x.data_ptr(), 1, self.gamma_in[l].data_ptr(), RMS_EPS, qweight.data_ptr(), qzeros.data_ptr(),
            scales.data_ptr(), None if bias is None else bias.data_ptr(), H, G, self.pos.data_ptr(),
            self.q.data_ptr(), self.k_cache[l].data_ptr(), self.v_cache[l].data_ptr(), self.seqlen.data_ptr(),
            QH, KVH, D, self.max_seq, ROPE_THETA, self.workspace.data_ptr(), self.workspace.numel(),
            self.dev_err.data_ptr(), FLAG_OVERLAP, self.stream.cuda_stream), "anvilq_w4a16_gemv_qkv_rope")

    def _mlp_gemvs(self, l, w):
        """Layer l's MLP as two fused GEMVs: gate/up with the SiLU product in its
        epilogue and down on those activations (gu_act), or gate/up to fp16
        [gate | up] and down with the SiLU prologue."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        if self.gu_act:
            self._gemv((*self.mlp_gu[l], None), self.x, 1, self.gamma_post[l], self.act, 2, H, 2 * I)
            self._gemv(w["down"], self.act, 0, None, self.x, 1, I, H)
        else:
            self._gemv(w["gu"], self.x, 1, self.gamma_post[l], self.gu, 0, H, 2 * I)
            self._gemv(w["down"], self.gu, 2, None, self.x, 1, I, H)

    def _mlp(self, l, w):
        """Layer l's MLP in one launch: x += down(silu(gate) up) of RMSNorm(x)."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        gq, gz, gs = self.mlp_gu[l]
        dq, dz, ds = w["down"][:3]
        _lib.check(_lib.load().anvilq_w4a16_mlp(
            self.x.data_ptr(), self.gamma_post[l].data_ptr(), RMS_EPS, gq.data_ptr(), gz.data_ptr(), gs.data_ptr(),
            dq.data_ptr(), dz.data_ptr(), ds.data_ptr(), H, I, G, self.mlp_ws.data_ptr(), self.mlp_ws.numel(),
            self.dev_err.data_ptr(), FLAG_OVERLAP, self.stream.cuda_stream), "anvilq_w4a16_mlp")

    def _layers_fused(self):
        """Every layer of the step as one persistent kernel (anvilq_decode_layers)."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        _lib.check(_lib.load().anvilq_decode_layers(
            self.layer_table.data_ptr(), L, H, I, QH, KVH, D, G, self.max_seq, RMS_EPS, ROPE_THETA,
            self.embedding.data_ptr(), V, self.token.data_ptr(), self.pos.data_ptr(), self.seqlen.data_ptr(),
            self.x.data_ptr(), self.key.data_ptr(), self.fused_ws.data_ptr(), self.fused_ws.numel(),
            self.dev_err.data_ptr(), self.stream.cuda_stream), "anvilq_decode_layers")

    def _enqueue(self, host_io: bool):
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        lib = _lib.load()
        s = self.stream.cuda_stream
        if host_io:
            self.token.copy_(self.token_in, non_blocking=True)
        if self.fused:
            self._layers_fused()
            _lib.check(lib.anvilq_lmhead_argmax(
                self.x.data_ptr(), self.gamma_final.data_ptr(), RMS_EPS, self.embedding.data_ptr(),
                None if self.logits is None else self.logits.data_ptr(), self.key.data_ptr(), H, V, FLAG_OVERLAP,
                s), "anvilq_lmhead_argmax")
            _lib.check(lib.anvilq_argmax_commit(self.key.data_ptr(), self.token.data_ptr(), self.pos.data_ptr(),
                                                FLAG_OVERLAP, s), "anvilq_argmax_commit")
            if host_io:
                self.token_out.copy_(self.token, non_blocking=True)
            return
        _lib.check(lib.anvilq_embed(self.embedding.data_ptr(), self.token.data_ptr(), self.x.data_ptr(), H, V,
                                    self.key.data_ptr(), self.dev_err.data_ptr(), FLAG_OVERLAP, s), "anvilq_embed")
        for l, w in enumerate(self.layers):
            self._qkv_rope(l, w)
            _lib.check(lib.anvilq_gqa_decode_ex(
                self.q.data_ptr(), self.k_cache[l].data_ptr(), self.v_cache[l].data_ptr(), self.seqlen.data_ptr(),
                self.attn.data_ptr(), 1, QH, KVH, D, self.max_seq, 0.0, self.workspace.data_ptr(),
                self.workspace.numel(), self.dev_err.data_ptr(), FLAG_OVERLAP, s), "anvilq_gqa_decode_ex")
            self._gemv(w["o"], self.attn, 0, None, self.x, 1, QH * D, H)
            if self.mlp:
                self._mlp(l, w)
            else:
                self._mlp_gemvs(l, w)
        _lib.check(lib.anvilq_lmhead_argmax(
            self.x.data_ptr(), self.gamma_final.data_ptr(), RMS_EPS, self.embedding.data_ptr(),
            None if self.logits is None else self.logits.data_ptr(), self.key.data_ptr(), H, V, FLAG_OVERLAP, s),
            "anvilq_lmhead_argmax")
        _lib.check(lib.anvilq_argmax_commit(self.key.data_ptr(), self.token.data_ptr(), self.pos.data_ptr(),
                                            FLAG_OVERLAP, s), "anvilq_argmax_commit")
        if host_io:
            self.token_out.copy_(self.token, non_blocking=True)

    def kernels_per_step(self) -> int:
        return 3 if self.fused else 1 + (4 if self.mlp else 5) * self.shape[0] + 2

    def record_layers(self):
        """A CUDA graph of the fused layers kernel alone (the step without the
        lm_head), for timing it on its own; position and token stay as they are."""
        if not self.fused:
            raise ValueError("the decoder runs one kernel per operation")
        with torch.cuda.stream(self.stream):
            self._layers_fused()
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self._layers_fused()
        return graph

    def layer_bytes_per_step(self, context: int) -> int:
        """Algorithmic HBM bytes of the layers of one step (no lm_head): the
        projections with their activation traffic and K / V read once."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        return self.gemv_bytes_per_step() + L * (context * KVH * D * 2 * 2)

    def reset(self, token: int):
        """Start a new sequence at position 0 with `token` as the first input."""
        with torch.cuda.stream(self.stream):
            self.pos.zero_()
            self.token.fill_(int(token))
            self.token_in.fill_(int(token))
        self.stream.synchronize()

    def set_position(self, token: int, pos: int):
        """Make the next step run `token` at position `pos` of the current
        sequence: cache rows [0, pos) are kept, row pos is (re)written."""
        if not 0 <= int(pos) < self.max_seq:
            raise ValueError(f"position {pos} outside the cache [0, {self.max_seq})")
        with torch.cuda.stream(self.stream):
            self.pos.fill_(int(pos))
            self.token.fill_(int(token))
            self.token_in.fill_(int(token))

    def capture(self, host_io: bool = False):
        """Record one step as a CUDA graph (warming the kernels first) and make it
        the graph that ``step`` replays.  host_io=True puts the copy of the
        input token from pinned host memory and of the chosen token back to it
        inside the graph (``token_in`` / ``token_out``)."""
        self.graph = self.record(host_io)
        return self

    def record(self, host_io: bool = False):
        """A CUDA graph of one step; the decoder state (position, token) is left as it was."""
        save_pos = self.pos.clone()
        save_tok = self.token.clone()
        with torch.cuda.stream(self.stream):
            self._enqueue(host_io)
        self.stream.synchronize()
        with torch.cuda.stream(self.stream):
            self.pos.copy_(save_pos)
            self.token.copy_(save_tok)
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self._enqueue(host_io)
        return graph

    def record_gemvs(self):
        """A CUDA graph of only this step's W4A16 GEMVs (same weights, buffers and
        fused modes, same order), for timing the GEMV kernel on its own."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape

        def enqueue():
            for l, w in enumerate(self.layers):
                self._qkv_rope(l, w)
                self._gemv(w["o"], self.attn, 0, None, self.x, 1, QH * D, H)
                if self.mlp:
                    self._mlp(l, w)
                else:
                    self._mlp_gemvs(l, w)

        with torch.cuda.stream(self.stream):
            enqueue()
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            enqueue()
        return graph

    def gemv_bytes_per_step(self) -> int:
        """Algorithmic HBM bytes of the step's 4 L GEMV launches, with each fused
        mode's own activation traffic: the weights of the projection (int4,
        zeros, scales, bias) plus what the prologue reads and the epilogue
        writes -- QKV: fp32 residual and fp16 gamma in, q and the new K / V rows
        out (fp16); O: fp16 attention output in, fp32 residual read and written;
        gate/up: fp32 residual and gamma in, fp16 [gate | up] out (fp16 silu(g) u
        with gu_act); down: fp16 gate and up in (the fp16 products with gu_act),
        fp32 residual read and written."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        w = lambda K, N, bias: synthetic.gemv_bytes(1, K, N, G, bias) - 2 * K - 2 * N   # weights only
        nqkv = (QH + 2 * KVH) * D
        act = I if getattr(self, "gu_act", False) else 2 * I   # fp16 elements between gate/up and down
        b = w(H, nqkv, True) + 4 * H + 2 * H + 2 * nqkv
        b += w(QH * D, H, False) + 2 * QH * D + 8 * H
        b += w(H, 2 * I, False) + 4 * H + 2 * H + 2 * act
        b += w(I, H, False) + 2 * act + 8 * H
        return b * L

    def fill_context(self, length: int, seed: int = 0):
        """Fill cache rows [0, length) with N(0,1) keys and values (a synthetic
        context) and set the position to `length`."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        with torch.cuda.stream(self.stream):
            self.k_cache[:, :length].normal_(generator=g)
            self.v_cache[:, :length].normal_(generator=g)
            self.pos.fill_(length)
        self.stream.synchronize()

    def step(self):
        """Enqueue one token on ``self.stream`` (the graph if captured)."""
        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._enqueue(False)

    def generate(self, first_token: int, n: int):
        """Greedy-decode n tokens after `first_token`; returns the n chosen ids."""
        self.reset(first_token)
        out = []
        for _ in range(n):
            self.step()
            self.stream.synchronize()
            out.append(int(self.token.item()))
        self.check_errors()
        return out

    def check_errors(self):
        v = int(self.dev_err.item())
        if v:
            self.dev_err.zero_()
            raise _lib.AnvilqError(f"decode step device error bits 0x{v:x}")

    # -- M draft tokens in one pass (speculative verification) -----------------
    def _verify_buffers(self, M: int):
        bufs = getattr(self, "_vbufs", {})
        if M not in bufs:
            L, H, I, QH, KVH, D, G, V, _ = self.shape
            dev = self.device
            z = lambda shape, dt: torch.zeros(shape, dtype=dt, device=dev)
            bufs[M] = dict(
                tok=z(M, torch.int32), pos=z(M, torch.int32), key=z(M, torch.int64), out=z(M, torch.int32),
                x=z((M, H), torch.float32), h=z((M, H), torch.float16), y=z((M, H), torch.float16),
                qkv=z((M, (QH + 2 * KVH) * D), torch.float16), q=z((M, QH, D), torch.float16),
                attn=z((M, QH, D), torch.float16), gu=z((M, 2 * I), torch.float16), act=z((M, I), torch.float16),
                row=z(M, torch.int32), anc=z(M, torch.int32))
            self._vbufs = bufs
        return bufs[M]

    def verify_tokens(self, tokens, pos: int):
        """Run M draft tokens at positions pos .. pos + M - 1 through the model in
        one pass and return the greedy choice after each of them.

        The batched counterpart of M decode steps (FP32Model.token per token,
        official_weights.py:451-509): every projection is one M-row W4A16 GEMM,
        so the weights stream once for all M tokens; each token's K/V row is
        written at its position and token m attends to the cache rows [0, pos)
        and the draft tokens 0..m (tree attention with a chain of ancestors).
        Rows pos + m of the caches are overwritten.  The decoder's own token and
        position are left unchanged."""
        return self.verify_tree(tokens, list(range(-1, len(tokens) - 1)), pos)

    def verify_tree(self, tokens, parents, pos: int):
        """Run a tree of M draft tokens through the model in one pass and return
        the greedy choice after each node.

        Node m holds token ``tokens[m]`` and continues node ``parents[m]``
        (-1: the committed prefix [0, pos); parents come first, parents[m] < m).
        Its depth d (0 for a child of the prefix) makes it the token at position
        pos + d: it is rotated to that position, staged in cache row pos + m, and
        attends to the prefix and its own ancestors (itself included) only --
        per-node positions, RoPE and ancestor visibility of the draft-tree
        decoder (anvil-q3-ht2/design/SPEC.md:71-86; ancestor contract
        anvil-q1-ht3/design/SPEC.md:528-533).  A chain is verify_tokens.  Rows
        pos .. pos + M - 1 of the caches are overwritten."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        M = len(tokens)
        if M < 1 or M > 32 or len(parents) != M or pos < 0 or pos + M > self.max_seq:
            raise ValueError(f"{M} draft nodes at position {pos} do not fit the cache of {self.max_seq}")
        depth, anc = [], []
        for m, par in enumerate(parents):
            par = int(par)
            if not -1 <= par < m:
                raise ValueError(f"node {m}: parent {par} must be -1 or an earlier node")
            depth.append(0 if par < 0 else depth[par] + 1)
            anc.append((1 << m) | (0 if par < 0 else anc[par]))
        lib = _lib.load()
        b = self._verify_buffers(M)
        s = self.stream.cuda_stream
        chk = _lib.check
        with torch.cuda.stream(self.stream):
            b["tok"].copy_(torch.tensor([int(t) for t in tokens], dtype=torch.int32), non_blocking=False)
            b["pos"].copy_(torch.tensor([pos + d for d in depth], dtype=torch.int32), non_blocking=False)
            b["row"].copy_(torch.arange(pos, pos + M, dtype=torch.int32), non_blocking=False)
            b["anc"].copy_(torch.tensor(anc, dtype=torch.int64).to(torch.int32), non_blocking=False)
            for m in range(M):
                chk(lib.anvilq_embed(self.embedding.data_ptr(), b["tok"][m:].data_ptr(), b["x"][m].data_ptr(), H, V,
                                     b["key"][m:].data_ptr(), self.dev_err.data_ptr(), 0, s), "anvilq_embed")
            for l, w in enumerate(self.layers):
                chk(lib.anvilq_rmsnorm_rows(b["x"].data_ptr(), self.gamma_in[l].data_ptr(), RMS_EPS,
                                            b["h"].data_ptr(), M, H, 0, s), "anvilq_rmsnorm_rows")
                ops.gemm(b["h"], *w["qkv"], G, out=b["qkv"], dev_err=self.dev_err)
                for m in range(M):
                    chk(lib.anvilq_rope_kv_append_at(b["qkv"][m].data_ptr(), b["pos"][m:].data_ptr(),
                                                     b["row"][m:].data_ptr(), b["q"][m].data_ptr(),
                                                     self.k_cache[l].data_ptr(), self.v_cache[l].data_ptr(), QH, KVH,
                                                     D, self.max_seq, ROPE_THETA, self.dev_err.data_ptr(), 0, s),
                        "anvilq_rope_kv_append_at")
                ops.tree_attention(b["q"], self.k_cache[l], self.v_cache[l], b["anc"], pos, out=b["attn"],
                                   dev_err=self.dev_err)
                ops.gemm(b["attn"].view(M, QH * D), *w["o"][:3], None, G, out=b["y"], dev_err=self.dev_err)
                chk(lib.anvilq_residual_add_rows(b["x"].data_ptr(), b["y"].data_ptr(), M, H, 0, s),
                    "anvilq_residual_add_rows")
                chk(lib.anvilq_rmsnorm_rows(b["x"].data_ptr(), self.gamma_post[l].data_ptr(), RMS_EPS,
                                            b["h"].data_ptr(), M, H, 0, s), "anvilq_rmsnorm_rows")
                ops.gemm(b["h"], *w["gu"][:3], None, G, out=b["gu"], dev_err=self.dev_err)
                chk(lib.anvilq_silu_mul_rows(b["gu"].data_ptr(), b["act"].data_ptr(), M, I, 0, s),
                    "anvilq_silu_mul_rows")
                ops.gemm(b["act"], *w["down"][:3], None, G, out=b["y"], dev_err=self.dev_err)
                chk(lib.anvilq_residual_add_rows(b["x"].data_ptr(), b["y"].data_ptr(), M, H, 0, s),
                    "anvilq_residual_add_rows")
            for m in range(M):
                chk(lib.anvilq_lmhead_argmax(b["x"][m].data_ptr(), self.gamma_final.data_ptr(), RMS_EPS,
                                             self.embedding.data_ptr(), None, b["key"][m:].data_ptr(), H, V, 0, s),
                    "anvilq_lmhead_argmax")
                chk(lib.anvilq_argmax_commit(b["key"][m:].data_ptr(), b["out"][m:].data_ptr(), None, 0, s),
                    "anvilq_argmax_commit")
        self.stream.synchronize()
        self.check_errors()
        return [int(t) for t in b["out"].cpu()]

    def commit_tree_path(self, path, pos: int):
        """After verify_tree at `pos`, move the staged K/V rows of the accepted
        nodes ``path`` (node indices, root first) to rows pos, pos + 1, ... --
        where sequential decoding would have written them (each was rotated to
        exactly that position).  Path nodes have increasing indices, so no row
        is read after it was overwritten."""
        with torch.cuda.stream(self.stream):
            for d, m in enumerate(path):
                if m < d:
                    raise ValueError("a path node cannot come before its depth")
                if m != d:
                    self.k_cache[:, pos + d].copy_(self.k_cache[:, pos + m])
                    self.v_cache[:, pos + d].copy_(self.v_cache[:, pos + m])
        self.stream.synchronize()

    def bytes_per_step(self, context: int) -> int:
        """Algorithmic HBM bytes of one step at a given context length."""
        L, H, I, QH, KVH, D, G, V, _ = self.shape
        b = self.gemv_bytes_per_step()
        b += L * (context * KVH * D * 2 * 2)    # K and V read once per layer
        b += V * H * 2                            # tied lm_head
        return b
