"""Torch-tensor front end of the C ABI: shape/dtype checks, workspaces, device errors.

PyTorch only provides device memory and streams here; every computation runs in
libanvilq.so.  All functions take CUDA tensors and enqueue on the current torch
stream.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_state = threading.local()
_dev_err = {}          # device index -> int32[1] device error word
_workspaces = {}       # (device index, stream ptr) -> uint8 workspace
_lock = threading.Lock()


def _stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def device_error_word(device) -> torch.Tensor:
    """Per-device int32 word that kernels OR their ANVILQ_DEV_ERR_* bits into."""
    idx = torch.device(device).index
    with _lock:
        w = _dev_err.get(idx)
        if w is None:
            w = torch.zeros(1, dtype=torch.int32, device=device)
            _dev_err[idx] = w
    return w


def raise_device_errors(device=None):
    """Synchronise the device error word, clear it, and raise if a kernel flagged an error.

    Mirrors the reference, where an invalid AWQ scale fails the operation
    (anvil-q1/tests/official_weights.py:430, anvil-q1/design/SPEC.md:175-177).
    """
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = device_error_word(device)
    value = int(w.item())
    if value:
        w.zero_()
        what = []
        if value & 1:
            what.append("invalid AWQ scale (negative nonzero or nonfinite)")
        if value & 2:
            what.append("sequence length outside [1, Tmax]")
        if value & 4:
            what.append("bounded wait expired inside a kernel")
        if value & 8:
            what.append("token id outside [0, V)")
        if value & 16:
            what.append("nonfinite binary16 parameter (bias)")
        if value & 32:
            what.append("page-table entry of a live page absent or out of range")
        if value & 64:
            what.append("draft-node ancestor mask breaks the tree contract")
        if value & 128:
            what.append("legacy cache block with a forbidden code, padding or metadata")
        raise _lib.AnvilqError(f"device error bits 0x{value:x}: " + "; ".join(what))


def workspace(device, nbytes: int) -> torch.Tensor:
    """Zero-filled scratch reused by calls on the current stream (kernels leave it zeroed)."""
    idx = torch.device(device).index
    key = (idx, _stream_ptr(device))
    with _lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws


def _check_awq(qweight, qzeros, scales, group):
    if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32:
        raise TypeError("qweight and qzeros must be int32 (AWQ packed)")
    if scales.dtype != torch.float16:
        raise TypeError("scales must be float16")
    if qweight.dim() != 2 or qzeros.dim() != 2 or scales.dim() != 2:
        raise ValueError("qweight, qzeros and scales must be 2-D")
    K, W8 = qweight.shape
    N = W8 * 8
    if group < 1:
        raise ValueError("group size must be >= 1")
    groups = -(-K // group)   # row k uses group k // G; a partial last group is allowed
    if tuple(qzeros.shape) != (groups, W8) or tuple(scales.shape) != (groups, N):
        raise ValueError("qzeros/scales shapes do not match qweight and the group size")
    for t in (qweight, qzeros, scales):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("AWQ tensors must be contiguous CUDA tensors")
    return K, N


GEMM_OVERLAP_PRIOR = 1


def gemm(x, qweight, qzeros, scales, bias=None, group: int = 128, out=None, dev_err=None,
         overlap_prior: bool = False, tensor_cores: bool = False):
    """y[M, N] = x[M, K] @ dequant(qweight, qzeros, scales) (+ bias), fp16 out.

    GPU counterpart of FP32Model.linear (anvil-q1/tests/official_weights.py:418-437)
    for M rows at once.  Device-side scale errors are OR-ed into `dev_err`
    (default: the per-device word read by ``raise_device_errors``).
    overlap_prior: the weights are not written by the preceding work on the
    stream, so the kernel may start streaming them before that work ends.
    """
    K, N = _check_awq(qweight, qzeros, scales, group)
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dtype != torch.float16 or x2.dim() != 2 or x2.shape[1] != K:
        raise ValueError(f"x must be float16 [M, {K}]")
    if not x2.is_contiguous() or x2.device != qweight.device:
        raise ValueError("x must be contiguous and on the weights' device")
    M = x2.shape[0]
    if bias is not None and (bias.dtype != torch.float16 or bias.numel() != N or not bias.is_contiguous()):
        raise ValueError("bias must be contiguous float16 [N]")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=x2.device)
    elif out.dtype != torch.float16 or tuple(out.shape) not in ((M, N), (N,) if squeeze else (M, N)) \
            or not out.is_contiguous():
        raise ValueError("out must be contiguous float16 [M, N]")
    lib = _lib.load()
    need = lib.anvilq_w4a16_gemm_workspace_size(M, K, N, group)
    ws = workspace(x2.device, need)
    err = device_error_word(x2.device) if dev_err is None else dev_err
    if tensor_cores:
        _lib.check(lib.anvilq_w4a16_verify_gemm(_ptr(x2), _ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(bias),
                                                _ptr(out), M, K, N, group, _ptr(ws), ws.numel(), _ptr(err),
                                                _stream_ptr(x2.device)), "anvilq_w4a16_verify_gemm")
        return out.view(N) if squeeze else out
    flags = GEMM_OVERLAP_PRIOR if overlap_prior else 0
    _lib.check(lib.anvilq_w4a16_gemm_ex(_ptr(x2), _ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(bias),
                                        _ptr(out), M, K, N, group, _ptr(ws), ws.numel(), _ptr(err), flags,
                                        _stream_ptr(x2.device)), "anvilq_w4a16_gemm_ex")
    return out.view(N) if squeeze else out


def gemv_plan(K: int, N: int, group: int = 128, kernel: int | None = None) -> dict:
    """The plan ``gemm`` uses for one row (anvilq_w4a16_gemv_plan), or with
    ``kernel`` the best plan of that kernel (anvilq_w4a16_gemv_kernel_plan):
    kernel (``_lib.GEMV_KERNEL_CLUSTER`` / ``_lib.GEMV_KERNEL_STREAM``),
    band_cols, cluster, kc, warps, stages, ctas."""
    plan = _lib.GemvPlan()
    lib = _lib.load()
    if kernel is None:
        _lib.check(lib.anvilq_w4a16_gemv_plan(K, N, group, ctypes.byref(plan)), "anvilq_w4a16_gemv_plan")
    else:
        _lib.check(lib.anvilq_w4a16_gemv_kernel_plan(int(kernel), K, N, group, ctypes.byref(plan)),
                   "anvilq_w4a16_gemv_kernel_plan")
    return plan.as_dict()


CHAIN_WIDE_BYTES = 40 << 20   # int4 bytes of a chain's largest projection above which CTAs get 16 warps


def chain_plans(shapes, group: int = 128) -> list:
    """Plans for a chain of M = 1 projections [(K, N), ...] launched back to back
    (one tensor-parallel rank's slices of a layer): the stream-K kernel for every
    one, all with the same CTA shape -- 16 warps when the largest projection
    holds at least ``CHAIN_WIDE_BYTES`` of int4, 8 otherwise -- so consecutive
    launches under programmatic dependent launch never switch between block
    shapes or kernels.  Measured on B200 over the 70B-class slices (8192x8192,
    8192x28672, 28672x8192 split W ways, one CUDA graph per layer): per layer
    52.5 -> 43.8 us at W = 2, 37.7 -> 30.5 at W = 4, 28.6 -> 24.3 at W = 8
    against the per-shape defaults, which mix 8 and 16 warps or the cluster
    kernel; unchanged at W = 1.  Falls back to the per-shape plans of
    ``gemv_plan`` when a projection does not fit the stream-K kernel."""
    shapes = [(int(K), int(N)) for K, N in shapes]
    try:
        plans = [gemv_plan(K, N, group, kernel=_lib.GEMV_KERNEL_STREAM) for K, N in shapes]
    except _lib.AnvilqError:
        return [gemv_plan(K, N, group) for K, N in shapes]
    warps = 16 if max(K * N // 2 for K, N in shapes) >= CHAIN_WIDE_BYTES else 8
    for p in plans:
        p["warps"] = warps
    return plans


def gemv_planned(x, qweight, qzeros, scales, bias=None, group: int = 128, plan=None, out=None, dev_err=None,
                 overlap_prior: bool = False):
    """y[N] = x[K] @ dequant(W) (+ bias) under an explicit plan (a dict with
    the fields of ``gemv_plan``); the library checks the plan against the
    kernel's rules and raises on one it does not accept."""
    K, N = _check_awq(qweight, qzeros, scales, group)
    x1 = x.reshape(-1)
    if x1.dtype != torch.float16 or x1.numel() != K or not x1.is_contiguous():
        raise ValueError(f"x must be contiguous float16 [{K}]")
    if out is None:
        out = torch.empty(N, dtype=torch.float16, device=x1.device)
    p = _lib.GemvPlan(**plan)
    lib = _lib.load()
    need = lib.anvilq_w4a16_gemv_plan_workspace_size(K, N, group, ctypes.byref(p))
    if need == 0:
        raise _lib.AnvilqError(f"plan {plan} does not fit K={K}, N={N}, G={group}")
    ws = workspace(x1.device, need)
    err = device_error_word(x1.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_w4a16_gemv_planned(_ptr(x1), _ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(bias),
                                             _ptr(out), K, N, group, ctypes.byref(p), _ptr(ws), ws.numel(),
                                             _ptr(err), GEMM_OVERLAP_PRIOR if overlap_prior else 0,
                                             _stream_ptr(x1.device)), "anvilq_w4a16_gemv_planned")
    return out


def mlp_interleave(qweight, qzeros, scales):
    """gate|up AWQ tensors (gate columns first: qweight and qzeros [rows, 2I/8],
    scales [groups, 2I]) in the unit-interleaved column order ``mlp`` takes: for
    every 32 intermediate rows, the gate's 4 words (32 columns) then the up's 4."""
    def perm(t, per):
        r, n = t.shape
        return t.view(r, 2, n // (2 * per), per).permute(0, 2, 1, 3).reshape(r, n).contiguous()
    return perm(qweight, 4), perm(qzeros, 4), perm(scales, 32)


def mlp(r, gamma, gu, down, group: int = 128, eps: float = 1e-6, dev_err=None, overlap_prior: bool = False):
    """The decode step's MLP in one launch (anvilq_w4a16_mlp), in place on the fp32
    residual r [H]: r += fp16(silu(g) u) @ W_down with g, u = fp16(RMSNorm(r) gamma @
    W_gate / W_up).  gu: (qweight, qzeros, scales) in the order of ``mlp_interleave``;
    down: AWQ (qweight, qzeros, scales) [I, H/8]."""
    if r.dtype != torch.float32 or r.dim() != 1 or not r.is_contiguous():
        raise ValueError("r must be a contiguous float32 vector")
    H = r.numel()
    gq, gz, gs = gu
    dq, dz, ds = down[:3]
    I = dq.shape[0]
    if gq.shape != (H, 2 * I // 8) or dq.shape != (I, H // 8):
        raise ValueError(f"gate/up must be [{H}, {2 * I // 8}] and down [{I}, {H // 8}] words")
    lib = _lib.load()
    need = lib.anvilq_w4a16_mlp_workspace_size(H, I, group)
    ws = workspace(r.device, need)
    err = device_error_word(r.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_w4a16_mlp(_ptr(r), _ptr(gamma), eps, _ptr(gq), _ptr(gz), _ptr(gs), _ptr(dq), _ptr(dz),
                                    _ptr(ds), H, I, group, _ptr(ws), ws.numel(), _ptr(err),
                                    GEMM_OVERLAP_PRIOR if overlap_prior else 0, _stream_ptr(r.device)),
               "anvilq_w4a16_mlp")
    return r


def verify_gemm(x, qweight, qzeros, scales, bias=None, group: int = 128, out=None, dev_err=None):
    """The speculative-verify GEMM forced onto the tcgen05 tensor-core kernel for any M.

    ``gemm`` already picks it for M >= 16; this is for callers (and tests) that
    want the tensor-core path at every M.  Needs group 128, K % 128 == 0, N % 32 == 0.
    """
    return gemm(x, qweight, qzeros, scales, bias, group, out, dev_err, tensor_cores=True)


def gemm_q16(x_q16, qweight, qzeros, scales, bias=None, group: int = 128, out=None, dev_err=None):
    """Integer golden projection on the GPU: Q16.16 int32 x [M, K] -> Q16.16 int32 y [M, N].

    Bit-identical to the reference's integer model (anvil-q1/tests/official_weights.py:592-612):
    exact integer sum of x * (q - z) * round_away(scale * 2^16), plus
    clip32(round_away(bias * 2^16)) * 65536, then clip32(round_away(total / 65536)).
    """
    K, N = _check_awq(qweight, qzeros, scales, group)
    squeeze = x_q16.dim() == 1
    x2 = x_q16.unsqueeze(0) if squeeze else x_q16
    if x2.dtype != torch.int32 or x2.dim() != 2 or x2.shape[1] != K or not x2.is_contiguous():
        raise ValueError(f"x_q16 must be contiguous int32 [M, {K}]")
    M = x2.shape[0]
    if bias is not None and (bias.dtype != torch.float16 or bias.numel() != N):
        raise ValueError("bias must be float16 [N]")
    if out is None:
        out = torch.empty((M, N), dtype=torch.int32, device=x2.device)
    lib = _lib.load()
    ws = workspace(x2.device, lib.anvilq_w4a16_gemm_q16_workspace_size(M, K, N, group))
    err = device_error_word(x2.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_w4a16_gemm_q16(_ptr(x2), _ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(bias),
                                         _ptr(out), M, K, N, group, _ptr(ws), ws.numel(), _ptr(err),
                                         _stream_ptr(x2.device)), "anvilq_w4a16_gemm_q16")
    return out.view(N) if squeeze else out


def tc_pack(qweight, group: int = 128):
    """qweight int32 [K, N/8] (AWQ) -> the tensor-core kernel's resident layout (int32, 1-D).

    One-time rewrite for weights that stay on the device (anvilq_w4a16_tc_pack);
    use the result with ``verify_gemm_packed``.
    """
    if qweight.dtype != torch.int32 or qweight.dim() != 2 or not qweight.is_contiguous():
        raise ValueError("qweight must be contiguous int32 [K, N/8]")
    K, W8 = qweight.shape
    lib = _lib.load()
    nbytes = lib.anvilq_w4a16_tc_pack_size(K, W8 * 8, group)
    if nbytes == 0:
        raise ValueError("tensor-core layout needs group 128, K % 128 == 0 and N % 32 == 0")
    out = torch.empty(nbytes // 4, dtype=torch.int32, device=qweight.device)
    _lib.check(lib.anvilq_w4a16_tc_pack(_ptr(qweight), _ptr(out), K, W8 * 8, group, _stream_ptr(qweight.device)),
               "anvilq_w4a16_tc_pack")
    return out


def verify_gemm_packed(x, packed, qzeros, scales, bias=None, group: int = 128, out=None, dev_err=None):
    """``verify_gemm`` on weights rewritten by ``tc_pack``; qzeros/scales/bias as for ``gemm``."""
    if qzeros.dtype != torch.int32 or scales.dtype != torch.float16 or scales.dim() != 2:
        raise TypeError("qzeros int32 [K/G, N/8] and scales float16 [K/G, N] expected")
    K, N = scales.shape[0] * group, scales.shape[1]
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dtype != torch.float16 or x2.dim() != 2 or x2.shape[1] != K or not x2.is_contiguous():
        raise ValueError(f"x must be contiguous float16 [M, {K}]")
    M = x2.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=x2.device)
    lib = _lib.load()
    ws = workspace(x2.device, lib.anvilq_w4a16_gemm_workspace_size(M, K, N, group))
    err = device_error_word(x2.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_w4a16_verify_gemm_packed(_ptr(x2), _ptr(packed), _ptr(qzeros), _ptr(scales), _ptr(bias),
                                                   _ptr(out), M, K, N, group, _ptr(ws), ws.numel(), _ptr(err),
                                                   _stream_ptr(x2.device)), "anvilq_w4a16_verify_gemm_packed")
    return out.view(N) if squeeze else out


def gemm_exact(x, qweight, qzeros, scales, bias=None, group: int = 128, dev_err=None):
    """Reference-order GEMM: fp32 output bit-identical to FP32Model.linear."""
    K, N = _check_awq(qweight, qzeros, scales, group)
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    if x2.dtype != torch.float16 or x2.shape[1] != K or not x2.is_contiguous():
        raise ValueError(f"x must be contiguous float16 [M, {K}]")
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=x2.device)
    err = device_error_word(x2.device) if dev_err is None else dev_err
    _lib.check(_lib.load().anvilq_w4a16_gemm_exact(_ptr(x2), _ptr(qweight), _ptr(qzeros), _ptr(scales),
                                                   _ptr(bias), _ptr(out), M, K, N, group, _ptr(err),
                                                   _stream_ptr(x2.device)), "anvilq_w4a16_gemm_exact")
    return out.view(N) if x.dim() == 1 else out


def dequant(qweight, qzeros, scales, group: int = 128, dev_err=None):
    """(delta int8 [K, N], w float32 [K, N]) through the kernels' in-register unpack."""
    K, N = _check_awq(qweight, qzeros, scales, group)
    delta = torch.empty((K, N), dtype=torch.int8, device=qweight.device)
    w = torch.empty((K, N), dtype=torch.float32, device=qweight.device)
    err = device_error_word(qweight.device) if dev_err is None else dev_err
    _lib.check(_lib.load().anvilq_awq_dequant(_ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(delta), _ptr(w),
                                              K, N, group, _ptr(err), _stream_ptr(qweight.device)),
               "anvilq_awq_dequant")
    return delta, w


def pack(codes):
    """Row-major codes uint8 [rows, N] -> AWQ int32 [rows, N/8]."""
    if codes.dtype != torch.uint8 or codes.dim() != 2 or codes.shape[1] % 8 or not codes.is_contiguous():
        raise ValueError("codes must be contiguous uint8 [rows, N], N % 8 == 0")
    out = torch.empty((codes.shape[0], codes.shape[1] // 8), dtype=torch.int32, device=codes.device)
    _lib.check(_lib.load().anvilq_awq_pack(_ptr(codes), _ptr(out), codes.shape[0], codes.shape[1],
                                           _stream_ptr(codes.device)), "anvilq_awq_pack")
    return out


def unpack(packed, n: int | None = None):
    """AWQ int32 [rows, N/8] -> codes uint8 [rows, N]."""
    if packed.dtype != torch.int32 or packed.dim() != 2 or not packed.is_contiguous():
        raise ValueError("packed must be contiguous int32 [rows, N/8]")
    n = packed.shape[1] * 8 if n is None else n
    if n != packed.shape[1] * 8:
        raise ValueError("invalid packed output shape")
    out = torch.empty((packed.shape[0], n), dtype=torch.uint8, device=packed.device)
    _lib.check(_lib.load().anvilq_awq_unpack(_ptr(packed), _ptr(out), packed.shape[0], n,
                                             _stream_ptr(packed.device)), "anvilq_awq_unpack")
    return out


def pack_lanes(codes):
    """awq_prepare.pack_lanes signature (anvil-q1-fp/tests/awq_prepare.py:84-91):
    output-major codes [N, K] -> int32 [K, N/8]."""
    return pack(codes.t().contiguous())


def unpack_lanes(words, outputs: int):
    """awq_prepare.unpack_lanes signature (awq_prepare.py:94-99): int32 [K, N/8] -> uint8 [N, K]."""
    return unpack(words, outputs).t().contiguous()


def gqa_decode(q, k_cache, v_cache, seqlens, scale: float = 0.0, out=None, dev_err=None):
    """Flash-decoding GQA attention: q [B, Hq, D], caches [B, Tmax, Hkv, D] fp16,
    seqlens int32 [B] on the device; returns fp16 [B, Hq, D].

    GPU counterpart of attention(q, keys, values) (anvil-q1-fp/tests/fp64_reference.py:164-170),
    batched over sequences of individual lengths.
    """
    if q.dtype != torch.float16 or k_cache.dtype != torch.float16 or v_cache.dtype != torch.float16:
        raise TypeError("q and the KV caches must be float16")
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("q [B, Hq, D], k_cache/v_cache [B, Tmax, Hkv, D]")
    B, Hq, D = q.shape
    Bk, Tmax, Hkv, Dk = k_cache.shape
    if Bk != B or Dk != D:
        raise ValueError("batch or head_dim of q and the caches differ")
    if seqlens.dtype != torch.int32 or seqlens.numel() != B or not seqlens.is_cuda:
        raise ValueError("seqlens must be an int32 CUDA tensor [B]")
    for t in (q, k_cache, v_cache, seqlens):
        if not t.is_contiguous():
            raise ValueError("inputs must be contiguous")
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    need = lib.anvilq_gqa_decode_workspace_size(B, Hq, Hkv, D, Tmax)
    if need == 0:
        raise ValueError(f"unsupported attention shape B={B} Hq={Hq} Hkv={Hkv} D={D} Tmax={Tmax}")
    ws = workspace(q.device, need)
    err = device_error_word(q.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_gqa_decode(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(seqlens), _ptr(out), B, Hq,
                                     Hkv, D, Tmax, float(scale), _ptr(ws), ws.numel(), _ptr(err),
                                     _stream_ptr(q.device)), "anvilq_gqa_decode")
    return out


def gqa_decode_paged(q, k_pool, v_pool, page_table, seqlens, max_pages: int | None = None, scale: float = 0.0,
                     out=None, dev_err=None):
    """gqa_decode over a paged fp16 cache: pools [num_pages, page_tokens, Hkv, D],
    page_table int32 [B, max_pages] (uint32 entries: bit 31 valid, bits 30:0 the
    physical page; the Anvil-Q4 page table, anvil-q4/design/SPEC.md:205-208).
    Logical position t of sequence b is row t % page_tokens of page
    page_table[b, t // page_tokens].  Returns fp16 [B, Hq, D]."""
    if q.dtype != torch.float16 or k_pool.dtype != torch.float16 or v_pool.dtype != torch.float16:
        raise TypeError("q and the KV pools must be float16")
    if q.dim() != 3 or k_pool.dim() != 4 or v_pool.shape != k_pool.shape:
        raise ValueError("q [B, Hq, D], k_pool/v_pool [num_pages, page_tokens, Hkv, D]")
    B, Hq, D = q.shape
    num_pages, page_tokens, Hkv, Dk = k_pool.shape
    if Dk != D:
        raise ValueError("head_dim of q and the pools differ")
    if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != B or not page_table.is_cuda:
        raise ValueError("page_table must be an int32 CUDA tensor [B, max_pages]")
    if seqlens.dtype != torch.int32 or seqlens.numel() != B or not seqlens.is_cuda:
        raise ValueError("seqlens must be an int32 CUDA tensor [B]")
    for t in (q, k_pool, v_pool, page_table, seqlens):
        if not t.is_contiguous():
            raise ValueError("inputs must be contiguous")
    max_pages = page_table.shape[1] if max_pages is None else int(max_pages)
    if max_pages != page_table.shape[1]:
        raise ValueError("max_pages must equal page_table.shape[1]")
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    need = lib.anvilq_gqa_decode_workspace_size(B, Hq, Hkv, D, page_tokens * max_pages)
    if need == 0:
        raise ValueError(f"unsupported attention shape B={B} Hq={Hq} Hkv={Hkv} D={D}")
    ws = workspace(q.device, need)
    err = device_error_word(q.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_gqa_decode_paged(_ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(page_table), _ptr(seqlens),
                                           _ptr(out), B, Hq, Hkv, D, page_tokens, max_pages, num_pages,
                                           float(scale), _ptr(ws), ws.numel(), _ptr(err),
                                           _stream_ptr(q.device)), "anvilq_gqa_decode_paged")
    return out


def tree_attention(q, k_cache, v_cache, ancestors, prefix_len: int, scale: float = 0.0, out=None, dev_err=None):
    """Attention of M speculative draft nodes: q [M, Hq, D], one sequence's caches
    [Tmax, Hkv, D] fp16 holding the committed prefix in rows [0, prefix_len) and
    draft node j in row prefix_len + j, ancestors int32 [M] (bit j of entry m:
    node m sees node j; itself included).  Returns fp16 [M, Hq, D].

    Per-node causal tree attention (anvil-q3-ht2/design/SPEC.md:71-86, ancestor
    contract anvil-q1-ht3/design/SPEC.md:528-533)."""
    if q.dtype != torch.float16 or k_cache.dtype != torch.float16 or v_cache.dtype != torch.float16:
        raise TypeError("q and the caches must be float16")
    if q.dim() != 3 or k_cache.dim() != 3 or v_cache.shape != k_cache.shape:
        raise ValueError("q [M, Hq, D], k_cache/v_cache [Tmax, Hkv, D]")
    M, Hq, D = q.shape
    Tmax, Hkv, Dk = k_cache.shape
    if Dk != D:
        raise ValueError("head_dim of q and the caches differ")
    if ancestors.dtype != torch.int32 or ancestors.numel() != M or not ancestors.is_cuda:
        raise ValueError("ancestors must be an int32 CUDA tensor [M]")
    for t in (q, k_cache, v_cache, ancestors):
        if not t.is_contiguous():
            raise ValueError("inputs must be contiguous")
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    need = lib.anvilq_tree_attention_workspace_size(M, Hq, Hkv, D, Tmax)
    if need == 0:
        raise ValueError(f"unsupported tree attention shape M={M} Hq={Hq} Hkv={Hkv} D={D} Tmax={Tmax}")
    ws = workspace(q.device, need)
    err = device_error_word(q.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_tree_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(ancestors), int(prefix_len),
                                         _ptr(out), M, Hq, Hkv, D, Tmax, float(scale), _ptr(ws), ws.numel(),
                                         _ptr(err), _stream_ptr(q.device)), "anvilq_tree_attention")
    return out


def legacy_kv_shape(H: int, D: int, block: int, fmt: int):
    """(blocks per head B, words per block W) of the legacy cache layout."""
    bits = 8 if fmt == 1 else 4
    return (D + block - 1) // block, (block * bits + 31) // 32


def legacy_kv_encode(values, H: int, D: int, block: int, fmt: int):
    """Q16.16 rows int32 [R, H*D] -> (payload int32 [R, H*B*W], metadata int32
    [R, H*B]) in the legacy cache format fmt (1 INT8 symmetric, 2 INT4
    symmetric, 3 INT4 asymmetric; anvil-q4/tests/legacy_reference.py:71-97);
    uint32 words are held as int32."""
    if values.dtype != torch.int32 or values.dim() != 2 or values.shape[1] != H * D or not values.is_contiguous():
        raise ValueError("values must be contiguous int32 [R, H*D]")
    R = values.shape[0]
    B, W = legacy_kv_shape(H, D, block, fmt)
    payload = torch.empty((R, H * B * W), dtype=torch.int32, device=values.device)
    meta = torch.empty((R, H * B), dtype=torch.int32, device=values.device)
    lib = _lib.load()
    _lib.check(lib.anvilq_legacy_kv_encode(_ptr(values), _ptr(payload), _ptr(meta), R, H, D, block, fmt,
                                           _stream_ptr(values.device)), "anvilq_legacy_kv_encode")
    return payload, meta


def legacy_kv_decode(payload, meta, H: int, D: int, block: int, fmt: int, dev_err=None):
    """The legacy cache rows back to Q16.16 int32 [R, H*D]: sat32((code - z) 2^e)."""
    R = payload.shape[0]
    B, W = legacy_kv_shape(H, D, block, fmt)
    if payload.dtype != torch.int32 or tuple(payload.shape) != (R, H * B * W) or tuple(meta.shape) != (R, H * B):
        raise ValueError("payload int32 [R, H*B*W] and metadata int32 [R, H*B] expected")
    out = torch.empty((R, H * D), dtype=torch.int32, device=payload.device)
    lib = _lib.load()
    err = device_error_word(payload.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_legacy_kv_decode(_ptr(payload), _ptr(meta), _ptr(out), R, H, D, block, fmt, _ptr(err),
                                           _stream_ptr(payload.device)), "anvilq_legacy_kv_decode")
    return out


def kv_int8_store(src, codes, meta, escape=None, start=None, dev_err=None):
    """Encode K or V rows src [B, T, H, D] (fp16 or fp32) into an INT8 cache:
    codes int8 [B, Tmax, H, D], meta int32 [B, H, Tmax] (uint32 scale bits or the
    escape marker 0x7FC00000), escape fp32 [B, Tmax, H, D] or None; rows go to
    positions start[b] + t (start: int32 CUDA tensor [B], or None for 0).

    The Anvil-Q4 per-head INT8 cache with FP32 escape (anvil-q4/tests/cache_reference.py:54-83)."""
    if src.dim() != 4 or src.dtype not in (torch.float16, torch.float32) or not src.is_contiguous():
        raise ValueError("src must be contiguous fp16/fp32 [B, T, H, D]")
    B, T, H, D = src.shape
    if codes.dtype != torch.int8 or codes.dim() != 4 or codes.shape[0] != B or codes.shape[2:] != (H, D):
        raise ValueError("codes must be int8 [B, Tmax, H, D]")
    Tmax = codes.shape[1]
    if meta.dtype != torch.int32 or tuple(meta.shape) != (B, H, Tmax):
        raise ValueError("meta must be int32 [B, H, Tmax]")
    if escape is not None and (escape.dtype != torch.float32 or escape.shape != codes.shape):
        raise ValueError("escape must be float32 with the shape of codes")
    if start is not None and (start.dtype != torch.int32 or start.numel() != B or not start.is_cuda):
        raise ValueError("start must be an int32 CUDA tensor [B]")
    lib = _lib.load()
    err = device_error_word(src.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_kv_int8_store(_ptr(src), 1 if src.dtype == torch.float16 else 0, B, T, H, D, Tmax,
                                        _ptr(start), _ptr(codes), _ptr(meta), _ptr(escape), _ptr(err),
                                        _stream_ptr(src.device)), "anvilq_kv_int8_store")


def gqa_decode_int8(q, k_codes, k_meta, v_codes, v_meta, seqlens, k_escape=None, v_escape=None, scale: float = 0.0,
                    out=None, dev_err=None):
    """gqa_decode over INT8 caches (kv_int8_store's format); returns fp16 [B, Hq, D]."""
    if q.dtype != torch.float16 or q.dim() != 3 or not q.is_contiguous():
        raise TypeError("q must be contiguous float16 [B, Hq, D]")
    B, Hq, D = q.shape
    if k_codes.dtype != torch.int8 or k_codes.dim() != 4 or v_codes.shape != k_codes.shape:
        raise ValueError("k_codes/v_codes must be int8 [B, Tmax, Hkv, D]")
    _, Tmax, Hkv, Dk = k_codes.shape
    if Dk != D or k_codes.shape[0] != B:
        raise ValueError("batch or head_dim of q and the caches differ")
    if k_meta.dtype != torch.int32 or tuple(k_meta.shape) != (B, Hkv, Tmax) or v_meta.shape != k_meta.shape:
        raise ValueError("k_meta/v_meta must be int32 [B, Hkv, Tmax]")
    if seqlens.dtype != torch.int32 or seqlens.numel() != B or not seqlens.is_cuda:
        raise ValueError("seqlens must be an int32 CUDA tensor [B]")
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    need = lib.anvilq_gqa_decode_workspace_size(B, Hq, Hkv, D, Tmax)
    if need == 0:
        raise ValueError(f"unsupported attention shape B={B} Hq={Hq} Hkv={Hkv} D={D} Tmax={Tmax}")
    ws = workspace(q.device, need)
    err = device_error_word(q.device) if dev_err is None else dev_err
    _lib.check(lib.anvilq_gqa_decode_int8(_ptr(q), _ptr(k_codes), _ptr(k_meta), _ptr(k_escape), _ptr(v_codes),
                                          _ptr(v_meta), _ptr(v_escape), _ptr(seqlens), _ptr(out), B, Hq, Hkv, D,
                                          Tmax, float(scale), _ptr(ws), ws.numel(), _ptr(err),
                                          _stream_ptr(q.device)), "anvilq_gqa_decode_int8")
    return out
