"""ctypes binding of libanvilq.so (include/anvilq.h).

The library is the only compute path: if it is missing or fails to load this
module raises, it never substitutes a CPU or PyTorch computation.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("ANVILQ_LIB", PKG / "libanvilq.so"))

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes); kept in the order of include/anvilq.h
SIGNATURES = {
    "anvilq_abi_version": (I, []),
    "anvilq_strerror": (ctypes.c_char_p, [I]),
    "anvilq_w4a16_gemm_workspace_size": (SZ, [I, I, I, I]),
    "anvilq_w4a16_gemm": (I, [P, P, P, P, P, P, I, I, I, I, P, SZ, P, P]),
    "anvilq_w4a16_gemm_ex": (I, [P, P, P, P, P, P, I, I, I, I, P, SZ, P, ctypes.c_uint, P]),
    "anvilq_w4a16_gemv_plan": (I, [I, I, I, P]),
    "anvilq_w4a16_gemv_kernel_plan": (I, [I, I, I, I, P]),
    "anvilq_w4a16_gemv_plan_workspace_size": (SZ, [I, I, I, P]),
    "anvilq_w4a16_gemv_planned": (I, [P, P, P, P, P, P, I, I, I, P, P, SZ, P, ctypes.c_uint, P]),
    "anvilq_w4a16_gemm_exact": (I, [P, P, P, P, P, P, I, I, I, I, P, P]),
    "anvilq_w4a16_verify_gemm": (I, [P, P, P, P, P, P, I, I, I, I, P, SZ, P, P]),
    "anvilq_w4a16_tc_pack_size": (SZ, [I, I, I]),
    "anvilq_w4a16_tc_pack": (I, [P, P, I, I, I, P]),
    "anvilq_w4a16_verify_gemm_packed": (I, [P, P, P, P, P, P, I, I, I, I, P, SZ, P, P]),
    "anvilq_w4a16_gemm_q16_workspace_size": (SZ, [I, I, I, I]),
    "anvilq_w4a16_gemm_q16": (I, [P, P, P, P, P, P, I, I, I, I, P, SZ, P, P]),
    "anvilq_awq_dequant": (I, [P, P, P, P, P, I, I, I, P, P]),
    "anvilq_awq_pack": (I, [P, P, I, I, P]),
    "anvilq_awq_unpack": (I, [P, P, I, I, P]),
    "anvilq_gqa_decode_workspace_size": (SZ, [I, I, I, I, I]),
    "anvilq_gqa_decode": (I, [P, P, P, P, P, I, I, I, I, I, F, P, SZ, P, P]),
    "anvilq_gqa_decode_noalloc": (I, [P, P, P, P, P, I, I, I, I, I, F, P, P]),
    "anvilq_kv_int8_store": (I, [P, I, I, I, I, I, I, P, P, P, P, P, P]),
    "anvilq_gqa_decode_int8": (I, [P, P, P, P, P, P, P, P, P, I, I, I, I, I, F, P, SZ, P, P]),
    "anvilq_w4a16_gemv_fused": (I, [P, I, P, F, P, P, P, P, P, I, I, I, I, P, SZ, P, ctypes.c_uint, P]),
    "anvilq_w4a16_gemv_qkv_rope": (I, [P, I, P, F, P, P, P, P, I, I, P, P, P, P, P, I, I, I, I, F, P, SZ, P,
                                       ctypes.c_uint, P]),
    "anvilq_w4a16_mlp_workspace_size": (SZ, [I, I, I]),
    "anvilq_gqa_decode_ex": (I, [P, P, P, P, P, I, I, I, I, I, F, P, SZ, P, ctypes.c_uint, P]),
    "anvilq_w4a16_mlp": (I, [P, P, F, P, P, P, P, P, P, I, I, I, P, SZ, P, ctypes.c_uint, P]),
    "anvilq_peer_handle_size": (SZ, []),
    "anvilq_peer_export": (I, [P, P, ctypes.POINTER(ctypes.c_size_t)]),
    "anvilq_peer_import": (I, [P, SZ, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
    "anvilq_peer_close": (I, [P]),
    "anvilq_w4a16_gemv_allgather": (I, [P, P, P, P, P, I, I, I, I, I, I, I, P, P, P, P, SZ, P, ctypes.c_uint, P]),
    "anvilq_w4a16_gemv_allgather_planned": (I, [P, P, P, P, P, I, I, I, I, I, I, I, P, P, P, P, P, SZ, P,
                                                ctypes.c_uint, P]),
    "anvilq_peer_wait": (I, [P, I, P, P, P]),
    "anvilq_embed": (I, [P, P, P, I, I, P, P, ctypes.c_uint, P]),
    "anvilq_rope_kv_append": (I, [P, P, P, P, P, P, I, I, I, I, F, P, ctypes.c_uint, P]),
    "anvilq_rope_kv_append_at": (I, [P, P, P, P, P, P, I, I, I, I, F, P, ctypes.c_uint, P]),
    "anvilq_block_columns": (I, [P, P, I, I, I, I, P]),
    "anvilq_decode_layers_workspace_size": (SZ, [I, I, I, I, I, I, I, I]),
    "anvilq_decode_layers": (I, [P, I, I, I, I, I, I, I, I, F, F, P, I, P, P, P, P, P, P, SZ, P, P]),
    "anvilq_lmhead_argmax": (I, [P, P, F, P, P, P, I, I, ctypes.c_uint, P]),
    "anvilq_argmax_commit": (I, [P, P, P, ctypes.c_uint, P]),
    "anvilq_gqa_decode_paged": (I, [P, P, P, P, P, P, I, I, I, I, I, I, I, F, P, SZ, P, P]),
    "anvilq_tree_attention_workspace_size": (SZ, [I, I, I, I, I]),
    "anvilq_tree_attention": (I, [P, P, P, P, I, P, I, I, I, I, I, F, P, SZ, P, P]),
    "anvilq_rmsnorm_rows": (I, [P, P, F, P, I, I, ctypes.c_uint, P]),
    "anvilq_residual_add_rows": (I, [P, P, I, I, ctypes.c_uint, P]),
    "anvilq_silu_mul_rows": (I, [P, P, I, I, ctypes.c_uint, P]),
    "anvilq_legacy_kv_encode": (I, [P, P, P, I, I, I, I, I, P]),
    "anvilq_legacy_kv_decode": (I, [P, P, P, I, I, I, I, I, P, P]),
}

GEMV_KERNEL_CLUSTER = 0
GEMV_KERNEL_STREAM = 1


class GemvPlan(ctypes.Structure):
    """anvilq_gemv_plan: the kernel and launch shape of one batch-1 GEMV."""
    _fields_ = [("kernel", I), ("band_cols", I), ("cluster", I), ("kc", I), ("warps", I), ("stages", I),
                ("ctas", I)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


_lib = None


class AnvilqError(RuntimeError):
    """A libanvilq call returned a negative status or a kernel raised a device error."""


def load(path: Path | None = None):
    """Load (once) and return the bound library."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise AnvilqError(f"{p} is missing: build it with `python -m anvilq_b200.build`")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.anvilq_abi_version() != 1:
        raise AnvilqError("libanvilq ABI version mismatch")
    if path is None:
        _lib = lib
    return lib


def check(status: int, what: str = "anvilq call"):
    if status != 0:
        msg = load().anvilq_strerror(status).decode()
        raise AnvilqError(f"{what} failed with status {status}: {msg}")
