"""anvilq_b200 -- B200 (sm_100a) W4A16 AWQ decode datapath.

Hand-written CUDA kernels behind a C ABI (include/anvilq.h, libanvilq.so),
with a Python host side that keeps the reference's AWQ storage layout and
golden-model call signatures (aHappend/anvil-q, anvil-q1/tests/official_weights.py).
"""
from . import synthetic
from ._lib import AnvilqError
from .checkpoint import ArrayCheckpoint, CheckpointError, PROJECTIONS

__all__ = ["synthetic", "AnvilqError", "ArrayCheckpoint", "CheckpointError", "PROJECTIONS",
           "ops", "golden_api"]


def __getattr__(name):
    # torch-dependent modules load lazily so the host logic imports without CUDA
    if name in ("ops", "golden_api"):
        import importlib
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
