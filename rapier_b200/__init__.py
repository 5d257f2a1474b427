"""rapier_b200 — B200-native (sm_100a) decode hot path of the Rapier engine for the qwen35 hybrid model.

The product is librapier_b200.so (C-ABI in include/rapier_b200.h): hand-written CUDA kernels and the
C++ decode engine. This package is the host-side mirror of the reference's operator surface (ops) and
a thin wrapper over the engine (engine). The library is loaded on first use; every entry point raises
ImportError if it is missing: there is no CPU fallback.
"""
from . import _lib, ops  # noqa: F401

__all__ = ["ops", "load"]
__version__ = "0.1.0"


def load():
    """Load librapier_b200.so now (raises ImportError when it has not been built)."""
    return _lib.lib()
