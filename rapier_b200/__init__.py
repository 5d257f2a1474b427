"""rapier_b200 — B200-native (sm_100a) decode hot path of the Rapier engine for the qwen35 hybrid model.

The product is librapier_b200.so (C-ABI in include/rapier_b200.h): hand-written CUDA kernels and the
C++ decode engine. This package is the host-side mirror of the reference's operator surface (ops) and
a thin wrapper over the engine (engine). Importing it loads the library and fails loudly if it is
missing: there is no CPU fallback.
"""
from . import _lib

_lib.lib()

from . import ops  # noqa: E402

__all__ = ["ops"]
__version__ = "0.1.0"
