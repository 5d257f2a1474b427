"""The reference-kernel library for the GDN pin (oracle/_ref/libref_gdn.so: the reference's own
src/fused_gdn.cu built by oracle/Makefile's `ref` target) loads without a GPU and exports the three C entry
points tests/test_ref_pin_gpu.py calls. Skipped where it was not built (no reference tree at build time).
CPU only: nothing here launches a kernel."""
import ctypes as C
import os

import pytest

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libref_gdn.so")


def test_reference_gdn_library_exports_its_entry_points():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libref_gdn.so not built")
    lib = C.CDLL(LIB)
    for name in ("ref_gdn_conv_l2", "ref_gdn_ab", "ref_gdn_step_norm_silu_q8"):
        assert hasattr(lib, name), name
