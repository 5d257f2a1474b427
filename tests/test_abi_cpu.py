"""The C-ABI library loads without a GPU, exports every function include/rapier_b200.h declares, and its
host-side validation rejects bad arguments with RK_EINVAL before touching the device. CPU only."""
import ctypes as C

import pytest

from rapier_b200 import _lib, ops


def test_library_loads_and_exports_every_header_symbol():
    L = _lib.lib()
    declared = _lib.header_functions()
    assert len(declared) >= 25
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"
    unbound = [n for n in declared if n not in _lib.SIGNATURES]
    assert not unbound, f"declared but without a ctypes signature: {unbound}"


def test_version_and_sizes():
    L = _lib.lib()
    assert L.rk_version() >= 1
    assert L.rk_q8_1_bytes(4096, 1) == 4608
    assert L.rk_q8_1_bytes(12288, 2) == 2 * 13824
    assert L.rk_q8_1_bytes(100, 1) == 0
    assert L.rk_weight_bytes(14, 4096, 12288) == 41287680
    assert L.rk_weight_bytes(8, 4096, 4096) == 4096 * 128 * 34
    assert L.rk_packed_bytes(14, 4096, 12288) == 41287680
    assert L.rk_packed_bytes(14, 768, 4) == 0  # n_in % 1024
    assert L.rk_packed_bytes(14, 4096, 6) == 0  # n_out % 4


FAKE = 0x10000  # an aligned, never-dereferenced address: validation fails before any device access


@pytest.mark.parametrize("args,frag", [
    ((14, FAKE, FAKE, FAKE, 4000, 8, 1, FAKE), "divisible"),
    ((14, FAKE, FAKE, FAKE, 4096, 0, 1, FAKE), "n_out"),
    ((14, FAKE, FAKE, FAKE, 4096, 8, 17, FAKE), "ncols"),
    ((14, FAKE, 0, FAKE, 4096, 8, 1, FAKE), "aligned"),
    ((14, FAKE, FAKE + 2, FAKE, 4096, 8, 1, FAKE), "aligned"),
    ((14, FAKE, FAKE, FAKE, 4096, 8, 1, 0), "stream"),
    ((3, FAKE, FAKE, FAKE, 4096, 8, 1, FAKE), "unsupported"),
])
def test_mmvq_validation(args, frag):
    with pytest.raises(ValueError) as ei:
        ops.native_mmvq(*args[:7], stream=args[7])
    assert frag in str(ei.value)


def test_packed_validation_messages():
    with pytest.raises(ValueError, match="1024"):
        ops.mmvq_packed(14, FAKE, FAKE, FAKE, 768, 4, 1, stream=FAKE)
    with pytest.raises(ValueError, match="16-byte"):
        ops.mmvq_packed(14, FAKE + 4, FAKE, FAKE, 1024, 4, 1, stream=FAKE)
    with pytest.raises(ValueError, match="stream"):
        ops.native_quantize_q8_1(FAKE, FAKE, 4096, 1, stream=0)


def test_rk_error_carries_code():
    try:
        ops.native_mmvq(14, FAKE, FAKE, FAKE, 4000, 8, 1, stream=FAKE)
    except ops.RkError as e:
        assert e.code == _lib.RK_EINVAL
    else:
        raise AssertionError("expected RkError")
    assert "divisible" in _lib.last_error()


def test_last_error_is_per_thread():
    import threading

    ops.InvalidArgument  # noqa: B018
    try:
        ops.native_mmvq(14, FAKE, FAKE, FAKE, 4000, 8, 1, stream=FAKE)
    except ValueError:
        pass
    seen = {}

    def other():
        seen["msg"] = _lib.last_error()

    th = threading.Thread(target=other)
    th.start()
    th.join()
    assert seen["msg"] == ""
    assert C.string_at(_lib.lib().rk_last_error())  # the calling thread keeps its message
