"""Helpers shared by the tests: numpy <-> device buffers and the stated tolerances."""
from __future__ import annotations

import numpy as np

# fp32 outputs: |gpu - oracle| <= RTOL * (|oracle| + mean|oracle|) elementwise (1e-3 relative, with the
# vector's mean magnitude as the floor so values near zero are judged against the vector's scale).
RTOL = 1e-3


def to_dev(a: np.ndarray):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda")


def empty_dev(n: int, dtype):
    import torch

    return torch.empty(n, dtype=dtype, device="cuda")


def to_np(t) -> np.ndarray:
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_close(got: np.ndarray, want: np.ndarray, rtol: float = RTOL, what: str = ""):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    tol = rtol * (np.abs(want) + np.mean(np.abs(want)))
    bad = np.abs(got - want) > tol
    if bad.any():
        i = int(np.argmax(np.abs(got - want) - tol))
        raise AssertionError(f"{what}: {int(bad.sum())}/{bad.size} outside rtol {rtol}; worst index {i}: "
                             f"got {got[i]!r} want {want[i]!r}")


def rel_err(got, want) -> float:
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def assert_bits(got, want, what: str = ""):
    """Bit-for-bit equality of fp32 arrays (the kernels and the oracle run the same operation sequence)."""
    got = np.ascontiguousarray(got, np.float32).ravel()
    want = np.ascontiguousarray(want, np.float32).ravel()
    assert got.shape == want.shape, (got.shape, want.shape)
    same = got.view(np.uint32) == want.view(np.uint32)
    if not same.all():
        d = np.abs(got.astype(np.float64) - want)
        i = int(np.argmax(d))
        raise AssertionError(f"{what}: {int((~same).sum())}/{same.size} values differ in their bits; worst index "
                             f"{i}: got {got[i]!r} want {want[i]!r}")
