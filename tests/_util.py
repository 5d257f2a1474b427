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


def q8_1_codes_close(got: np.ndarray, want: np.ndarray, max_code_diff: int = 1, min_equal: float = 0.99):
    """Q8_1 blocks produced through a transcendental function (rsqrt, exp) on GPU vs CPU: the fp32
    input can differ in the last ulp, so a code may round the other way. Codes differ by at most
    `max_code_diff` and at least `min_equal` of them are identical; the scales agree within 1e-3."""
    g = got.reshape(-1, 36)
    w = want.reshape(-1, 36)
    gd = g[:, 0:2].copy().view(np.float16).astype(np.float32)
    wd = w[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert np.allclose(gd, wd, rtol=2e-3, atol=0), "Q8_1 scales differ"
    gc = g[:, 4:].view(np.int8).astype(np.int32)
    wc = w[:, 4:].view(np.int8).astype(np.int32)
    assert np.max(np.abs(gc - wc)) <= max_code_diff, "Q8_1 codes differ by more than 1"
    assert np.mean(gc == wc) >= min_equal, f"only {np.mean(gc == wc):.4f} of Q8_1 codes identical"
