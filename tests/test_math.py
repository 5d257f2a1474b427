"""The exactly specified fp32 transcendentals (exp by Cody-Waite reduction + Taylor polynomial, log by the
atanh series, log1p by Goldberg's correction, 1/sqrt as two correctly rounded operations) that the CUDA
kernels and the CPU oracle both run in place of the vendor library, so every value that passes through
them (RMS scales, SiLU, sigmoid gates, the GDN decay, softmax weights) is bit-exact between the two.

CPU: the oracle's sequences against float64 numpy (ulp bounds). GPU: the device sequences bitwise equal to
the oracle's on the same inputs, and within the documented error bound of CUDA's own expf (2 ulp)."""
import numpy as np
import pytest

RNG = np.random.default_rng(2024)


def _inputs(fn: str) -> np.ndarray:
    r = RNG
    if fn == "exp":
        x = [r.uniform(-103.9, 88.7, 400_000), r.normal(0, 3, 200_000), np.linspace(-0.5, 0.5, 20001),
             [0.0, -0.0, 88.72, 88.73, -87.3, -103.9, -104.5, 1e-8, -1e-8, np.inf, -np.inf]]
    elif fn in ("log", "rsqrt"):
        x = [r.uniform(1e-30, 1e30, 200_000), r.uniform(0.5, 2.0, 200_000), np.exp(r.uniform(-85, 85, 200_000)),
             [1.0, 2.0, 0.5, 1e-40, 3.4e38]]
    elif fn == "log1p":
        x = [np.exp(r.uniform(-90, 20, 400_000)), r.uniform(0, 1, 100_000), [0.0, 1e-30, 4.85e8]]
    else:
        x = [r.normal(0, 5, 400_000), r.uniform(-90, 90, 100_000), [0.0, -0.0, 20.0, -20.0]]
    return np.concatenate([np.asarray(a, np.float64) for a in x]).astype(np.float32)


def _ref64(fn: str, x: np.ndarray) -> np.ndarray:
    v = x.astype(np.float64)
    with np.errstate(over="ignore"):
        return {"exp": np.exp, "log": np.log, "log1p": np.log1p, "rsqrt": lambda a: 1.0 / np.sqrt(a),
                "sigmoid": lambda a: 1.0 / (1.0 + np.exp(-a)), "silu": lambda a: a / (1.0 + np.exp(-a))}[fn](v)


def _ulps(got: np.ndarray, want: np.ndarray) -> np.ndarray:
    """|got - want| in units of the float32 spacing at want (normal range only)."""
    sp = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
    return np.abs(got.astype(np.float64) - want) / sp


# bounds in float32 ulps against the exact (float64) value, normal results
ULP_BOUND = {"exp": 1.0, "log": 2.0, "log1p": 4.0, "rsqrt": 1.5, "sigmoid": 3.0, "silu": 3.0}


@pytest.mark.parametrize("fn", sorted(ULP_BOUND))
def test_oracle_sequences_against_float64(oracle, fn):
    x = _inputs(fn)
    got = oracle.math(fn, x)
    want = _ref64(fn, x)
    normal = np.isfinite(want) & (np.abs(want) > 1.2e-38) & (np.abs(want) < 3.4e38)
    if fn == "silu":  # x / (1 + exp(-x)) is -0 once exp(-x) overflows (x < -88.7), in any fp32 evaluation
        normal &= x > -80.0
    assert np.all(_ulps(got[normal], want[normal]) <= ULP_BOUND[fn]), fn
    # specials: inf / 0 / subnormal results
    if fn == "exp":
        assert oracle.math("exp", np.array([np.inf, -np.inf, 89.0, -105.0], np.float32)).tolist() == \
            [np.inf, 0.0, np.inf, 0.0]
        assert np.isnan(oracle.math("exp", np.array([np.nan], np.float32))[0])
        sub = np.abs(want) <= 1.2e-38  # subnormal or zero results
        assert np.all(np.abs(got[sub].astype(np.float64) - want[sub]) <= 2 * 1.4013e-45)  # 2 subnormal steps


@pytest.mark.gpu
@pytest.mark.parametrize("fn", sorted(ULP_BOUND))
def test_device_sequences_bitwise_equal_oracle(cuda, oracle, fn):
    import torch

    from rapier_b200 import ops
    from tests._util import to_dev, to_np

    x = _inputs(fn)
    dx = to_dev(x)
    dy = torch.empty_like(dx)
    ops.math_probe(fn, dx, dy, x.size)
    got = to_np(dy)
    want = oracle.math(fn, x)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), f"{fn}: {int((~same).sum())} of {x.size} values differ from the oracle's bits"


@pytest.mark.gpu
def test_device_exp_within_cuda_expf_bound(cuda):
    """rk_expf stays within the 2-ulp bound CUDA documents for its own expf, and within 1 ulp of exp."""
    import torch

    from rapier_b200 import ops
    from tests._util import to_dev, to_np

    x = _inputs("exp")
    dx = to_dev(x)
    ours, lib = torch.empty_like(dx), torch.empty_like(dx)
    ops.math_probe("exp", dx, ours, x.size)
    ops.math_probe("cuda_expf", dx, lib, x.size)
    got, ref = to_np(ours), to_np(lib)
    want = _ref64("exp", x)
    normal = np.isfinite(want) & (want > 1.2e-38) & (want < 3.4e38)
    assert np.max(_ulps(got[normal], want[normal])) <= 1.0
    assert np.max(_ulps(ref[normal], want[normal])) <= 2.0  # the library's own documented bound
    assert np.max(np.abs(got[normal].astype(np.float64) - ref[normal]) / np.spacing(ref[normal])) <= 3.0
