"""The allocation-free attention entry point (rk_gqa_decode_f16_noalloc) against the entry point that takes a
caller scratch buffer. It is for callers that cannot allocate device memory (an application that keeps all
device memory in its own pool, a loop that cannot afford cudaMalloc's synchronization), so it keeps its chunk
partials in an array built into the library instead. This file is collected last so a failing run has
already run every other test."""
import numpy as np
import pytest
import torch

from tests._util import assert_bits, empty_dev, to_dev, to_np

pytestmark = pytest.mark.gpu


def _case(seed, n_kv, max_ctx, ncols):
    rng = np.random.default_rng(seed)
    k16 = rng.standard_normal((n_kv, max_ctx, 256)).astype(np.float16)
    v16 = rng.standard_normal((n_kv, max_ctx, 256)).astype(np.float16)
    q = (rng.standard_normal((ncols, 4 * n_kv, 256)) * 0.5).astype(np.float32)
    return to_dev(k16.view(np.uint16)), to_dev(v16.view(np.uint16)), q


def test_noalloc_matches_scratch_entry_on_two_calls(cuda):
    from rapier_b200 import ops

    n_head, n_kv, hd, ncols, max_ctx = 16, 4, 256, 2, 8193
    dk, dv, _ = _case(5, n_kv, max_ctx, ncols)
    sb = ops.gqa_scratch_bytes(n_head, ncols, max_ctx)
    scratch = empty_dev(sb // 4, torch.float32)
    # two calls in a row with different queries and positions: the shared array keeps the first call's
    # partials, the second call must not depend on them
    for call, pos in enumerate([max_ctx - 2, 1500]):
        q = to_dev(np.random.default_rng(100 + call).standard_normal((ncols, n_head, hd)).astype(np.float32) * 0.5)
        p = to_dev(np.array([pos], np.int32))
        want = empty_dev(ncols * n_head * hd, torch.float32)
        ops.gqa_decode_f16(q, dk, dv, want, n_head, n_kv, hd, ncols, p, max_ctx, 0.0625, scratch, sb)
        got = empty_dev(ncols * n_head * hd, torch.float32)
        ops.gqa_decode_f16_noalloc(q, dk, dv, got, n_head, n_kv, hd, ncols, p, max_ctx, 0.0625)
        # the same kernels on the same inputs: bit for bit
        assert_bits(to_np(got), to_np(want), what=f"no-alloc call {call}")
    assert ops.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_array(cuda):
    from rapier_b200 import ops

    n_head, n_kv, hd, ncols, max_ctx = 16, 4, 256, 2, 262144  # needs ~33 MiB of partials
    assert ops.gqa_scratch_bytes(n_head, ncols, max_ctx) > 16 << 20
    q = empty_dev(ncols * n_head * hd, torch.float32)
    o = empty_dev(ncols * n_head * hd, torch.float32)
    kc = empty_dev(1024, torch.int16)
    pos = to_dev(np.array([0], np.int32))
    with pytest.raises(ValueError, match="above the built-in"):
        ops.gqa_decode_f16_noalloc(q, kc, kc, o, n_head, n_kv, hd, ncols, pos, max_ctx, 0.0625)
