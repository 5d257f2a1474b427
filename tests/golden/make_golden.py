"""Generate tests/golden/ggml_formats.npz from gguf-py 0.19.0 (an independent implementation of the ggml
block formats, shipped with llama.cpp). Run in a container where `import gguf` works:

    python tests/golden/make_golden.py

The fixture pins the oracle's restatement of the formats the reference path uses
(src/native_mmvq.cu:98-139 of the reference; ggml's block_q6_K / block_q8_0 / block_q8_1):

* q6k_raw / q6k_deq        random Q6_K blocks (random codes and signed scales, finite fp16 d) and
                           gguf's dequantization of them;
* q6k_codes                the signed codes (q - 32) recovered from gguf's floats (exact: every product
                           d * scale * code is exactly representable in fp32);
* q80_src / q80_raw        fp32 weights and gguf's Q8_0 encoding of them;
* xq_codes / xq_d          Q8_1 activation codes and scales for the integer identity;
* q6k_isums / q80_isums    integer sub-block sums computed from the gguf-recovered codes in int64:
                           Q6_K: sum over each 16-value sub-block of (code) * x_code * scale;
                           Q8_0: sum over each 32-value block of w_code * x_code.

The activation bytes are built here from seeded integers (not by the oracle), so the identity is
independent of the oracle's quantizer.
"""
from __future__ import annotations

import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ggml_formats.npz")


def main() -> None:
    rng = np.random.default_rng(20261201)
    n_in, n_out = 2048, 8

    # --- Q6_K: random bytes, nonzero scales, normal finite fp16 d ---
    nb = n_in // 256
    raw = rng.integers(0, 256, size=(n_out * nb, 210), dtype=np.uint8)
    sc = rng.integers(-128, 128, size=(n_out * nb, 16)).astype(np.int8)
    sc[sc == 0] = 1
    raw[:, 192:208] = sc.view(np.uint8)
    d = (rng.standard_normal(n_out * nb) * 0.01 + np.sign(rng.standard_normal(n_out * nb)) * 0.003).astype(np.float16)
    raw[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    raw = raw.reshape(n_out, nb * 210)
    deq = quants.dequantize(raw, T.Q6_K).astype(np.float32).reshape(n_out, n_in)
    scale = (d.astype(np.float32)[:, None] * sc.astype(np.float32)).reshape(n_out, nb, 16)
    codes = (deq.reshape(n_out, nb, 16, 16) / scale[..., None]).astype(np.float64)
    assert np.all(codes == np.round(codes)), "codes not exactly recovered"
    codes = codes.astype(np.int64).reshape(n_out, n_in)
    assert codes.min() >= -32 and codes.max() <= 31

    # --- Q8_0: gguf's encoder ---
    w = (rng.standard_normal((n_out, n_in)) * 0.02).astype(np.float32)
    q80 = quants.quantize(w, T.Q8_0).reshape(n_out, -1)
    q80_blocks = q80.reshape(n_out, n_in // 32, 34)
    q80_codes = q80_blocks[:, :, 2:].view(np.int8).astype(np.int64).reshape(n_out, n_in)

    # --- Q8_1 activation (two columns) from seeded integers ---
    ncols = 2
    xq_codes = rng.integers(-127, 128, size=(ncols, n_in)).astype(np.int8)
    xq_d = (np.abs(rng.standard_normal((ncols, n_in // 32))) * 0.02 + 0.001).astype(np.float16)
    xq_s = (rng.standard_normal((ncols, n_in // 32))).astype(np.float16)
    xq = np.zeros((ncols, n_in // 32, 36), np.uint8)
    xq[:, :, 0:2] = xq_d.view(np.uint8).reshape(ncols, -1, 2)
    xq[:, :, 2:4] = xq_s.view(np.uint8).reshape(ncols, -1, 2)
    xq[:, :, 4:] = xq_codes.view(np.uint8).reshape(ncols, -1, 32)

    # --- integer identities ---
    xc = xq_codes.astype(np.int64)
    sc_full = np.repeat(sc.astype(np.int64).reshape(n_out, nb * 16), 16, axis=1)  # per value
    prod6 = codes[None, :, :] * xc[:, None, :] * sc_full[None, :, :]
    q6k_isums = prod6.reshape(ncols, n_out, n_in // 16, 16).sum(axis=-1)
    prod8 = q80_codes[None, :, :] * xc[:, None, :]
    q80_isums = prod8.reshape(ncols, n_out, n_in // 32, 32).sum(axis=-1)

    np.savez_compressed(
        OUT,
        n_in=n_in, n_out=n_out, ncols=ncols,
        q6k_raw=raw.ravel(), q6k_deq=deq.ravel(), q6k_codes=codes.astype(np.int8).ravel(),
        q80_src=w.ravel(), q80_raw=q80.ravel(),
        xq=xq.ravel(), xq_codes=xq_codes.ravel(), xq_d=xq_d.view(np.uint16).ravel(),
        q6k_isums=q6k_isums.astype(np.int32).ravel(), q80_isums=q80_isums.astype(np.int32).ravel(),
        gguf_version=np.array("0.19.0"),
    )
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
