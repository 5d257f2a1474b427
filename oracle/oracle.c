/*
 * oracle.c — CPU restatement of the reference decode path. TEST INFRASTRUCTURE ONLY: the checker for
 * the CUDA kernels, never the product path.
 *
 * Reference source it restates (paths inside jollyroger1480/rapier):
 *   src/native_mmvq.cu  : Q8_1 quantizer :158-173, Q6_K dot :642-655 / :733-748, Q6_K GEMV :750-789,
 *                         Q8_0 dot :835-847, small GEMV :865-900, multi-column GEMV :1261-1356,
 *                         residual epilogues :3096-3185, host validation :2312-2331.
 *   src/fused_gdn.cu    : gdn_step_norm_kernel :39-111, gdn_conv_l2_kernel :113-133.
 *   src/qwythos.cpp     : argmax :70-84, split_qg :320-327, store_kv2 :340-345, gqa_head :380-442,
 *                         add_partials / row_sum_partials / rms_quant_apply / rms_norm_out :602-672,
 *                         swiglu_quant / sig_mul_quant / beta_gate :676-715.
 *
 * Third-party pieces that the reference #includes but does not ship (Strata fork, tag
 * port/qwythos-0.2.16 @ 79f278bb7; ggml formats from llama.cpp 3cf03257):
 *   - ggml block formats block_q6_K / block_q8_0 / block_q8_1 and dequantize_row_q6_K: restated from
 *     the published ggml format; PINNED by tests/golden against gguf-py 0.19.0.
 *   - q8_1_finite / q8_1_quant / q8_1_ds (strata/kernels/q8_1_finite.hpp): not in the tree. Written
 *     definition below (or_q8_finite_d, or_q8_quant, or_q8_ds_sum). PARITY UNPINNED for these rules.
 *   - rms_norm_weighted and native_rope_apply (Strata): not in the tree. Written definition below
 *     (or_rms_norm_rows, or_rope_*). PARITY UNPINNED for these rules.
 *
 * Arithmetic conventions: every fp32 operation is written explicitly (fmaf where the reference's
 * compiler contracts a multiply-add in the reference expression; -ffp-contract=off everywhere else);
 * exp, log1p and 1/sqrt are the exactly specified sequences below (or_expf, or_log1pf, 1/sqrtf), the
 * same sequences the CUDA kernels run, so outputs that pass through them are bit-exact too.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256
#define QK8 32

/* ------------------------------------------------------------------------------------------------ */
/* fp16 <-> fp32, round to nearest even (IEEE 754 binary16)                                          */
/* ------------------------------------------------------------------------------------------------ */
uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf or nan */
        if (ax > 0x7f800000u) return (uint16_t) (sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
        return (uint16_t) (sign | 0x7c00u);
    }
    if (ax >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u); /* rounds to >= 65520: overflow to inf */
    if (ax < 0x38800000u) { /* result is subnormal (or zero) in fp16 */
        if (ax < 0x33000000u) return (uint16_t) sign; /* < 2^-25: rounds to zero (2^-25 itself ties to 0) */
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e; /* 14..24 */
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) r += 1u;
        return (uint16_t) (sign | r);
    }
    /* normal */
    uint32_t r = ax - 0x38000000u; /* rebias exponent 127 -> 15 */
    const uint32_t rem = r & 0x1fffu;
    r >>= 13;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1u;
    return (uint16_t) (sign | r);
}

float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t) h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: normalize */
            e = 127 - 15 + 1;
            while ((m & 0x400u) == 0) { m <<= 1; e--; }
            m &= 0x3ffu;
            x = sign | (e << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void or_f32_to_f16_n(const float* x, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = or_f32_to_f16(x[i]);
}
void or_f16_to_f32_n(const uint16_t* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = or_f16_to_f32(x[i]);
}

/* ------------------------------------------------------------------------------------------------ */
/* Transcendentals with an exactly specified operation sequence (the CUDA kernels write the same      */
/* sequence, rapier_b200/csrc/common.cuh): every step is one IEEE-754 fp32 operation rounded to        */
/* nearest even (fmaf is the correctly rounded fused multiply-add), so both sides get the same bits.  */
/* The reference uses the vendor library (expf / __expf / log1pf / rsqrtf), whose last ulp is not      */
/* specified; these stay within ~1 ulp of the true value (tests compare with float64).               */
/*                                                                                                    */
/* or_expf: Cody-Waite reduction + Taylor polynomial (Cody & Waite, "Software Manual for the          */
/* Elementary Functions", 1980, ch. 6): n = rint(x log2 e); r = x - n C1 - n C2, C1 = 355/512 (exact    */
/* product), C2 = ln2 - C1; exp(r) = sum_{k<=7} r^k/k! by Horner with fmaf; times 2^(n/2) 2^(n - n/2).   */
/* or_logf: x = m 2^e, m in [sqrt(1/2), sqrt(2)); s = (m-1)/(m+1); log m = 2s(1 + s^2/3 + ... + s^10/11).  */
/* or_log1pf: u = 1 + t; t if u == 1 else log(u) t / (u - 1) (Goldberg 1991, Theorem 4).                */
/* ------------------------------------------------------------------------------------------------ */
static float f_from_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
static uint32_t f_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}
static float or_pow2i(int e) { return f_from_bits((uint32_t) (e + 127) << 23); }
float or_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return f_from_bits(0x7f800000u);
    if (x < -104.0f) return 0.0f;
    const float n = rintf(x * 1.44269502f);
    float r = fmaf(-n, 0.693359375f, x);
    r = fmaf(-n, -2.12194440e-4f, r);
    float p = 1.98412698e-4f;
    p = fmaf(p, r, 1.38888889e-3f);
    p = fmaf(p, r, 8.33333333e-3f);
    p = fmaf(p, r, 4.16666667e-2f);
    p = fmaf(p, r, 1.66666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int) n, n1 = ni / 2;
    return (p * or_pow2i(n1)) * or_pow2i(ni - n1);
}
float or_logf(float x) {
    int bias = 0;
    if (x < 1.17549435e-38f) {
        x = x * 16777216.0f;
        bias = -24;
    }
    const uint32_t bits = f_bits(x);
    int e = (int) ((bits >> 23) & 0xffu) - 127;
    float m = f_from_bits((bits & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421354f) {
        m = m * 0.5f;
        e += 1;
    }
    e += bias;
    const float s = (m - 1.0f) / (m + 1.0f);
    const float s2 = s * s;
    float q = 9.09090909e-2f;
    q = fmaf(q, s2, 1.11111111e-1f);
    q = fmaf(q, s2, 1.42857143e-1f);
    q = fmaf(q, s2, 2.00000000e-1f);
    q = fmaf(q, s2, 3.33333333e-1f);
    const float lm = fmaf((2.0f * s) * s2, q, 2.0f * s);
    const float fe = (float) e;
    return fmaf(fe, 0.693359375f, fmaf(fe, -2.12194440e-4f, lm));
}
float or_log1pf(float t) {
    if (t != t || t == f_from_bits(0x7f800000u)) return t;
    const float u = 1.0f + t;
    if (u == 1.0f) return t;
    return (or_logf(u) * t) / (u - 1.0f);
}
static float or_rsqrtf(float x) { return 1.0f / sqrtf(x); }
static float or_sigmoidf(float x) { return 1.0f / (1.0f + or_expf(-x)); }
static float or_siluf(float x) { return x / (1.0f + or_expf(-x)); }
void or_math_n(int fn, const float* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        switch (fn) {
            case 0: y[i] = or_expf(x[i]); break;
            case 1: y[i] = or_logf(x[i]); break;
            case 2: y[i] = or_log1pf(x[i]); break;
            case 3: y[i] = or_sigmoidf(x[i]); break;
            case 4: y[i] = or_siluf(x[i]); break;
            default: y[i] = or_rsqrtf(x[i]); break;
        }
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Seeded synthetic values. A counter-based generator so the CPU and the GPU produce the same bits:  */
/* value(i) = (sum of the four 16-bit fields of hash(seed, i) - 131070) * scale + mean, where scale   */
/* already folds sqrt(3)/65536 * std (the sum of four uniform u16 has std 65536/sqrt(3)). All float  */
/* steps are one IEEE multiply and one add, so any IEEE machine reproduces them.                     */
/* ------------------------------------------------------------------------------------------------ */
uint64_t or_hash64(uint64_t seed, uint64_t idx) {
    uint64_t z = seed * 0x9E3779B97F4A7C15ull + idx + 0x632BE59BD9B4E019ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void or_synth_normal(uint64_t seed, uint64_t offset, float scale, float mean, float* out, size_t n) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long) n; ++i) {
        const uint64_t h = or_hash64(seed, offset + (uint64_t) i);
        const int s = (int) (h & 0xffff) + (int) ((h >> 16) & 0xffff) + (int) ((h >> 32) & 0xffff) +
                      (int) ((h >> 48) & 0xffff) - 131070;
        const float v = (float) s * scale;
        out[i] = v + mean;
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Q8_1 (ggml block_q8_1: half2 {d, s}, int8 qs[32]) — src/native_mmvq.cu:158-173                     */
/* ------------------------------------------------------------------------------------------------ */
/* q8_1_finite (Strata q8_1_finite.hpp, out of tree): written definition — d that is NaN, infinite or
 * above the fp16 maximum is clamped to 65504, so the stored half stays finite. */
static float or_q8_finite_d(float d) {
    if (!(d <= 65504.0f)) return 65504.0f;
    return d;
}
/* q8_1_quant: written definition — 0 for an all-zero block, else roundf(x / d) clamped to [-127, 127]
 * (the clamp only matters when d was clamped by or_q8_finite_d; a NaN code becomes -127). */
static int8_t or_q8_quant(float x, float d, float amax) {
    if (amax == 0.0f) return 0;
    float q = roundf(x / d);
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    return (int8_t) q;
}
/* q8_1_ds: the block sum stored as half, clamped into the finite fp16 range (NaN stores 0). */
static float or_q8_ds_sum(float s) {
    if (s != s) return 0.0f;
    return fminf(fmaxf(s, -65504.0f), 65504.0f);
}

/* The 32-lane xor-butterfly reductions of the reference's warp_sum / warp_max (native_mmvq.cu:142-156):
 * level offsets 16, 8, 4, 2, 1; IEEE addition is commutative, so every lane ends with the same value. */
static float or_xor_sum32(const float* v) {
    float a[32], b[32];
    memcpy(a, v, sizeof a);
    for (int off = 16; off > 0; off >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ off];
        memcpy(a, b, sizeof a);
    }
    return a[0];
}
static float or_xor_max32(const float* v) {
    float a[32], b[32];
    memcpy(a, v, sizeof a);
    for (int off = 16; off > 0; off >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = fmaxf(a[l], a[l ^ off]);
        memcpy(a, b, sizeof a);
    }
    return a[0];
}

/* One Q8_1 block from 32 fp32 values: amax and sum by the warp trees, d = finite(amax / 127). */
static void or_q8_1_block(const float* v, uint8_t* blk) {
    float av[32];
    for (int l = 0; l < 32; ++l) av[l] = fabsf(v[l]);
    const float amax = or_xor_max32(av);
    const float sum = or_xor_sum32(v);
    const float d = or_q8_finite_d(amax / 127.0f);
    const uint16_t dh = or_f32_to_f16(d);
    const uint16_t sh = or_f32_to_f16(or_q8_ds_sum(sum));
    memcpy(blk, &dh, 2);
    memcpy(blk + 2, &sh, 2);
    for (int l = 0; l < 32; ++l) blk[4 + l] = (uint8_t) or_q8_quant(v[l], d, amax);
}

size_t or_q8_1_bytes(int n_in, int ncols) { return (size_t) ncols * (size_t) (n_in / 32) * 36u; }

void or_quantize_q8_1(const float* x, void* y, int n_in, int ncols) {
    const long long nb = (long long) n_in / 32 * ncols; /* columns are contiguous: one long vector */
    uint8_t* out = (uint8_t*) y;
#pragma omp parallel for schedule(static)
    for (long long b = 0; b < nb; ++b) or_q8_1_block(x + b * 32, out + b * 36);
}

void or_dequantize_q8_1(const void* y, float* x, int n) {
    const uint8_t* in = (const uint8_t*) y;
    for (int b = 0; b < n / 32; ++b) {
        uint16_t dh;
        memcpy(&dh, in + b * 36, 2);
        const float d = or_f16_to_f32(dh);
        for (int l = 0; l < 32; ++l) x[b * 32 + l] = d * (float) (int8_t) in[b * 36 + 4 + l];
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Weights: ggml block_q6_K {ql[128], qh[64], int8 scales[16], half d} (210 B / 256 values) and      */
/* block_q8_0 {half d, int8 qs[32]} (34 B / 32 values). src/native_mmvq.cu:98-116, :133-139.          */
/* ------------------------------------------------------------------------------------------------ */
size_t or_weight_bytes(int type, int n_in, int n_out) {
    if (type == 14) return (size_t) (n_in / 256) * 210u * (size_t) n_out;
    if (type == 13) return (size_t) (n_in / 256) * 176u * (size_t) n_out;
    if (type == 12) return (size_t) (n_in / 256) * 144u * (size_t) n_out;
    if (type == 8) return (size_t) (n_in / 32) * 34u * (size_t) n_out;
    return 0;
}

/* The unsigned 6-bit code of value v (0..255) of a Q6_K block, following ggml's dequantize_row_q6_K:
 * half h = v/128; within it j = (v%128)/32, l = v%32; low nibble from ql[64h + l + 32(j&1)] (nibble
 * j>>1), high two bits from qh[32h + l] bits 2j..2j+1. Scale index = v/16. */
static int q6k_code(const uint8_t* blk, int v) {
    const int h = v >> 7, vv = v & 127, j = vv >> 5, l = vv & 31;
    const uint8_t qlb = blk[64 * h + l + 32 * (j & 1)];
    const int lo = (j >> 1) ? (qlb >> 4) : (qlb & 15);
    const int hi = (blk[128 + 32 * h + l] >> (2 * j)) & 3;
    return lo | (hi << 4);
}
static void q6k_set_code(uint8_t* blk, int v, int code) {
    const int h = v >> 7, vv = v & 127, j = vv >> 5, l = vv & 31;
    uint8_t* qlb = &blk[64 * h + l + 32 * (j & 1)];
    if (j >> 1) *qlb = (uint8_t) ((*qlb & 0x0f) | ((code & 15) << 4));
    else *qlb = (uint8_t) ((*qlb & 0xf0) | (code & 15));
    uint8_t* qhb = &blk[128 + 32 * h + l];
    *qhb = (uint8_t) ((*qhb & ~(3 << (2 * j))) | (((code >> 4) & 3) << (2 * j)));
}
static float q6k_d(const uint8_t* blk) {
    uint16_t dh;
    memcpy(&dh, blk + 208, 2);
    return or_f16_to_f32(dh);
}

/* Synthetic Q6_K encoder (the reference ships none; this is this project's definition, reproduced
 * bit for bit by the device generator): per 16-value sub-block amax_j; d = half((max_j amax_j / 31)
 * / 127); scale_j = clamp(roundf((amax_j / 31) / d), 0, 127); code = clamp(roundf(x / (d * scale_j)),
 * -32, 31) + 32 (32 where d * scale_j == 0). */
static void q6k_encode_block(const float* x, uint8_t* blk) {
    memset(blk, 0, 210);
    float amax[16];
    float smax = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float a = 0.0f;
        for (int i = 0; i < 16; ++i) a = fmaxf(a, fabsf(x[16 * j + i]));
        amax[j] = a;
        smax = fmaxf(smax, a);
    }
    const uint16_t dbits = or_f32_to_f16((smax / 31.0f) / 127.0f);
    const float dh = or_f16_to_f32(dbits);
    memcpy(blk + 208, &dbits, 2);
    for (int j = 0; j < 16; ++j) {
        int sc = 0;
        if (dh > 0.0f) {
            const float s = roundf((amax[j] / 31.0f) / dh);
            sc = (int) fminf(fmaxf(s, 0.0f), 127.0f);
        }
        blk[192 + j] = (uint8_t) (int8_t) sc;
        const float eff = dh * (float) sc;
        for (int i = 0; i < 16; ++i) {
            int q = 0;
            if (eff > 0.0f) {
                const float r = roundf(x[16 * j + i] / eff);
                q = (int) fminf(fmaxf(r, -32.0f), 31.0f);
            }
            q6k_set_code(blk, 16 * j + i, q + 32);
        }
    }
}

/* ggml quantize_row_q8_0_ref: d = amax / 127, id = d ? 1/d : 0, q = roundf(x * id). */
static void q8_0_encode_block(const float* x, uint8_t* blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t dh = or_f32_to_f16(d);
    memcpy(blk, &dh, 2);
    for (int i = 0; i < 32; ++i) blk[2 + i] = (uint8_t) (int8_t) roundf(x[i] * id);
}

void or_quantize_weights(int type, const float* w, void* dst, int n_in, int n_out) {
    uint8_t* out = (uint8_t*) dst;
    if (type == 14) {
        const long long nb = (long long) n_out * (n_in / 256);
#pragma omp parallel for schedule(static)
        for (long long b = 0; b < nb; ++b) q6k_encode_block(w + b * 256, out + b * 210);
    } else if (type == 8) {
        const long long nb = (long long) n_out * (n_in / 32);
#pragma omp parallel for schedule(static)
        for (long long b = 0; b < nb; ++b) q8_0_encode_block(w + b * 32, out + b * 34);
    }
}

/* ggml dequantize_row_q6_K: y = d * scale * (code - 32), evaluated as (d * (float)scale) * (float)q. */
void or_dequantize_weights(int type, const void* w, float* dst, int n_in, int n_out) {
    const uint8_t* in = (const uint8_t*) w;
    if (type == 14) {
        const long long nb = (long long) n_out * (n_in / 256);
#pragma omp parallel for schedule(static)
        for (long long b = 0; b < nb; ++b) {
            const uint8_t* blk = in + b * 210;
            const float d = q6k_d(blk);
            for (int v = 0; v < 256; ++v) {
                const float ds = d * (float) (int8_t) blk[192 + v / 16];
                dst[b * 256 + v] = ds * (float) (q6k_code(blk, v) - 32);
            }
        }
    } else if (type == 8) {
        const long long nb = (long long) n_out * (n_in / 32);
#pragma omp parallel for schedule(static)
        for (long long b = 0; b < nb; ++b) {
            const uint8_t* blk = in + b * 34;
            uint16_t dh;
            memcpy(&dh, blk, 2);
            const float d = or_f16_to_f32(dh);
            for (int i = 0; i < 32; ++i) dst[b * 32 + i] = d * (float) (int8_t) blk[2 + i];
        }
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Packed tile layout (this project's lossless repack; defines rk_pack_weights). Requires            */
/* n_in % 1024 == 0 and n_out % 4 == 0. A tile covers 4 rows x 1024 values; tile (rt, kc) sits at      */
/* byte offset (rt * (n_in/1024) + kc) * TILE.                                                         */
/*   Q6_K (TILE = 3360 = 4 x 840):                                                                     */
/*     ql @0    [row 4][group 32][16 B]  int t (0..3), byte b: low nibble = code(4t+b),                */
/*                                       high nibble = code(16+4t+b) of the 32-value group             */
/*     qh @2048 [row 4][group 32][8 B]   int u (0..1), byte b, bits 2s..2s+1 = code(4(4u+s)+b) >> 4    */
/*     sc @3072 [group 32][row 4][2 B]   int8 scales of the group's two 16-value sub-blocks            */
/*     d  @3328 [superblock 4][row 4][2 B]  fp16 d                                                     */
/*   group g of a tile = super-block 4kc + g/8, values 32(g%8)..32(g%8)+31 of it.                      */
/*   Q8_0 (TILE = 4352 = 4 x 32 x 34):                                                                 */
/*     qs @0    [row 4][half 2][group 32][16 B]  int8 codes 16h..16h+15 of block 32kc + g              */
/*     d  @4096 [group 32][row 4][2 B]   fp16 d                                                        */
/* ------------------------------------------------------------------------------------------------ */
size_t or_packed_bytes(int type, int n_in, int n_out) {
    if (n_in % 1024 != 0 || n_out % 4 != 0) return 0;
    return or_weight_bytes(type, n_in, n_out);
}

static void q6k_pack_tile(const uint8_t* raw, int n_in, int rt, int kc, uint8_t* tile) {
    const int nb = n_in / 256;
    for (int r = 0; r < 4; ++r) {
        for (int g = 0; g < 32; ++g) {
            const int sb = 4 * kc + g / 8, gi = g % 8;
            const uint8_t* blk = raw + ((size_t) (4 * rt + r) * nb + sb) * 210;
            int code[32];
            for (int e = 0; e < 32; ++e) code[e] = q6k_code(blk, 32 * gi + e);
            /* A (16 B): byte 4t + b = code[4t + b] (6 bits) | (code[16 + 4t + b] >> 4) << 6;
             * B (8 B): byte 4u + b = low nibble of code[16 + 8u + b] | low nibble of code[20 + 8u + b] << 4 */
            uint8_t* qa = tile + (size_t) (r * 32 + g) * 16;
            for (int t = 0; t < 4; ++t)
                for (int b = 0; b < 4; ++b)
                    qa[4 * t + b] = (uint8_t) ((code[4 * t + b] & 63) | ((code[16 + 4 * t + b] >> 4) << 6));
            uint8_t* qb = tile + 2048 + (size_t) (r * 32 + g) * 8;
            for (int u = 0; u < 2; ++u)
                for (int b = 0; b < 4; ++b)
                    qb[4 * u + b] = (uint8_t) ((code[16 + 8 * u + b] & 15) | ((code[20 + 8 * u + b] & 15) << 4));
            uint8_t* sc = tile + 3072 + (size_t) (g * 4 + r) * 2;
            sc[0] = blk[192 + 2 * gi];
            sc[1] = blk[192 + 2 * gi + 1];
        }
        for (int s = 0; s < 4; ++s) {
            const uint8_t* blk = raw + ((size_t) (4 * rt + r) * nb + 4 * kc + s) * 210;
            memcpy(tile + 3328 + (size_t) (s * 4 + r) * 2, blk + 208, 2);
        }
    }
}

static void q6k_unpack_tile(const uint8_t* tile, int n_in, int rt, int kc, uint8_t* raw) {
    const int nb = n_in / 256;
    for (int r = 0; r < 4; ++r) {
        for (int g = 0; g < 32; ++g) {
            const int sb = 4 * kc + g / 8, gi = g % 8;
            uint8_t* blk = raw + ((size_t) (4 * rt + r) * nb + sb) * 210;
            const uint8_t* qa = tile + (size_t) (r * 32 + g) * 16;
            const uint8_t* qb = tile + 2048 + (size_t) (r * 32 + g) * 8;
            for (int e = 0; e < 32; ++e) {
                int code;
                if (e < 16) {
                    code = qa[e] & 63;
                } else {
                    const int T = (e - 16) / 4, b = e % 4;
                    code = ((qb[4 * (T / 2) + b] >> (4 * (T % 2))) & 15) | ((qa[4 * T + b] >> 6) << 4);
                }
                q6k_set_code(blk, 32 * gi + e, code);
            }
            const uint8_t* sc = tile + 3072 + (size_t) (g * 4 + r) * 2;
            blk[192 + 2 * gi] = sc[0];
            blk[192 + 2 * gi + 1] = sc[1];
        }
        for (int s = 0; s < 4; ++s) {
            uint8_t* blk = raw + ((size_t) (4 * rt + r) * nb + 4 * kc + s) * 210;
            memcpy(blk + 208, tile + 3328 + (size_t) (s * 4 + r) * 2, 2);
        }
    }
}

static void q80_pack_tile(const uint8_t* raw, int n_in, int rt, int kc, uint8_t* tile) {
    const int nb = n_in / 32;
    for (int r = 0; r < 4; ++r)
        for (int g = 0; g < 32; ++g) {
            const uint8_t* blk = raw + ((size_t) (4 * rt + r) * nb + 32 * kc + g) * 34;
            memcpy(tile + (size_t) ((r * 2 + 0) * 32 + g) * 16, blk + 2, 16);
            memcpy(tile + (size_t) ((r * 2 + 1) * 32 + g) * 16, blk + 18, 16);
            memcpy(tile + 4096 + (size_t) (g * 4 + r) * 2, blk, 2);
        }
}

static void q80_unpack_tile(const uint8_t* tile, int n_in, int rt, int kc, uint8_t* raw) {
    const int nb = n_in / 32;
    for (int r = 0; r < 4; ++r)
        for (int g = 0; g < 32; ++g) {
            uint8_t* blk = raw + ((size_t) (4 * rt + r) * nb + 32 * kc + g) * 34;
            memcpy(blk + 2, tile + (size_t) ((r * 2 + 0) * 32 + g) * 16, 16);
            memcpy(blk + 18, tile + (size_t) ((r * 2 + 1) * 32 + g) * 16, 16);
            memcpy(blk, tile + 4096 + (size_t) (g * 4 + r) * 2, 2);
        }
}

int or_pack_weights(int type, const void* src, void* dst, int n_in, int n_out) {
    if (or_packed_bytes(type, n_in, n_out) == 0 || (type != 14 && type != 8)) return -1;
    const int KC = n_in / 1024;
    const size_t tile = type == 14 ? 3360 : 4352;
    const long long nt = (long long) (n_out / 4) * KC;
#pragma omp parallel for schedule(static)
    for (long long t = 0; t < nt; ++t) {
        const int rt = (int) (t / KC), kc = (int) (t % KC);
        uint8_t* out = (uint8_t*) dst + (size_t) t * tile;
        if (type == 14) q6k_pack_tile((const uint8_t*) src, n_in, rt, kc, out);
        else q80_pack_tile((const uint8_t*) src, n_in, rt, kc, out);
    }
    return 0;
}

int or_unpack_weights(int type, const void* src, void* dst, int n_in, int n_out) {
    if (or_packed_bytes(type, n_in, n_out) == 0 || (type != 14 && type != 8)) return -1;
    const int KC = n_in / 1024;
    const size_t tile = type == 14 ? 3360 : 4352;
    const long long nt = (long long) (n_out / 4) * KC;
    if (type == 14) memset(dst, 0, or_weight_bytes(type, n_in, n_out)); /* set_code read-modify-writes */
#pragma omp parallel for schedule(static)
    for (long long t = 0; t < nt; ++t) {
        const int rt = (int) (t / KC), kc = (int) (t % KC);
        const uint8_t* in = (const uint8_t*) src + (size_t) t * tile;
        if (type == 14) q6k_unpack_tile(in, n_in, rt, kc, (uint8_t*) dst);
        else q80_unpack_tile(in, n_in, rt, kc, (uint8_t*) dst);
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------------ */
/* GEMV restatement                                                                                  */
/* ------------------------------------------------------------------------------------------------ */
static int32_t load_i32(const uint8_t* p) { /* load_int_b2: two little-endian u16 */
    uint16_t a, b;
    memcpy(&a, p, 2);
    memcpy(&b, p + 2, 2);
    return (int32_t) ((uint32_t) a | ((uint32_t) b << 16));
}
static int dp4a_ss(int32_t a, int32_t b, int c) {
    for (int i = 0; i < 4; ++i) c += (int) (int8_t) (a >> (8 * i)) * (int) (int8_t) (b >> (8 * i));
    return c;
}
/* __vsubss4(x, 0x20202020) on bytes 0..63: plain per-byte subtraction (nothing saturates). */
static int32_t sub32_bytes(int32_t x) {
    uint32_t r = 0;
    for (int i = 0; i < 4; ++i) {
        const int v = (int) ((x >> (8 * i)) & 0xff) - 32;
        r |= ((uint32_t) (uint8_t) (int8_t) v) << (8 * i);
    }
    return (int32_t) r;
}
static float q81_d(const uint8_t* blk) {
    uint16_t h;
    memcpy(&h, blk, 2);
    return or_f16_to_f32(h);
}

/* q6_q8_dot (native_mmvq.cu:733-748) + q6_q8_dot_impl (:642-655) for one lane iqs of one block.
 * isum_out (optional) receives the two integer products dp4a(vi, u) * sc. */
static float q6_q8_dot(const uint8_t* blk, const uint8_t* x, int iqs, int* isum_out) {
    const int bq8_offset = 4 * (iqs / 16) + (iqs % 16) / 8;
    const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
    const int vh_shift = 2 * ((iqs % 16) / 8);
    const int32_t vl = load_i32(blk + 4 * iqs);
    const int32_t vh = (int32_t) ((uint32_t) load_i32(blk + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift);
    const float d = q6k_d(blk);
    float sumf = 0.0f;
    for (int i = 0; i < 2; ++i) {
        const uint8_t* xb = x + (size_t) (bq8_offset + 2 * i) * 36;
        const int32_t u = load_i32(xb + 4 + 4 * (iqs % 8));
        const float d8 = q81_d(xb);
        const int sc = (int8_t) blk[192 + scale_offset + 4 * i];
        const int32_t vil = (int32_t) (((uint32_t) vl >> (4 * i)) & 0x0f0f0f0fu);
        const int32_t vih = (int32_t) ((((uint32_t) vh >> (4 * i)) << 4) & 0x30303030u);
        const int32_t vi = sub32_bytes(vil | vih);
        const int p = dp4a_ss(vi, u, 0) * sc;
        if (isum_out) isum_out[i] = p;
        sumf = fmaf(d8, (float) p, sumf);
    }
    return d * sumf;
}

/* small_q8_dot for Q8_0 (native_mmvq.cu:835-847): kqs = 2*(tid%4), two ints per thread. */
static float q80_q8_dot(const uint8_t* blk, const uint8_t* xb, int iqs, int* isum_out) {
    int sumi = 0;
    for (int i = 0; i < 2; ++i) {
        const int32_t v = load_i32(blk + 2 + 4 * (iqs + i));
        const int32_t u = load_i32(xb + 4 + 4 * (iqs + i));
        sumi = dp4a_ss(v, u, sumi);
    }
    if (isum_out) *isum_out = sumi;
    uint16_t dh;
    memcpy(&dh, blk, 2);
    const float d0 = or_f16_to_f32(dh);
    const float d1 = q81_d(xb);
    return d0 * d1 * (float) sumi;
}

/* ---- Q5_K / Q4_K (ggml's K-quants with a per-32-value 6-bit scale and min) ----
 * Block: half2 dm {d, dmin}, scales[12], (Q5_K: qh[32]), qs[128]; 256 values in 8 sub-blocks of 32.
 * Sub-block j's (scale, min) are ggml's get_scale_min_k4: j < 4: (s[j] & 63, s[j+4] & 63); else
 * ((s[j+4] & 15) | ((s[j-4] >> 6) << 4), (s[j+4] >> 4) | ((s[j] >> 6) << 4)). Value k of sub-block j:
 * low 4 bits = nibble (j & 1) of qs[32 * (j / 2) + k]; Q5_K's fifth bit = bit j of qh[k];
 * value = d * scale * code - dmin * min. */
static void kq_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}
static int kq_code(int type, const uint8_t* blk, int v) {
    const int j = v / 32, k = v % 32;
    const uint8_t* qs = blk + (type == 13 ? 48 : 16);
    int code = (qs[32 * (j / 2) + k] >> (4 * (j & 1))) & 15;
    if (type == 13) code |= ((blk[16 + k] >> j) & 1) << 4;
    return code;
}
void or_dequant_kq(int type, const void* w, float* y, int n_values) {
    const size_t bb = type == 13 ? 176u : 144u;
    for (int b = 0; b < n_values / 256; ++b) {
        const uint8_t* blk = (const uint8_t*) w + bb * (size_t) b;
        uint16_t h[2];
        memcpy(h, blk, 4);
        const float d = or_f16_to_f32(h[0]), dmin = or_f16_to_f32(h[1]);
        for (int v = 0; v < 256; ++v) {
            int sc, m;
            kq_scale_min(blk + 4, v / 32, &sc, &m);
            y[b * 256 + v] = d * (float) sc * (float) kq_code(type, blk, v) - dmin * (float) m;
        }
    }
}

/* vec_dot_q5_K_q8_1 / vec_dot_q4_K_q8_1 as the reference pins them (native_mmvq.cu:191-252, :543-595):
 * thread iqs (even, 0..30) covers sub-blocks bq8 = 2 * ((iqs / 2) / 4) and bq8 + 1, and within each the
 * ints (iqs / 2) % 4 and + 4 of the Q8_1 block (8 values). Per sub-block i: dot1 = sum(code * q8),
 * dot2 = sum(q8) (dp4a chains in the reference's order), sumf_d += d8 * (dot1 * sc), sumf_m += d8 *
 * (dot2 * m); the result d * sumf_d - dmin * sumf_m. isum_out (optional): dot1 * sc, dot2 * m per i. */
static float kq_q8_dot(int type, const uint8_t* blk, const uint8_t* x, int iqs, int* isum_out) {
    const int bq8 = 2 * ((iqs / 2) / 4), k4 = (iqs / 2) % 4;
    const uint8_t* qs = blk + (type == 13 ? 48 : 16);
    const int32_t vl0 = load_i32(qs + 16 * bq8 + 4 * k4), vl1 = load_i32(qs + 16 * bq8 + 4 * k4 + 16);
    int32_t vh0 = 0, vh1 = 0;
    if (type == 13) {
        vh0 = (int32_t) ((uint32_t) load_i32(blk + 16 + 4 * k4) >> bq8);
        vh1 = (int32_t) ((uint32_t) load_i32(blk + 16 + 4 * k4 + 16) >> bq8);
    }
    uint16_t h[2];
    memcpy(h, blk, 4);
    const float d = or_f16_to_f32(h[0]), dmin = or_f16_to_f32(h[1]);
    float sumf_d = 0.0f, sumf_m = 0.0f;
    for (int i = 0; i < 2; ++i) {
        int sc, m;
        kq_scale_min(blk + 4, bq8 + i, &sc, &m);
        const uint8_t* xb = x + (size_t) (bq8 + i) * 36;
        const int32_t u0 = load_i32(xb + 4 + 4 * k4), u1 = load_i32(xb + 4 + 4 * k4 + 16);
        int32_t v0 = (int32_t) (((uint32_t) vl0 >> (4 * i)) & 0x0f0f0f0fu);
        int32_t v1 = (int32_t) (((uint32_t) vl1 >> (4 * i)) & 0x0f0f0f0fu);
        if (type == 13) {
            v0 |= (int32_t) ((((uint32_t) vh0 >> i) << 4) & 0x10101010u);
            v1 |= (int32_t) ((((uint32_t) vh1 >> i) << 4) & 0x10101010u);
        }
        /* Q5_K chains v0 into v1 (the reference's dp4a(v0, u0, dp4a(v1, u1, 0))); Q4_K v1 into v0 */
        const int dot1 = type == 13 ? dp4a_ss(v0, u0, dp4a_ss(v1, u1, 0)) : dp4a_ss(v1, u1, dp4a_ss(v0, u0, 0));
        const int dot2 = type == 13 ? dp4a_ss(0x01010101, u0, dp4a_ss(0x01010101, u1, 0))
                                    : dp4a_ss(0x01010101, u1, dp4a_ss(0x01010101, u0, 0));
        const float d8 = q81_d(xb);
        if (isum_out) {
            isum_out[2 * i] = dot1 * sc;
            isum_out[2 * i + 1] = dot2 * m;
        }
        sumf_d += d8 * (float) (dot1 * sc);
        sumf_m += d8 * (float) (dot2 * m);
    }
    return d * sumf_d - dmin * sumf_m;
}

/* Per row and column, the reference's reduction order: 4 warps x 32 lanes; warp w walks blocks
 * w, w+4, ... (Q6_K) and accumulates per lane; warps 1..3 add into warp 0 in order; then the xor tree.
 * (Q8_0 with n_in/32 >= 32: one row per block, kbx = tid/4 step 32, kqs = 2*(tid%4).) */
static float or_row_dot(int type, const uint8_t* wrow, const uint8_t* xcol, int n_in) {
    float tmp[4][32];
    for (int w = 0; w < 4; ++w)
        for (int l = 0; l < 32; ++l) {
            const int tid = 32 * w + l;
            float acc = 0.0f;
            if (type == 14) {
                const int nb = n_in / 256;
                for (int kbx = tid / 32; kbx < nb; kbx += 4) {
                    const float f = q6_q8_dot(wrow + (size_t) kbx * 210, xcol + (size_t) kbx * 8 * 36, tid % 32, NULL);
                    acc = acc + f;
                }
            } else if (type == 13 || type == 12) { /* QI 32, VDR 2: kbx = tid/16 step 8, kqs = 2*(tid%16) */
                const int nb = n_in / 256;
                for (int kbx = tid / 16; kbx < nb; kbx += 8) {
                    const float f = kq_q8_dot(type, wrow + (size_t) kbx * (type == 13 ? 176 : 144),
                                              xcol + (size_t) kbx * 8 * 36, 2 * (tid % 16), NULL);
                    acc = acc + f;
                }
            } else { /* kbx = tid/4 step 32 for both SmallK variants (they differ only in rows per block) */
                const int nb = n_in / 32;
                for (int kbx = tid / 4; kbx < nb; kbx += 32) {
                    const float f = q80_q8_dot(wrow + (size_t) kbx * 34, xcol + (size_t) kbx * 36, 2 * (tid % 4), NULL);
                    acc = acc + f;
                }
            }
            tmp[w][l] = acc;
        }
    for (int l = 0; l < 32; ++l)
        for (int w = 1; w < 4; ++w) tmp[0][l] = tmp[0][l] + tmp[w][l];
    return or_xor_sum32(tmp[0]);
}

void or_mmvq(int type, const void* w, const void* xq, float* y, int n_in, int n_out, int ncols) {
    const size_t rb = or_weight_bytes(type, n_in, 1);
    const size_t xb = or_q8_1_bytes(n_in, 1);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n_out; ++r)
        for (int j = 0; j < ncols; ++j)
            y[(size_t) j * n_out + r] =
                or_row_dot(type, (const uint8_t*) w + rb * r, (const uint8_t*) xq + xb * j, n_in);
}

/* Residual epilogue (native_mmvq.cu:3096-3185): y[r] = acc + res[r]; partials[r/4] = sum over the 4
 * rows of y^2, accumulated in row order. Column j uses y + j*n_out, res + j*n_out and
 * partials + j*ceil(n_out/4). */
void or_mmvq_res(int type, const void* w, const void* xq, float* y, const float* res, float* partials,
                 int n_in, int n_out, int ncols) {
    const size_t rb = or_weight_bytes(type, n_in, 1);
    const size_t xb = or_q8_1_bytes(n_in, 1);
    const int nslots = (n_out + 3) / 4;
    for (int j = 0; j < ncols; ++j) {
#pragma omp parallel for schedule(static)
        for (int s = 0; s < nslots; ++s) {
            float p = 0.0f;
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * s + i;
                if (r >= n_out) break;
                const float acc = or_row_dot(type, (const uint8_t*) w + rb * r, (const uint8_t*) xq + xb * j, n_in);
                const float v = acc + res[(size_t) j * n_out + r];
                y[(size_t) j * n_out + r] = v;
                p = fmaf(v, v, p);
            }
            partials[(size_t) j * nslots + s] = p;
        }
    }
}

/* The same GEMV in the summation order of the packed-tile kernel (rk_pack_weights' tiles of 4 rows x 1024
 * values): lane l of the row's warp takes 32-value group g = 32 kc + l of every 1024-value chunk kc; per
 * group the two 16-value sub-block sums (code - 32) * x times their int8 scales are added as integers
 * (exact), then acc = fmaf((float) isum, d8 * d, acc) over kc in order (d8 the group's Q8_1 scale, d the
 * row's super-block scale; Q8_0: the 32-value integer dot, d its block scale). With an even chunk count
 * KC >= 2 the chain runs separately over each half, kc < KC/2 and kc >= KC/2 (two warps can take the
 * halves), and the lane's value is lo + hi. The lanes are added by the 32-lane xor tree. Same integers as
 * the reference order above, different fp32 rounding (a few ulp): this is the order the decode engine's
 * GEMVs run in. Q6_K and Q8_0, n_in % 1024 == 0. */
static float packed_row_dot(int type, const uint8_t* wrow, const uint8_t* xcol, int n_in) {
    float lanes[32];
    const int KC = n_in / 1024;
    const int split = KC >= 2 && KC % 2 == 0 ? KC / 2 : KC;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f, lo = 0.0f;
        for (int kc = 0; kc < KC; ++kc) {
            if (kc == split) {
                lo = acc;
                acc = 0.0f;
            }
            const int g = 32 * kc + l;
            const uint8_t* xb = xcol + (size_t) g * 36;
            const int8_t* xq = (const int8_t*) (xb + 4);
            const float d8 = q81_d(xb);
            int isum;
            float d;
            if (type == 14) {
                const uint8_t* blk = wrow + (size_t) (g / 8) * 210;
                const int v0 = (g % 8) * 32;
                int s0 = 0, s1 = 0;
                for (int i = 0; i < 16; ++i) s0 += (q6k_code(blk, v0 + i) - 32) * xq[i];
                for (int i = 16; i < 32; ++i) s1 += (q6k_code(blk, v0 + i) - 32) * xq[i];
                isum = s0 * (int) (int8_t) blk[192 + (g % 8) * 2] + s1 * (int) (int8_t) blk[192 + (g % 8) * 2 + 1];
                d = q6k_d(blk);
            } else {
                const uint8_t* blk = wrow + (size_t) g * 34;
                int sd = 0;
                for (int i = 0; i < 32; ++i) sd += (int) (int8_t) blk[2 + i] * xq[i];
                isum = sd;
                uint16_t hb;
                memcpy(&hb, blk, 2);
                d = or_f16_to_f32(hb);
            }
            acc = fmaf((float) isum, d8 * d, acc);
        }
        lanes[l] = split < KC ? lo + acc : acc;
    }
    return or_xor_sum32(lanes);
}
void or_mmvq_packed(int type, const void* w, const void* xq, float* y, const float* res, float* partials, int n_in,
                    int n_out, int ncols) {
    const size_t rb = or_weight_bytes(type, n_in, 1);
    const size_t xb = or_q8_1_bytes(n_in, 1);
    const int nslots = (n_out + 3) / 4;
    for (int j = 0; j < ncols; ++j) {
#pragma omp parallel for schedule(static)
        for (int s = 0; s < nslots; ++s) {
            float p = 0.0f;
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * s + i;
                if (r >= n_out) break;
                float v = packed_row_dot(type, (const uint8_t*) w + rb * r, (const uint8_t*) xq + xb * j, n_in);
                if (res) v = v + res[(size_t) j * n_out + r];
                y[(size_t) j * n_out + r] = v;
                p = fmaf(v, v, p);
            }
            if (partials) partials[(size_t) j * nslots + s] = p;
        }
    }
}

/* Exact integer sums, the bit-exact parity target. Layout out[((j * n_out) + r) * nsub + s]:
 *   Q6_K: nsub = n_in/16, s = 16-value sub-block: sum over its 16 values of (code-32) * x_code * scale
 *         (the sum of the reference's per-lane dp4a(vi, u) * sc over the four lanes that cover it);
 *   Q8_0: nsub = n_in/32, s = 32-value block: sum of w_code * x_code;
 *   Q5_K / Q4_K: nsub = 2 * n_in/32, entries 2s and 2s+1 of 32-value sub-block s: the sums of dot1 * scale
 *         and dot2 * min over the four threads that cover it. */
void or_mmvq_isums(int type, const void* w, const void* xq, int32_t* out, int n_in, int n_out, int ncols) {
    const size_t rb = or_weight_bytes(type, n_in, 1);
    const size_t xbytes = or_q8_1_bytes(n_in, 1);
    const int nsub = type == 14 ? n_in / 16 : (type == 13 || type == 12) ? 2 * (n_in / 32) : n_in / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n_out; ++r)
        for (int j = 0; j < ncols; ++j) {
            const uint8_t* wrow = (const uint8_t*) w + rb * r;
            const uint8_t* xcol = (const uint8_t*) xq + xbytes * j;
            int32_t* o = out + ((size_t) j * n_out + r) * nsub;
            for (int s = 0; s < nsub; ++s) o[s] = 0;
            if (type == 14) {
                for (int kbx = 0; kbx < n_in / 256; ++kbx)
                    for (int iqs = 0; iqs < 32; ++iqs) {
                        int p[2];
                        q6_q8_dot(wrow + (size_t) kbx * 210, xcol + (size_t) kbx * 8 * 36, iqs, p);
                        /* lane iqs, half i covers values of Q8 block bq8_offset + 2i, ints iqs%8 -> the
                         * 16-value sub-block index is scale_offset + 4i within the super-block */
                        const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
                        for (int i = 0; i < 2; ++i) o[kbx * 16 + scale_offset + 4 * i] += p[i];
                    }
            } else if (type == 13 || type == 12) {
                /* per 32-value sub-block s: (sum of dot1 * sc, sum of dot2 * m) over the four threads */
                for (int kbx = 0; kbx < n_in / 256; ++kbx)
                    for (int iqs = 0; iqs < 32; iqs += 2) {
                        int p[4];
                        kq_q8_dot(type, wrow + (size_t) kbx * (type == 13 ? 176 : 144), xcol + (size_t) kbx * 8 * 36, iqs, p);
                        const int bq8 = 2 * ((iqs / 2) / 4);
                        for (int i = 0; i < 2; ++i) {
                            o[2 * (kbx * 8 + bq8 + i)] += p[2 * i];
                            o[2 * (kbx * 8 + bq8 + i) + 1] += p[2 * i + 1];
                        }
                    }
            } else {
                for (int kbx = 0; kbx < n_in / 32; ++kbx)
                    for (int iqs = 0; iqs < 8; iqs += 2) {
                        int p;
                        q80_q8_dot(wrow + (size_t) kbx * 34, xcol + (size_t) kbx * 36, iqs, &p);
                        o[kbx] += p;
                    }
            }
        }
}

/* ------------------------------------------------------------------------------------------------ */
/* Norms and elementwise (src/qwythos.cpp:602-715)                                                   */
/* ------------------------------------------------------------------------------------------------ */
/* row_sum_partials_kernel :616-623 — partials[b] = sum of x^2 over rows 4b..4b+3, in row order. */
void or_row_sumsq_partials(const float* x, float* partials, int n) {
    for (int b = 0; b < (n + 3) / 4; ++b) {
        float p = 0.0f;
        for (int i = 4 * b; i < 4 * b + 4 && i < n; ++i) p = fmaf(x[i], x[i], p);
        partials[b] = p;
    }
}
/* add_partials_1024_kernel :602-614 — x += o, partials of the new x. */
void or_add_partials(float* x, const float* o, float* partials, int n) {
    for (int b = 0; b < (n + 3) / 4; ++b) {
        float p = 0.0f;
        for (int i = 4 * b; i < 4 * b + 4 && i < n; ++i) {
            const float v = x[i] + o[i];
            x[i] = v;
            p = fmaf(v, v, p);
        }
        partials[b] = p;
    }
}
/* The block reduction of rms_quant_apply_kernel :634-641 over nslots partials with 256 threads:
 * thread t sums slots t, t+256, ... in order; shfl_down tree inside each warp (lane 0 receives
 * ((l0 + l16) + (l8 + l24)) ... ), then red[0] + ... + red[7] in order. */
float or_partials_sumsq(const float* partials, int nslots) {
    float part[256];
    for (int t = 0; t < 256; ++t) {
        float a = 0.0f;
        for (int p = t; p < nslots; p += 256) a = a + partials[p];
        part[t] = a;
    }
    float red[8];
    for (int w = 0; w < 8; ++w) {
        float v[32];
        memcpy(v, part + 32 * w, sizeof v);
        for (int off = 16; off > 0; off >>= 1)
            for (int l = 0; l + off < 32; ++l) v[l] = v[l] + v[l + off]; /* shfl_down: lane l += lane l+off */
        red[w] = v[0];
    }
    float ss = red[0];
    for (int w = 1; w < 8; ++w) ss = ss + red[w];
    return ss;
}
/* rms_quant_apply_kernel :627-655 — inv = rsqrt(ss/cols + eps); v = x * w * inv; Q8_1 of v. */
void or_rms_quant_q8_1(const float* x, const float* w, const float* partials, void* y, int cols, float eps) {
    const float ss = or_partials_sumsq(partials, cols / 4);
    const float inv = 1.0f / sqrtf(ss / (float) cols + eps);
    float v[32];
    for (int b = 0; b < cols / 32; ++b) {
        for (int l = 0; l < 32; ++l) v[l] = x[32 * b + l] * w[32 * b + l] * inv;
        or_q8_1_block(v, (uint8_t*) y + (size_t) b * 36);
    }
}
/* rms_norm_out_kernel :658-672 — out = x * w * inv. */
void or_rms_norm_out(const float* x, const float* w, const float* partials, float* out, int cols, float eps) {
    const float ss = or_partials_sumsq(partials, cols / 4);
    const float inv = 1.0f / sqrtf(ss / (float) cols + eps);
    for (int i = 0; i < cols; ++i) out[i] = x[i] * w[i] * inv;
}
/* swiglu_quant_kernel :676-689 — v = g / (1 + exp(-g)) * up. */
void or_swiglu_q8_1(const float* up, const float* gate, void* y, int n) {
    float v[32];
    for (int b = 0; b < n / 32; ++b) {
        for (int l = 0; l < 32; ++l) {
            const float g = gate[32 * b + l];
            v[l] = or_siluf(g) * up[32 * b + l];
        }
        or_q8_1_block(v, (uint8_t*) y + (size_t) b * 36);
    }
}
/* sig_mul_quant_kernel :692-704 — v = o * (1 / (1 + exp(-g))). */
void or_sigmul_q8_1(const float* o, const float* g, void* y, int n) {
    float v[32];
    for (int b = 0; b < n / 32; ++b) {
        for (int l = 0; l < 32; ++l) v[l] = o[32 * b + l] * or_sigmoidf(g[32 * b + l]);
        or_q8_1_block(v, (uint8_t*) y + (size_t) b * 36);
    }
}
/* beta_gate_kernel :707-715 — beta = sigmoid(beta); gate = softplus(alpha + dt) * ssm_a, softplus
 * passes v through above 20. */
void or_beta_gate(float* beta, const float* alpha, const float* dt, const float* ssm_a, float* gate, int n) {
    for (int i = 0; i < n; ++i) {
        beta[i] = or_sigmoidf(beta[i]);
        const float v = alpha[i] + dt[i];
        gate[i] = (v > 20.0f ? v : or_log1pf(or_expf(v))) * ssm_a[i];
    }
}
/* rms_norm_weighted (Strata, out of tree; called at src/qwythos.cpp:1206-1207): written definition —
 * per row of `cols`: ss = sum of x^2 in index order, inv = 1/sqrt(ss/cols + eps), x = x * inv * w. */
void or_rms_norm_rows(float* x, const float* w, int rows, int cols, float eps) {
    for (int r = 0; r < rows; ++r) {
        float* p = x + (size_t) r * cols;
        float ss = 0.0f;
        for (int i = 0; i < cols; ++i) ss = fmaf(p[i], p[i], ss);
        const float inv = 1.0f / sqrtf(ss / (float) cols + eps);
        for (int i = 0; i < cols; ++i) p[i] = p[i] * inv * w[i];
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Gated DeltaNet (src/fused_gdn.cu)                                                                 */
/* ------------------------------------------------------------------------------------------------ */
/* gdn_conv_l2_kernel :113-133, with the conv history kept as a 4-slot ring per channel
 * ring[c*4 + (p & 3)] = input at position p; the three taps before position pos are the slots of
 * pos-3, pos-2, pos-1 (oldest first), which is the reference's [v0, v1, v2] history after its slide.
 * sum = v0*w0 + v1*w1 + v2*w2 + x*w3 as fused multiply-adds in that order; y = sum / (1 + exp(-sum));
 * the first qk_heads 128-channel heads are scaled by 1/sqrt(sum_head y^2 + eps), the head sum taken
 * as four 32-lane xor trees added in order. */
void or_gdn_conv_l2(float* ring, const float* qkv, const float* conv_w, float* h, int channels, int qk_heads,
                    float eps, int pos) {
    float* y = (float*) malloc(sizeof(float) * (size_t) channels);
    for (int c = 0; c < channels; ++c) {
        const float* rc = ring + (size_t) c * 4;
        const float v0 = rc[(pos + 1) & 3], v1 = rc[(pos + 2) & 3], v2 = rc[(pos + 3) & 3];
        const float x = qkv[c];
        const float* w = conv_w + (size_t) c * 4;
        float sum = v0 * w[0];
        sum = fmaf(v1, w[1], sum);
        sum = fmaf(v2, w[2], sum);
        sum = fmaf(x, w[3], sum);
        y[c] = or_siluf(sum);
    }
    for (int c = 0; c < channels; ++c) ring[(size_t) c * 4 + (pos & 3)] = qkv[c];
    for (int hh = 0; hh < channels / 128; ++hh) {
        float* yh = y + (size_t) hh * 128;
        if (hh < qk_heads) {
            float part[4];
            for (int w = 0; w < 4; ++w) {
                float sq[32];
                for (int l = 0; l < 32; ++l) sq[l] = yh[32 * w + l] * yh[32 * w + l];
                part[w] = or_xor_sum32(sq);
            }
            const float ss = ((part[0] + part[1]) + part[2]) + part[3];
            const float inv = 1.0f / sqrtf(ss + eps);
            for (int i = 0; i < 128; ++i) h[(size_t) hh * 128 + i] = yh[i] * inv;
        } else {
            for (int i = 0; i < 128; ++i) h[(size_t) hh * 128 + i] = yh[i];
        }
    }
    free(y);
}

/* gdn_step_norm_kernel<SILU=true, WithQ8=true> :39-111. State layout [128 (k row i)][h_v][128 (v col j)].
 * v-head h pairs with k/q head h % h_k. Per column j the four 32-row groups accumulate with fmaf in row
 * order and are added group 0..3 in order. */
void or_gdn_step_norm_silu_q8(float* state, const float* q, const float* k, const float* v, const float* gate,
                              const float* beta, const float* z, const float* gamma, float eps, float* y,
                              void* q8, int h_k, int h_v) {
    const int S = 128;
    for (int head = 0; head < h_v; ++head) {
        const int qh = head % h_k;
        const float* sk = k + (size_t) qh * S;
        const float* sq = q + (size_t) qh * S;
        const float g = or_expf(gate[head]);
        float oc[128];
        for (int col = 0; col < S; ++col) {
            float kv[4], o[4];
            for (int rg = 0; rg < 4; ++rg) {
                float a = 0.0f;
                for (int r = 0; r < 32; ++r) {
                    const int i = rg * 32 + r;
                    a = fmaf(state[((size_t) i * h_v + head) * S + col], sk[i], a);
                }
                kv[rg] = a;
            }
            const float kv_col = ((kv[0] + kv[1]) + kv[2]) + kv[3];
            const float delta = (v[(size_t) head * S + col] - g * kv_col) * beta[head];
            for (int rg = 0; rg < 4; ++rg) {
                float a = 0.0f;
                for (int r = 0; r < 32; ++r) {
                    const int i = rg * 32 + r;
                    float* s = &state[((size_t) i * h_v + head) * S + col];
                    *s = fmaf(g, *s, sk[i] * delta);
                    a = fmaf(*s, sq[i], a);
                }
                o[rg] = a;
            }
            oc[col] = (((o[0] + o[1]) + o[2]) + o[3]) * (1.0f / sqrtf((float) S));
        }
        float part[4];
        for (int w = 0; w < 4; ++w) {
            float sq2[32];
            for (int l = 0; l < 32; ++l) sq2[l] = oc[32 * w + l] * oc[32 * w + l];
            part[w] = or_xor_sum32(sq2);
        }
        const float ss = ((part[0] + part[1]) + part[2]) + part[3];
        const float scale = 1.0f / sqrtf(ss / (float) S + eps);
        float yv[128];
        for (int col = 0; col < S; ++col) {
            const float zz = z[(size_t) head * S + col];
            const float gate_z = or_siluf(zz);
            yv[col] = oc[col] * scale * gamma[col] * gate_z;
            y[(size_t) head * S + col] = yv[col];
        }
        if (q8)
            for (int b = 0; b < 4; ++b) or_q8_1_block(yv + 32 * b, (uint8_t*) q8 + ((size_t) head * 4 + b) * 36);
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Attention                                                                                          */
/* ------------------------------------------------------------------------------------------------ */
/* native_rope_apply (Strata, out of tree; src/qwythos.cpp:1210-1211): written definition — NEOX
 * rotate-half over the first n_rot dims of each head, pairs (i, i + n_rot/2), angle = pos *
 * base^(-2i/n_rot). The cos/sin table is built in double precision and stored as float:
 * table[(pos * (n_rot/2) + i) * 2 + {0: cos, 1: sin}]. */
void or_rope_table(float* table, int max_pos, int n_rot, double freq_base) {
    const int half = n_rot / 2;
    for (int p = 0; p < max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const double inv = pow(freq_base, -2.0 * (double) i / (double) n_rot);
            const double a = (double) p * inv;
            table[((size_t) p * half + i) * 2 + 0] = (float) cos(a);
            table[((size_t) p * half + i) * 2 + 1] = (float) sin(a);
        }
}
void or_rope_apply(float* x, int heads, int hd, int n_rot, const float* table, int pos) {
    const int half = n_rot / 2;
    for (int h = 0; h < heads; ++h) {
        float* p = x + (size_t) h * hd;
        for (int i = 0; i < half; ++i) {
            const float c = table[((size_t) pos * half + i) * 2 + 0];
            const float s = table[((size_t) pos * half + i) * 2 + 1];
            const float x0 = p[i], x1 = p[i + half];
            p[i] = x0 * c - x1 * s;
            p[i + half] = x0 * s + x1 * c;
        }
    }
}
/* split_qg_kernel :320-327 — wq emits per head [q (hd) | gate (hd)]. */
void or_split_qg(const float* qg, float* q, float* g, int heads, int hd) {
    for (int h = 0; h < heads; ++h)
        for (int i = 0; i < hd; ++i) {
            q[(size_t) h * hd + i] = qg[(size_t) h * 2 * hd + i];
            g[(size_t) h * hd + i] = qg[(size_t) h * 2 * hd + hd + i];
        }
}
/* store_kv2_kernel :340-345, with an fp16 cache (the flash-decode workload's KV type): cache[pos * n + i]. */
void or_store_kv_f16(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v, int pos, int n) {
    for (int i = 0; i < n; ++i) {
        kcache[(size_t) pos * n + i] = or_f32_to_f16(k[i]);
        vcache[(size_t) pos * n + i] = or_f32_to_f16(v[i]);
    }
}
/* gqa_head_kernel :380-442 with fp16 K/V: per q-head h (kv head h / (n_head/n_kv)): score_t = (xor-tree
 * sum of the lanes' strided partial dots) * scale; softmax with max and sum; o = (sum_t p_t v_t) / sum. */
void or_gqa_decode_f16(const float* q, const uint16_t* kc, const uint16_t* vc, float* o, int n_head, int n_kv,
                       int hd, int n_tok, float scale) {
    float* sc = (float*) malloc(sizeof(float) * (size_t) n_tok);
    for (int h = 0; h < n_head; ++h) {
        const int kv = h / (n_head / n_kv);
        const float* qq = q + (size_t) h * hd;
        float mx = -1e30f;
        for (int t = 0; t < n_tok; ++t) {
            const uint16_t* kk = kc + ((size_t) t * n_kv + kv) * hd;
            float lanes[32];
            for (int l = 0; l < 32; ++l) {
                float dot = 0.0f;
                for (int i = l; i < hd; i += 32) dot = fmaf(qq[i], or_f16_to_f32(kk[i]), dot);
                lanes[l] = dot;
            }
            sc[t] = or_xor_sum32(lanes) * scale;
            mx = fmaxf(mx, sc[t]);
        }
        double sum = 0.0;
        for (int t = 0; t < n_tok; ++t) {
            sc[t] = or_expf(sc[t] - mx);
            sum += sc[t];
        }
        const float inv = (float) (1.0 / sum);
        for (int i = 0; i < hd; ++i) {
            double acc = 0.0;
            for (int t = 0; t < n_tok; ++t) acc += (double) sc[t] * (double) or_f16_to_f32(vc[((size_t) t * n_kv + kv) * hd + i]);
            o[(size_t) h * hd + i] = (float) acc * inv;
        }
    }
    free(sc);
}

/* The same attention step in the summation order of the decode engine's flash-decode kernels, so
 * the engine's outputs can be compared bit for bit (the reference's own order is a HIP block reduction
 * that no other machine reproduces; or_gqa_decode_f16 above restates it in float64, and the tests check
 * that both agree within the fp32 tolerance). Per column c (position pos + c) of proj [c][proj_stride]
 * = [n_head x (q 256 | gate 256) | k n_kv x 256 | v n_kv x 256]:
 *  - per head vector: ss = sum over j = 0..7 (in order) of the 32-lane xor-tree sum of x[32j + l]^2;
 *    inv = 1/sqrt(ss/256 + eps); x = (x * inv) * w; NEOX RoPE over the first n_rot dims (the table's
 *    cos / sin at pos + c); k and v stored as fp16 at pos + c (caches [max_ctx][n_kv][256]);
 *  - chunks of chunk_len tokens; chunk ch covers [ch*len, min(ch*len + len, pos + ncols)), tokens
 *    after pos + c scored -inf; score = xor-tree sum over lanes l of the fma chain over dims 8l..8l+7,
 *    times scale; m = max; e_t = exp(s_t - m); l = xor-tree sum over lanes of each lane's sum of e_t for
 *    t = lane, lane + 32, ...; o = sum over warps w = 0..7 in order of the fma chain over tokens
 *    [32w, 32w + 32) of e_t * v_t;
 *  - combine over the (pos + c)/len + 1 chunks: warp w takes chunks [w n/8, (w+1) n/8), m_w = their max,
 *    fma chains of exp(m_k - m_w) * o_k and * l_k; then over the warps with chunks, in order, fma chains
 *    of exp(m_w - M); o = num / den;
 *  - q8 (may be NULL): the Q8_1 blocks of o * sigmoid(gate) per column. */
static void attn_norm_rope(float* x, const float* w, const float* rope, int n_rot, int p, float eps) {
    float ss = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float sq[32];
        for (int l = 0; l < 32; ++l) sq[l] = x[32 * j + l] * x[32 * j + l];
        const float pj = or_xor_sum32(sq);
        ss = j == 0 ? pj : ss + pj;
    }
    const float inv = 1.0f / sqrtf(ss / 256.0f + eps);
    float r[256];
    for (int d = 0; d < 256; ++d) r[d] = (x[d] * inv) * w[d];
    const int half = n_rot / 2;
    for (int d = 0; d < 256; ++d) {
        if (d < n_rot) {
            const int i = d < half ? d : d - half;
            const float cs = rope[((size_t) p * half + i) * 2 + 0];
            const float sn = rope[((size_t) p * half + i) * 2 + 1];
            const float x0 = r[i], x1 = r[i + half];
            x[d] = d < half ? x0 * cs - x1 * sn : x0 * sn + x1 * cs;
        } else {
            x[d] = r[d];
        }
    }
}
void or_attn_flash_f16(const float* proj, int ncols, int proj_stride, const float* qn, const float* kn,
                       const float* rope, int n_rot, int n_head, int n_kv, uint16_t* kc, uint16_t* vc, int pos,
                       int chunk_len, float eps, float scale, float* o, void* q8) {
    const int HD = 256, G = n_head / n_kv;
    float* qs = (float*) malloc(sizeof(float) * (size_t) ncols * n_head * HD);
    for (int c = 0; c < ncols; ++c) {
        const float* col = proj + (size_t) c * proj_stride;
        for (int h = 0; h < n_head; ++h) {
            float* x = qs + ((size_t) c * n_head + h) * HD;
            memcpy(x, col + (size_t) h * 2 * HD, sizeof(float) * HD);
            attn_norm_rope(x, qn, rope, n_rot, pos + c, eps);
        }
        for (int kv = 0; kv < n_kv; ++kv) {
            float k[256];
            memcpy(k, col + (size_t) n_head * 2 * HD + (size_t) kv * HD, sizeof k);
            attn_norm_rope(k, kn, rope, n_rot, pos + c, eps);
            const float* v = col + (size_t) n_head * 2 * HD + (size_t) n_kv * HD + (size_t) kv * HD;
            for (int d = 0; d < HD; ++d) {
                kc[((size_t) (pos + c) * n_kv + kv) * HD + d] = or_f32_to_f16(k[d]);
                vc[((size_t) (pos + c) * n_kv + kv) * HD + d] = or_f32_to_f16(v[d]);
            }
        }
    }
    const int len = chunk_len, last = pos + ncols;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int c = 0; c < ncols; ++c)
        for (int h = 0; h < n_head; ++h) {
            const int kv = h / G;
            const float* q = qs + ((size_t) c * n_head + h) * HD;
            const int n = (pos + c) / len + 1;
            float* cm = (float*) malloc(sizeof(float) * (size_t) n * (2 + HD));
            float* cl = cm + n;
            float* co = cl + n;
            float sc[256];
            for (int ch = 0; ch < n; ++ch) {
                const int t0 = ch * len;
                const int ntok = (t0 + len < last ? t0 + len : last) - t0;
                float m = -INFINITY;
                for (int t = 0; t < ntok; ++t) {
                    if (t0 + t > pos + c) {
                        sc[t] = -INFINITY;
                        continue;
                    }
                    const uint16_t* kk = kc + ((size_t) (t0 + t) * n_kv + kv) * HD;
                    float lanes[32];
                    for (int l = 0; l < 32; ++l) {
                        float d = 0.0f;
                        for (int i = 0; i < 8; ++i) d = fmaf(q[8 * l + i], or_f16_to_f32(kk[8 * l + i]), d);
                        lanes[l] = d;
                    }
                    sc[t] = or_xor_sum32(lanes) * scale;
                    m = fmaxf(m, sc[t]);
                }
                float lane_l[32];
                for (int l = 0; l < 32; ++l) lane_l[l] = 0.0f;
                for (int t = 0; t < ntok; ++t) {
                    const float e = m == -INFINITY ? 0.0f : or_expf(sc[t] - m);
                    sc[t] = e;
                    lane_l[t & 31] = lane_l[t & 31] + e;
                }
                cm[ch] = m;
                cl[ch] = or_xor_sum32(lane_l);
                for (int d = 0; d < HD; ++d) {
                    float acc = 0.0f;
                    for (int w = 0; w < 8; ++w) {
                        float a = 0.0f;
                        for (int t = 32 * w; t < 32 * w + 32 && t < ntok; ++t) {
                            const float vv = or_f16_to_f32(vc[((size_t) (t0 + t) * n_kv + kv) * HD + d]);
                            a = fmaf(sc[t], vv, a);
                        }
                        acc = w == 0 ? a : acc + a;
                    }
                    co[(size_t) ch * HD + d] = acc;
                }
            }
            float wm[8], wden[8];
            float* wnum = (float*) malloc(sizeof(float) * 8 * HD);
            for (int w = 0; w < 8; ++w) {
                const int k0 = w * n / 8, k1 = (w + 1) * n / 8;
                float mw = -INFINITY;
                for (int k = k0; k < k1; ++k) mw = fmaxf(mw, cm[k]);
                float den = 0.0f;
                for (int d = 0; d < HD; ++d) wnum[w * HD + d] = 0.0f;
                for (int k = k0; k < k1; ++k) {
                    const float wk = or_expf(cm[k] - mw);
                    for (int d = 0; d < HD; ++d) wnum[w * HD + d] = fmaf(wk, co[(size_t) k * HD + d], wnum[w * HD + d]);
                    den = fmaf(wk, cl[k], den);
                }
                wm[w] = k1 > k0 ? mw : -INFINITY;
                wden[w] = den;
            }
            float M = -INFINITY;
            for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w]);
            for (int d = 0; d < HD; ++d) {
                float nu = 0.0f, de = 0.0f;
                for (int w = 0; w < 8; ++w)
                    if (wm[w] != -INFINITY) {
                        const float sw = or_expf(wm[w] - M);
                        nu = fmaf(sw, wnum[w * HD + d], nu);
                        de = fmaf(sw, wden[w], de);
                    }
                o[((size_t) c * n_head + h) * HD + d] = nu / de;
            }
            free(wnum);
            free(cm);
        }
    if (q8)
        for (int c = 0; c < ncols; ++c) {
            const float* col = proj + (size_t) c * proj_stride;
            for (int h = 0; h < n_head; ++h)
                for (int b = 0; b < HD / 32; ++b) {
                    float v[32];
                    for (int l = 0; l < 32; ++l) {
                        const int d = 32 * b + l;
                        v[l] = o[((size_t) c * n_head + h) * HD + d] * or_sigmoidf(col[(size_t) h * 2 * HD + HD + d]);
                    }
                    or_q8_1_block(v, (uint8_t*) q8 + (((size_t) c * n_head + h) * (HD / 32) + b) * 36);
                }
        }
    free(qs);
}

/* Host argmax of forward_token (src/qwythos.cpp:1803-1811): strict greater, lowest index wins ties. */
int or_argmax(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
