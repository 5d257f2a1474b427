// mmvq.cuh — the packed-tile Q6_K / Q8_0 x Q8_1 GEMV for sm_100a, shared by the C-ABI (mmvq.cu) and
// the decode engine (engine.cu), which instantiates its fused prologue / epilogue variants.
//
// Weight layout: rk_pack_weights' tiles of 4 rows x 1024 values (3360 B for Q6_K, 4352 B for Q8_0,
// the GGUF block's codes and scales, rearranged so each lane's 32-value group is one 16-byte and one 8-byte
// vector: q6_decode below gives the layout of the 6-bit codes).
// A "unit" is one row tile over the whole input (n_in/1024 tiles, contiguous in memory). Units are
// split into contiguous ranges per CTA (balanced per SM) and dealt round-robin to the CTA's warps.
// Each warp streams its tiles through a private ring of `stages` shared-memory slots filled by 1-D
// bulk copies (cp.async.bulk, no multicast) that complete on one mbarrier per slot; the warp's lane 0
// is the producer, so a slot is refilled right after the warp has read it, with no cross-warp sync.
// Lane g of a warp handles group g of each tile for the tile's 4 rows: the input column's 32 codes
// and scale stay in registers while 4 rows of weights are decoded against them.
//
// Integer arithmetic (bit-exact with the reference's q6_q8_dot_impl / small_q8_dot,
// src/native_mmvq.cu:642-655, :835-847): for each 16-value sub-block the 6-bit codes (0..63) are
// dotted with the int8 activations by dp4a with the accumulator seeded at -32 * sum(activations),
// which equals sum((code - 32) * x) exactly; times the int8 scale. Per group the two sub-block
// products are added as integers (|sum| < 2^24, so the float conversion is exact) and accumulated
// in fp32 as fma(float(isum), d8 * d, acc) per lane over the k-chunks, then reduced across the warp
// by the xor butterfly. The per-row order does not depend on ncols, so every column of a
// multi-column call is bitwise equal to a single-column call on that column.
//
// Activations, partials and residuals are read with ld.global.cg: the same prologues and epilogues run
// inside the persistent decode kernel, where the producing op ran on other SMs of the same launch.
#pragma once

#include "common.cuh"
#include "xch.cuh"

namespace rk {

constexpr int kMmvqWarps = 8;      // consumer warps per CTA (256 threads)
constexpr int kMmvqMaxStages = 8;  // ring slots per warp (runtime `stages` <= this)
constexpr int kRedCols = 4;        // columns whose RMS partial sums one prologue reduces (red: 8 floats each)
constexpr int kMmvqMaxCols = 4;    // columns per launch (more are split into launches over column chunks)

enum MmvqPro { PRO_Q8 = 0, PRO_RMS = 1 };
// EPI_SWIGLU: y as EPI_STORE for a [up (n_out/2) | gate (n_out/2)] matrix, and for every 32-position block
// whose 16 units (8 up + 8 gate) are done, the last warp to finish one of them writes the Q8_1 block of
// silu(gate) * up (the down GEMV's input; swiglu_quant_kernel, src/qwythos.cpp:676-689).
// EPI_XRES (persistent decode kernel under tensor parallelism): a row-parallel GEMV's partial sums are
// summed over the ranks (peer memory), then as EPI_RES (res != null) or EPI_STORE_P (res == null).
enum MmvqEpi { EPI_STORE = 0, EPI_RES = 1, EPI_ARGMAX = 2, EPI_STORE_P = 3, EPI_SWIGLU = 4, EPI_XRES = 5 };

struct MmvqParams {
    const uint8_t* w;  // packed tiles
    int n_in, n_out;
    int stages;
    int pair;                  // 16-warp launches: warp pairs share units (RK_MMVQ_PAIR=1; set by the launcher)
    int prefetch_before_wait;  // 1: weights are static, stream them before waiting on the upstream grid
    // prologue inputs
    const uint8_t* xq;  // PRO_Q8: Q8_1 blocks, column stride xq_stride bytes (0: rk_q8_1_bytes(n_in, 1))
    int xq_stride;
    const float* xa;    // PRO_RMS: x (column stride n_in)
    const float* xb;    // PRO_RMS: norm weight
    const float* pin;   // PRO_RMS: partials, column stride n_in/4
    float eps;
    // epilogue
    float* y;
    int y_stride;
    const float* res;   // EPI_RES, column stride res_stride
    int res_stride;
    float* pout;        // EPI_RES partials, column stride pout_stride
    int pout_stride;
    unsigned long long* amax;  // EPI_ARGMAX: one packed (value, ~row) slot per column
    int row_off;               // EPI_ARGMAX: global index of row 0 (a vocabulary shard's first row)
    uint8_t* q8out;            // EPI_SWIGLU: Q8_1 of silu(gate) * up, column stride rk_q8_1_bytes(n_out/2, 1)
    unsigned* cnt;             // EPI_SWIGLU: n_out/64 zeroed counters (left zeroed on exit)
    // PRO_RMS write-through (optional): CTA 0 stores the normalized fp32 row (x * w * inv) of every
    // column (stride n_in) and its 4-row sum-of-squares partials (stride n_in/4), the reference's
    // rms_norm_out + row_sum_partials of the final hidden (src/qwythos.cpp:1236-1237).
    float* xn_out;
    float* xn_part;
    const XchDesc* xch;  // EPI_XRES: the ranks' exchange buffers
};

// Smem bytes a launch of `warps` consumer warps needs for the activation staging and the rings.
inline size_t mmvq_smem_bytes(int type, int n_in, int ncols, int stages, int warps = kMmvqWarps) {
    const size_t tile = type == RK_TYPE_Q6_K ? kQ6Tile : kQ80Tile;
    return (size_t) warps * kMmvqMaxStages * 8 + (size_t) ncols * (n_in / 32) * 48 + (size_t) warps * stages * tile;
}

// ---------------------------------------------------------------------------------------------------
// The fixed-order reduction of rms_quant_apply_kernel (src/qwythos.cpp:634-641) over `nslots`
// partials, for a 256-thread block: thread t sums slots t, t+256, ... in order; shfl_down tree in each
// warp; red[0] + ... + red[7] in order. Every thread returns the same value. Uses `red` (8 floats).
// SMEM: the partials are in this block's shared memory (generic loads); else global, read through L2.
// ---------------------------------------------------------------------------------------------------
template <bool SMEM = false>
__device__ __forceinline__ float block256_partials_sum(const float* partials, int nslots, float* red) {
    const int t = threadIdx.x;
    float part = 0.0f;
    for (int p = t; p < nslots; p += 256) part = __fadd_rn(part, SMEM ? partials[p] : __ldcg(partials + p));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_down_sync(0xffffffffu, part, off));
    block_sync256();  // `red` may still be read by a previous call
    if ((t & 31) == 0) red[t >> 5] = part;
    block_sync256();
    float ss = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) ss = __fadd_rn(ss, red[w]);
    return ss;
}
__device__ __forceinline__ float rms_inv(float ss, int cols, float eps) {
    return rk_rsqrtf(__fadd_rn(__fdiv_rn(ss, (float) cols), eps));
}
// The fused-quantize producers (one value per lane), shared with the standalone kernels so a fused
// prologue writes the same bits the standalone kernel writes.
__device__ __forceinline__ float rms_value(float x, float w, float inv) { return __fmul_rn(__fmul_rn(x, w), inv); }
__device__ __forceinline__ float swiglu_value(float up, float g) {
    return __fmul_rn(rk_siluf(g), up);
}
__device__ __forceinline__ float sigmul_value(float o, float g) {
    return __fmul_rn(o, rk_sigmoidf(g));
}

// Staged activation group in shared memory: codes 0..15 in the lo plane, 16..31 in the hi plane
// (16 B per group each), and {d8 (the half-rounded Q8_1 scale), 32*sum(codes 0..15), 32*sum(16..31)}.
struct XStage {
    int4* lo;
    int4* hi;
    float4* meta;
};
__device__ __forceinline__ XStage xstage_col(uint8_t* xsm, int ng, int c) {
    XStage s;
    s.lo = reinterpret_cast<int4*>(xsm + (size_t) c * ng * 48);
    s.hi = s.lo + ng;
    s.meta = reinterpret_cast<float4*>(s.hi + ng);
    return s;
}

// One warp stores the Q8_1 block it just quantized (lane l owns code l) as a staged group.
__device__ __forceinline__ void xstage_put_warp(const XStage& s, int g, int code, uint32_t ds, int lane) {
    int8_t* lo = reinterpret_cast<int8_t*>(s.lo + g);
    int8_t* hi = reinterpret_cast<int8_t*>(s.hi + g);
    if (lane < 16) lo[lane] = (int8_t) code;
    else hi[lane - 16] = (int8_t) code;
    const int s0 = __reduce_add_sync(0xffffffffu, lane < 16 ? code : 0);
    const int s1 = __reduce_add_sync(0xffffffffu, lane < 16 ? 0 : code);
    if (lane == 0) s.meta[g] = make_float4(half_bits_to_float(ds), __int_as_float(32 * s0), __int_as_float(32 * s1), 0.0f);
}

// Build every column's staged activations, with every thread of the block (256 in the per-op kernel,
// 512 in the persistent one); the result does not depend on the block size.
// PRO_Q8: one thread per Q8_1 block (9 ints) -> planes + meta.
// PRO_RMS: the reference's rms_quant_apply (inv from the partials, v = x * w * inv, Q8_1 per 32 values)
// with one thread per 16-value half block: every load is issued before any arithmetic, the two halves of
// a block meet through one shuffle (amax), and each half's codes go to its plane. The codes and scale are
// those of the standalone kernel (same q8_* rules on the same fp32 values). The partial sums are reduced
// as block256_partials_sum does (threads 0..255, then the 8 warp totals in order), every column at once,
// with one block-wide barrier; `red` holds NC * 8 floats.
template <int NC, int PRO>
__device__ __forceinline__ void mmvq_build_x_body(const MmvqParams& p, uint8_t* xsm, float* red) {
    static_assert(PRO != PRO_RMS || NC <= kRedCols, "red holds kRedCols columns of warp totals");
    const int ng = p.n_in >> 5;
    if constexpr (PRO == PRO_Q8) {
        const size_t col_bytes = p.xq_stride > 0 ? (size_t) p.xq_stride : (size_t) ng * 36;
        for (int idx = threadIdx.x; idx < NC * ng; idx += (int) blockDim.x) {
            const int c = idx / ng, g = idx - c * ng;
            const int* blk = reinterpret_cast<const int*>(p.xq + (size_t) c * col_bytes + (size_t) g * 36);
            const uint32_t ds = (uint32_t) __ldcg(blk);
            const int4 a = make_int4(__ldcg(blk + 1), __ldcg(blk + 2), __ldcg(blk + 3), __ldcg(blk + 4));
            const int4 b = make_int4(__ldcg(blk + 5), __ldcg(blk + 6), __ldcg(blk + 7), __ldcg(blk + 8));
            const XStage s = xstage_col(xsm, ng, c);
            s.lo[g] = a;
            s.hi[g] = b;
            const int s0 = __dp4a(a.x, 0x01010101, __dp4a(a.y, 0x01010101, __dp4a(a.z, 0x01010101, __dp4a(a.w, 0x01010101, 0))));
            const int s1 = __dp4a(b.x, 0x01010101, __dp4a(b.y, 0x01010101, __dp4a(b.z, 0x01010101, __dp4a(b.w, 0x01010101, 0))));
            s.meta[g] = make_float4(half_bits_to_float(ds), __int_as_float(32 * s0), __int_as_float(32 * s1), 0.0f);
        }
    } else {
        const int items = NC * ng * 2;  // half blocks; the two halves of a block sit on adjacent lanes
        // The first pass's x / weight loads go out before the partial sums are reduced (they do not
        // depend on them), so the two global round trips overlap.
        float4 xv[4], wv[4];
        auto load = [&](int it) {
            const int c = it / (2 * ng);
            const int rem = it - c * 2 * ng;
            const int i0 = ((rem >> 1) << 5) + ((rem & 1) << 4);
            const float4* xp4 = reinterpret_cast<const float4*>(p.xa + (size_t) c * p.n_in + i0);
            const float4* wp4 = reinterpret_cast<const float4*>(p.xb + i0);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                xv[k] = __ldcg(xp4 + k);
                wv[k] = wp4[k];
            }
        };
        if ((int) threadIdx.x < items) load((int) threadIdx.x);
        if (threadIdx.x < 256) {
            const int t = (int) threadIdx.x, nslots = p.n_in / 4;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float* pc = p.pin + (size_t) c * nslots;
                float part = 0.0f;
                for (int q = t; q < nslots; q += 256) part = __fadd_rn(part, __ldcg(pc + q));
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_down_sync(0xffffffffu, part, off));
                if ((t & 31) == 0) red[c * 8 + (t >> 5)] = part;
            }
        }
        __syncthreads();
        float inv[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            float ss = red[c * 8];
#pragma unroll
            for (int w = 1; w < 8; ++w) ss = __fadd_rn(ss, red[c * 8 + w]);
            inv[c] = rms_inv(ss, p.n_in, p.eps);
        }
        for (int base = 0; base < items; base += (int) blockDim.x) {
            const int it = base + (int) threadIdx.x;
            const bool live = it < items;
            const int c = live ? it / (2 * ng) : 0;
            const int rem = it - c * 2 * ng;
            const int g = rem >> 1, h = rem & 1;
            const int i0 = (g << 5) + (h << 4);
            float v[16];
            if (live) {
                if (base > 0) load(it);
                float invc = inv[0];
#pragma unroll
                for (int cc = 1; cc < NC; ++cc)
                    if (c == cc) invc = inv[cc];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    v[4 * k + 0] = rms_value(xv[k].x, wv[k].x, invc);
                    v[4 * k + 1] = rms_value(xv[k].y, wv[k].y, invc);
                    v[4 * k + 2] = rms_value(xv[k].z, wv[k].z, invc);
                    v[4 * k + 3] = rms_value(xv[k].w, wv[k].w, invc);
                }
            } else {
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = 0.0f;
            }
            float amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(v[k]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            const float d = q8_finite_d(__fdiv_rn(amax, 127.0f));
            int packed[4] = {0, 0, 0, 0};
            int csum = 0;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int q = q8_quant(v[k], d, amax);
                csum += q;
                packed[k >> 2] |= (q & 0xff) << (8 * (k & 3));
            }
            const int other = __shfl_xor_sync(0xffffffffu, csum, 1);
            if (live) {
                const XStage s = xstage_col(xsm, ng, c);
                (h ? s.hi : s.lo)[g] = make_int4(packed[0], packed[1], packed[2], packed[3]);
                if (h == 0)
                    s.meta[g] = make_float4(__half2float(__float2half_rn(d)), __int_as_float(32 * csum),
                                            __int_as_float(32 * other), 0.0f);
            }
            // PRO_RMS write-through of the normalized row and its partials (CTA 0 only)
            if (p.xn_out != nullptr && blockIdx.x == 0 && live) {
                float* xo = p.xn_out + (size_t) c * p.n_in + i0;
#pragma unroll
                for (int k = 0; k < 16; ++k) xo[k] = v[k];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float part = __fmul_rn(v[4 * k], v[4 * k]);
                    part = __fmaf_rn(v[4 * k + 1], v[4 * k + 1], part);
                    part = __fmaf_rn(v[4 * k + 2], v[4 * k + 2], part);
                    part = __fmaf_rn(v[4 * k + 3], v[4 * k + 3], part);
                    p.xn_part[(size_t) c * (p.n_in / 4) + (i0 >> 2) + k] = part;
                }
            }
        }
    }
}
// The same as a call (the persistent kernel, whose op bodies stay out of line). mmvq_packed_kernel inlines
// the body: a call that takes the kernel's parameter block by reference makes every thread copy the block
// (184 bytes) to its stack at entry.
template <int NC, int PRO>
__device__ __noinline__ void mmvq_build_x(const MmvqParams& p, uint8_t* xsm, float* red) {
    mmvq_build_x_body<NC, PRO>(p, xsm, red);
}

// The 6-bit codes of one row of a group as eight ints (byte b of int T = code of value 4T + b), from the
// packed A (16 B: byte 4T + b holds the code of value 4T + b in its low 6 bits and the top 2 bits of
// value 16 + 4T + b above them) and B (8 B: byte 4u + b holds the low nibbles of values 16 + 8u + b and
// 20 + 8u + b). The first four ints are one mask each; the last four take a nibble plane and the top bits
// of an A word.
__device__ __forceinline__ void q6_decode(const uint4 a, const uint2 b, int v[8]) {
    v[0] = (int) (a.x & 0x3f3f3f3fu);
    v[1] = (int) (a.y & 0x3f3f3f3fu);
    v[2] = (int) (a.z & 0x3f3f3f3fu);
    v[3] = (int) (a.w & 0x3f3f3f3fu);
    v[4] = (int) ((b.x & 0x0f0f0f0fu) | ((a.x >> 2) & 0x30303030u));
    v[5] = (int) (((b.x >> 4) & 0x0f0f0f0fu) | ((a.y >> 2) & 0x30303030u));
    v[6] = (int) ((b.y & 0x0f0f0f0fu) | ((a.z >> 2) & 0x30303030u));
    v[7] = (int) (((b.y >> 4) & 0x0f0f0f0fu) | ((a.w >> 2) & 0x30303030u));
}
// sum over each 16-value sub-block of (code - 32) * x, exactly.
__device__ __forceinline__ void q6_subsums(const int v[8], const int4 xa, const int4 xb, int b0, int b1, int& s0,
                                           int& s1) {
    s0 = __dp4a(v[0], xa.x, -b0);
    s0 = __dp4a(v[1], xa.y, s0);
    s0 = __dp4a(v[2], xa.z, s0);
    s0 = __dp4a(v[3], xa.w, s0);
    s1 = __dp4a(v[4], xb.x, -b1);
    s1 = __dp4a(v[5], xb.y, s1);
    s1 = __dp4a(v[6], xb.z, s1);
    s1 = __dp4a(v[7], xb.w, s1);
}
__device__ __forceinline__ int sext8(uint32_t w, int byte) { return ((int) (w << (24 - 8 * byte))) >> 24; }

// One Q6_K tile (4 rows x this lane's group) against NC staged columns.
template <int NC>
__device__ __forceinline__ void q6_tile(const uint8_t* t, int lane, const int4 (&xa)[NC], const int4 (&xb)[NC],
                                        const float4 (&xm)[NC], float (&acc)[NC][4]) {
    const uint2 scw = *reinterpret_cast<const uint2*>(t + 3072 + lane * 8);
    const uint2 dw = *reinterpret_cast<const uint2*>(t + 3328 + (lane >> 3) * 8);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint4 ql = *reinterpret_cast<const uint4*>(t + (r * 32 + lane) * 16);
        const uint2 qh = *reinterpret_cast<const uint2*>(t + 2048 + (r * 32 + lane) * 8);
        int v[8];
        q6_decode(ql, qh, v);
        const uint32_t sw = r < 2 ? scw.x : scw.y;
        const int sc0 = sext8(sw, 2 * (r & 1)), sc1 = sext8(sw, 2 * (r & 1) + 1);
        const float dr = half_bits_to_float((r < 2 ? dw.x : dw.y) >> (16 * (r & 1)));
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            int s0, s1;
            q6_subsums(v, xa[c], xb[c], __float_as_int(xm[c].y), __float_as_int(xm[c].z), s0, s1);
            const int isum = s0 * sc0 + s1 * sc1;
            acc[c][r] = __fmaf_rn((float) isum, __fmul_rn(xm[c].x, dr), acc[c][r]);
        }
    }
}

// One Q8_0 tile.
template <int NC>
__device__ __forceinline__ void q80_tile(const uint8_t* t, int lane, const int4 (&xa)[NC], const int4 (&xb)[NC],
                                         const float4 (&xm)[NC], float (&acc)[NC][4]) {
    const uint2 dw = *reinterpret_cast<const uint2*>(t + 4096 + lane * 8);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int4 w0 = *reinterpret_cast<const int4*>(t + ((r * 2 + 0) * 32 + lane) * 16);
        const int4 w1 = *reinterpret_cast<const int4*>(t + ((r * 2 + 1) * 32 + lane) * 16);
        const float dr = half_bits_to_float((r < 2 ? dw.x : dw.y) >> (16 * (r & 1)));
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            int s = __dp4a(w0.x, xa[c].x, 0);
            s = __dp4a(w0.y, xa[c].y, s);
            s = __dp4a(w0.z, xa[c].z, s);
            s = __dp4a(w0.w, xa[c].w, s);
            s = __dp4a(w1.x, xb[c].x, s);
            s = __dp4a(w1.y, xb[c].y, s);
            s = __dp4a(w1.z, xb[c].z, s);
            s = __dp4a(w1.w, xb[c].w, s);
            acc[c][r] = __fmaf_rn((float) s, __fmul_rn(xm[c].x, dr), acc[c][r]);
        }
    }
}

// Monotonic key for the fused argmax: larger value -> larger key; among equal values the lower row wins.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    uint32_t b = __float_as_uint(v);
    b ^= (b >> 31) ? 0xffffffffu : 0x80000000u;
    return ((unsigned long long) b << 32) | (unsigned long long) (0xffffffffu - (uint32_t) row);
}
__host__ __device__ __forceinline__ int argmax_key_row(unsigned long long k) { return (int) (0xffffffffu - (uint32_t) (k & 0xffffffffu)); }

// The epilogue's warp reduction of a unit's 4 * NC row sums as a reduce-scatter: at xor offsets 16, 8, ...
// each lane keeps half of its values and adds the partner's copy of that half, until one value is left
// (then plain butterfly steps). Every step adds the same two partial sums that warp_sum adds for that
// value (fp32 addition is commutative), so the result is bitwise warp_sum's, with 4 * NC - 1 + (5 -
// log2(4 * NC)) shuffles instead of 20 * NC. Lane l ends with the sum of value j = c * 4 + r =
// l >> kRsShift<NC>; 3 columns are reduced as 4 (the fourth column's values are zeros, never stored).
template <int NC>
constexpr int kRsShift = NC == 1 ? 3 : NC == 2 ? 2 : 1;
template <int NC>
__device__ __forceinline__ float warp_sum_scatter(const float (&acc)[NC][4], int lane) {
    static_assert(NC >= 1 && NC <= 4, "up to 4 columns");
    constexpr int M = NC == 3 ? 16 : 4 * NC;
    float v[M];
#pragma unroll
    for (int j = 0; j < M; ++j) v[j] = j < 4 * NC ? acc[j >> 2][j & 3] : 0.0f;
    warp_reduce_scatter<M>(v, lane);
    return v[0];
}

// best[c] (EPI_ARGMAX): the warp's running packed (value, ~row) maximum of column c, held by the lanes
// whose reduced value is one of column c's rows; lane (4 * c) << kRsShift<NC> issues one atomicMax per
// column after the warp's last unit (mmvq_argmax_flush; the reference's atomicMax on (monotonic bits,
// n-1-idx), src/qwythos.cpp:70-84, with the lowest-index tie rule). resv (EPI_RES): lane c < NC holds the
// residual rows of column c for this unit, loaded by mmvq_res_prefetch when the unit started.
template <int NC, int EPI>
__device__ __forceinline__ void mmvq_epilogue(const MmvqParams& p, int unit, int lane, const float (&acc)[NC][4],
                                              unsigned long long (&best)[NC], const float (&resv)[4]) {
    constexpr int SH = kRsShift<NC>;
    const float out = warp_sum_scatter<NC>(acc, lane);
    const int j = lane >> SH;  // this lane's value: column j >> 2, row j & 3 of the unit
    const int row0 = unit * 4;
    if constexpr (EPI == EPI_STORE || EPI == EPI_ARGMAX || EPI == EPI_SWIGLU) {
        if (p.y != nullptr && (lane & ((1 << SH) - 1)) == 0 && (j >> 2) < NC)
            p.y[(size_t) (j >> 2) * p.y_stride + row0 + (j & 3)] = out;
        if constexpr (EPI == EPI_ARGMAX) {
            unsigned long long k = out == out ? argmax_key(out, p.row_off + row0 + (j & 3)) : 0ull;  // NaN never wins
            unsigned long long o = __shfl_xor_sync(0xffffffffu, k, 1 << SH);
            k = o > k ? o : k;
            o = __shfl_xor_sync(0xffffffffu, k, 2 << SH);
            k = o > k ? o : k;
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if ((j >> 2) == c && k > best[c]) best[c] = k;
        }
    } else {  // EPI_RES (y = acc + res) / EPI_STORE_P (y = acc), both with the 4-row partials
        const int cl = lane < NC ? lane : NC - 1;
        float rv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) rv[r] = __shfl_sync(0xffffffffu, out, (cl * 4 + r) << SH);
        if (lane < NC) {
            float* y = p.y + (size_t) lane * p.y_stride + row0;
            float part = 0.0f;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float v = EPI == EPI_RES ? __fadd_rn(rv[r], resv[r]) : rv[r];
                y[r] = v;
                part = __fmaf_rn(v, v, part);
            }
            p.pout[(size_t) lane * p.pout_stride + unit] = part;
        }
    }
}
template <int NC>
__device__ __forceinline__ void mmvq_argmax_flush(const MmvqParams& p, int lane, const unsigned long long (&best)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; ++c)
        if (lane == ((4 * c) << kRsShift<NC>) && best[c] != 0ull) atomicMax(p.amax + c, best[c]);
}

// EPI_RES: the residual rows of a unit, issued when the unit starts so the load overlaps its tiles.
template <int NC, int EPI>
__device__ __forceinline__ void mmvq_res_prefetch(const MmvqParams& p, int unit, int lane, float (&resv)[4]) {
    if constexpr (EPI == EPI_RES) {
        if (lane < NC) {
            const float* r = p.res + (size_t) lane * p.res_stride + (size_t) unit * 4;
#pragma unroll
            for (int k = 0; k < 4; ++k) resv[k] = __ldcg(r + k);
        }
    }
}

// EPI_XRES (tensor parallelism, both executors): a unit's 4 x NC row sums of this rank's share of the input
// (the xor butterfly per value) go as epoch-tagged words (xch.cuh) into this rank's source slot of every
// rank's partial buffer; `yoff` (xres_offset) selects the slot and the epoch's parity half.
__device__ __forceinline__ size_t xres_offset(const XchDesc* x, unsigned long long ep) {
    return (((size_t) (ep & 1ull) * kMaxRanks + x->rank) * 2) * x->rows;
}
template <int NC>
__device__ __forceinline__ void xres_push(const XchDesc* x, size_t yoff, unsigned long long ep, int unit, int lane,
                                          float (&acc)[NC][4]) {
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[c][r] = warp_sum(acc[c][r]);
    float out = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (lane == c * 4 + r) out = acc[c][r];
    if (lane < NC * 4) {
        const size_t o = yoff + (size_t) (lane >> 2) * x->rows + (size_t) unit * 4 + (lane & 3);
        const unsigned long long w = xch_word(ep, out);
        for (int q = 0; q < x->n; ++q) st_volatile_u64(x->buf[q] + o, w);
    }
}
// After a CTA's units: for each of the CTA's rows [4 ubeg, 4 uend) and columns, wait for every rank's word
// of this exchange and sum them in rank order (every rank gets the same bits), add the residual and write y
// and the 4-row partials as EPI_RES does (EPI_STORE_P without a residual). Returns false (this thread) when
// a wait gave up; a rank whose warp failed before pushing leaves its peers' waits to give up too.
template <int NC>
__device__ __forceinline__ bool xres_finish(const MmvqParams& p, int ubeg, int uend, unsigned long long ep,
                                            PSync* sync) {
    const XchDesc* x = p.xch;
    const int n = x->n;
    const unsigned long long* mine = x->buf[x->rank] + (size_t) (ep & 1ull) * kMaxRanks * 2 * x->rows;
    const size_t src_stride = (size_t) 2 * x->rows;
    bool ok = true;
    for (int idx = (int) threadIdx.x; idx < (uend - ubeg) * NC && ok; idx += (int) blockDim.x) {
        const int u = ubeg + idx / NC, c = idx % NC;
        float part = 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const size_t off = (size_t) c * x->rows + (size_t) u * 4 + r;
            float v = 0.0f;
            for (int q = 0; q < n && ok; ++q) {
                float pq = 0.0f;
                ok = xch_poll(mine + q * src_stride + off, ep, x, sync, pq);
                v = q == 0 ? pq : __fadd_rn(v, pq);
            }
            if (p.res != nullptr) v = __fadd_rn(v, __ldcg(p.res + (size_t) c * p.res_stride + (size_t) u * 4 + r));
            p.y[(size_t) c * p.y_stride + (size_t) u * 4 + r] = v;
            part = __fmaf_rn(v, v, part);
        }
        p.pout[(size_t) c * p.pout_stride + u] = part;
    }
    return ok;
}

// EPI_SWIGLU, after a warp's units [first, end) (stride `stride`) are written: one fence, then one arrival
// per unit (issued by different lanes at once); for every 32-position block whose 16 units (8 up + 8 gate)
// are done, the warp whose arrival completed it writes the Q8_1 block of silu(gate) * up (the down GEMV's
// input; swiglu_quant_kernel, src/qwythos.cpp:676-689) and re-zeroes the counter.
template <int NC>
__device__ __forceinline__ void mmvq_swiglu_finish(const MmvqParams& p, int first, int stride, int end, int lane) {
    if (first >= end) return;
    __threadfence();
    __syncwarp();
    const int half = p.n_out >> 1;
    for (int base = first; base < end; base += 32 * stride) {
        const int u = base + lane * stride;
        int grp = 0;
        bool last = false;
        if (u < end) {
            grp = (u < (half >> 2) ? u : u - (half >> 2)) >> 3;
            last = atomicAdd(p.cnt + grp, 1u) == 15u;
        }
        unsigned m = __ballot_sync(0xffffffffu, last);
        if (m) __threadfence();
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const int g = __shfl_sync(0xffffffffu, grp, src);
            const int i = (g << 5) + lane;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float up = __ldcg(p.y + (size_t) c * p.y_stride + i);
                const float gt = __ldcg(p.y + (size_t) c * p.y_stride + half + i);
                q8_1_warp_store(swiglu_value(up, gt), p.q8out + ((size_t) c * (half >> 5) + g) * 36, lane);
            }
            if (lane == 0) p.cnt[g] = 0u;
        }
    }
}

// The per-lane fp32 chain of a row runs over each half of an even chunk count separately (kc < KC/2 and
// kc >= KC/2), and the halves are added lo + hi: two warps can then take the halves of a unit. mmvq_split
// is the first chunk of the second half (KC when there is one chain).
__host__ __device__ __forceinline__ int mmvq_split(int KC) { return KC >= 2 && (KC & 1) == 0 ? KC >> 1 : KC; }
template <int NC>
__device__ __forceinline__ void mmvq_stash_half(float (&acc)[NC][4], float (&lo)[NC][4]) {
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            lo[c][r] = acc[c][r];
            acc[c][r] = 0.0f;
        }
}
template <int NC>
__device__ __forceinline__ void mmvq_join_halves(float (&acc)[NC][4], const float (&lo)[NC][4]) {
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[c][r] = __fadd_rn(lo[c][r], acc[c][r]);
}
// Bounded spin on a shared-memory word written by another warp of the block (warp pairs below).
__device__ __forceinline__ bool smem_wait_at_least(const volatile int* w, int v) {
    for (uint32_t it = 0; it < (1u << 24); ++it) {
        if (*w >= v) return true;
        if (it >= 64u) __nanosleep(32);
    }
    atomicOr(&g_rk_status, kStatusWaitTimeout);
    return false;
}
// Bytes of the warp-pair exchange slots of a 16-warp launch (two slots per pair of warps, NC x 4 floats per lane).
__host__ __device__ __forceinline__ size_t mmvq_pair_bytes(int ncols, int warps) { return warps == 16 ? (size_t) 8 * 2 * ncols * 4 * 32 * 4 : 0; }

template <int TYPE, int NC, int PRO, int EPI, int W = kMmvqWarps>
__global__ void __launch_bounds__(W * 32, 16 / W) mmvq_packed_kernel(const MmvqParams p) {
    constexpr int TILE = TYPE == RK_TYPE_Q6_K ? kQ6Tile : kQ80Tile;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[kRedCols * 8];
    __shared__ int pair_flag[8][2], pair_ack[8][2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KC = p.n_in >> 10;
    const int ng = p.n_in >> 5;
    const int stages = p.stages;
    const int split = mmvq_split(KC);
    // Warp pairs (16 warps, an even chunk count, p.pair set by the launcher): warps 2m and 2m + 1 take the
    // two halves of the same units, so a unit's tiles are consumed by two warps at once; the odd warp hands
    // its half's chains to the even one through a shared-memory slot, and the even warp adds them (lo + hi)
    // and runs the epilogue. Measured on the decode (same box, alternating): pairs in every 2-column launch
    // 3-4 % slower than 16 unpaired warps (the slots cost ring depth and the handoff waits); pairs where they
    // shorten the busiest warp's tile chain (mmvq_launch_w) 4.4 % faster with exact MTP.
    const bool paired = W == 16 && split < KC && p.pair != 0;
    const int PW = paired ? W / 2 : W;           // units in flight per CTA
    const int ul = paired ? warp >> 1 : warp;    // this warp's unit lane
    const int half = paired ? warp & 1 : 0;      // which half of each unit this warp consumes
    const int KT = paired ? split : KC;          // tiles per unit for this warp
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kMmvqMaxStages;
    float* pslots = reinterpret_cast<float*>(smem + W * kMmvqMaxStages * 8);
    uint8_t* xsm = smem + W * kMmvqMaxStages * 8 + (p.pair ? mmvq_pair_bytes(NC, W) : 0);
    uint8_t* ring = xsm + (size_t) NC * ng * 48 + (size_t) warp * stages * TILE;

    const int units = p.n_out >> 2;
    const int ubeg = (int) (((long long) blockIdx.x * units) / gridDim.x);
    const int uend = (int) (((long long) (blockIdx.x + 1) * units) / gridDim.x);
    const int my_units = (uend - ubeg > ul) ? (uend - ubeg - ul + PW - 1) / PW : 0;
    const int ntiles = my_units * KT;

    if (lane == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(smem_u32(bars + s), 1);
        fence_mbar_init();
    }
    if (threadIdx.x < 16) {
        pair_flag[threadIdx.x >> 1][threadIdx.x & 1] = 0;
        pair_ack[threadIdx.x >> 1][threadIdx.x & 1] = 0;
    }
    __syncwarp();
    const uint64_t pol = policy_evict_first();
    // Producer cursor (lane 0): the next tile to fetch walks this warp's tiles in order (a unit's tiles are
    // contiguous: KT of them from this warp's half; the next unit is PW units further), and tile i + stages
    // goes into the slot tile i just left, so the refill needs no division.
    const uint8_t* nsrc = p.w + ((size_t) (ubeg + ul) * KC + (size_t) half * KT) * TILE;
    int nkc = 0;
    const size_t unit_skip = (size_t) (PW * KC - KT) * TILE;
    auto issue = [&](int slot) {
        mbar_arrive_expect_tx(smem_u32(bars + slot), TILE);
        bulk_g2s(smem_u32(ring + (size_t) slot * TILE), nsrc, TILE, smem_u32(bars + slot), pol);
        nsrc += TILE;
        if (++nkc == KT) {
            nkc = 0;
            nsrc += unit_skip;
        }
    };
    const int npre = ntiles < stages ? ntiles : stages;
    if (p.prefetch_before_wait && lane == 0)
        for (int i = 0; i < npre; ++i) issue(i);
    pdl_wait();
    if (!p.prefetch_before_wait && lane == 0)
        for (int i = 0; i < npre; ++i) issue(i);
    // EPI_XRES (the graph executor under tensor parallelism): this CTA's exchange epoch, from the counter
    // of its flag slot (the previous exchange on this slot was written back by a launch now complete)
    __shared__ unsigned long long xep_sh;
    if constexpr (EPI == EPI_XRES)
        if (threadIdx.x == 0) xep_sh = xch_epoch_next(p.xch, (int) blockIdx.x);

    mmvq_build_x_body<NC, PRO>(p, xsm, red);
    __syncthreads();
    unsigned long long xep = 0ull;
    size_t yoff = 0;
    if constexpr (EPI == EPI_XRES) {
        xep = xep_sh;
        yoff = xres_offset(p.xch, xep);
    }
    bool ok = true;

    float acc[NC][4], lo[NC][4];
    unsigned long long best[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        best[c] = 0ull;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            acc[c][r] = 0.0f;
            lo[c][r] = 0.0f;
        }
    }

    int s = 0, kc = 0, unit = ubeg + ul, seq = 0;
    uint32_t parity = 0;
    float resv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (ntiles > 0 && half == 0) mmvq_res_prefetch<NC, EPI>(p, unit, lane, resv);
    const int kbase = half * KT;  // this warp's first chunk of a unit
    for (int i = 0; i < ntiles; ++i) {
        const bool landed = mbar_wait_bounded(smem_u32(bars + s), parity);
        if (!__all_sync(0xffffffffu, landed)) {
            ok = false;
            break;
        }
        if (!paired && kc == split) mmvq_stash_half<NC>(acc, lo);
        const uint8_t* t = ring + (size_t) s * TILE;
        int4 xa[NC], xb[NC];
        float4 xm[NC];
        const int g = ((kbase + kc) << 5) + lane;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const XStage xs = xstage_col(xsm, ng, c);
            xa[c] = xs.lo[g];
            xb[c] = xs.hi[g];
            xm[c] = xs.meta[g];
        }
        if constexpr (TYPE == RK_TYPE_Q6_K) q6_tile<NC>(t, lane, xa, xb, xm, acc);
        else q80_tile<NC>(t, lane, xa, xb, xm, acc);
        __syncwarp();
        if (lane == 0 && i + stages < ntiles) {
            fence_proxy_async_smem();
            issue(s);
        }
        if (++s == stages) {
            s = 0;
            parity ^= 1u;
        }
        if (++kc == KT) {
            if (!paired) {
                if (split < KC) mmvq_join_halves<NC>(acc, lo);
                if constexpr (EPI == EPI_XRES) xres_push<NC>(p.xch, yoff, xep, unit, lane, acc);
                else mmvq_epilogue<NC, EPI>(p, unit, lane, acc, best, resv);
            } else {
                float* slot = pslots + ((size_t) (ul * 2 + (seq & 1)) * NC * 4) * 32;
                if (half == 1) {  // hand the hi half over: slot free once the even warp took seq - 2
                    if (seq >= 2) smem_wait_at_least(&pair_ack[ul][seq & 1], seq - 1);
#pragma unroll
                    for (int c = 0; c < NC; ++c)
#pragma unroll
                        for (int r = 0; r < 4; ++r) slot[(c * 4 + r) * 32 + lane] = acc[c][r];
                    __syncwarp();
                    __threadfence_block();
                    if (lane == 0) *reinterpret_cast<volatile int*>(&pair_flag[ul][seq & 1]) = seq + 1;
                } else {
                    smem_wait_at_least(&pair_flag[ul][seq & 1], seq + 1);
                    __threadfence_block();
#pragma unroll
                    for (int c = 0; c < NC; ++c)
#pragma unroll
                        for (int r = 0; r < 4; ++r) acc[c][r] = __fadd_rn(acc[c][r], slot[(c * 4 + r) * 32 + lane]);
                    __syncwarp();
                    __threadfence_block();  // the slot is read before the odd warp may refill it
                    if (lane == 0) *reinterpret_cast<volatile int*>(&pair_ack[ul][seq & 1]) = seq + 1;
                    if constexpr (EPI == EPI_XRES) xres_push<NC>(p.xch, yoff, xep, unit, lane, acc);
                    else mmvq_epilogue<NC, EPI>(p, unit, lane, acc, best, resv);
                }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[c][r] = 0.0f;
            kc = 0;
            ++seq;
            unit += PW;
            if (unit < uend && half == 0) mmvq_res_prefetch<NC, EPI>(p, unit, lane, resv);
        }
    }
    // The next launch may start only now: its CTAs would otherwise queue their own bulk copies (and the
    // launches after it theirs) ahead of this launch's last refills, which gate the whole step (measured:
    // 1 % per token; with rings sized so two launches' CTAs share an SM and the next launch triggered once
    // every warp has issued its last copy, the decode step ran 20-25 % slower).
    pdl_trigger();
    if (half == 0) {
        if constexpr (EPI == EPI_SWIGLU) mmvq_swiglu_finish<NC>(p, ubeg + ul, PW, unit, lane);
        if constexpr (EPI == EPI_ARGMAX) mmvq_argmax_flush<NC>(p, lane, best);
    }
    if constexpr (EPI == EPI_XRES) {
        PSync* sync = p.xch->sync;
        if (!ok || !xres_finish<NC>(p, ubeg, uend, xep, sync))
            atomicExch(&sync->abort, 1u);  // for the host, and so that later waits of this rank end at once
        if (threadIdx.x == 0) xch_epoch_done(p.xch, (int) blockIdx.x, xep);
    }
}

// Host-side launcher for one instantiation: sets the smem attribute once, picks the stage count that
// keeps two CTAs per SM where possible, grid = one CTA per SM (capped by the unit count).
// Tuning knobs read once from the environment (like the reference's QWYTHOS_Q6ROWS sweep knob,
// src/native_mmvq.cu:3648-3651): RK_MMVQ_STAGES forces the ring depth, RK_MMVQ_CTAS the CTAs per SM.
int mmvq_env_stages();
int mmvq_env_ctas();
int mmvq_env_warps();
int mmvq_env_pair();  // RK_MMVQ_PAIR > 0: warp pairs in 16-warp launches

template <int TYPE, int NC, int PRO, int EPI, int W>
cudaError_t mmvq_launch_w(MmvqParams p, cudaStream_t s, bool pdl) {
    static int configured_smem = -1;
    static int max_optin = 0;
    if (max_optin == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (max_optin <= 0) max_optin = 227 * 1024;
    }
    const size_t tile = TYPE == RK_TYPE_Q6_K ? kQ6Tile : kQ80Tile;
    int ctas = 1;
    if (mmvq_env_ctas() > 0 && EPI != EPI_XRES) ctas = mmvq_env_ctas();  // an exchange CTA owns a flag slot per SM
    const int units = p.n_out / 4;
    int grid = num_sms() * ctas;
    if (grid > units) grid = units;
    // Warp pairs (16 warps, an even chunk count): the two halves of each unit's chunks go to two warps. By
    // default where that shortens the busiest warp's tile chain by a quarter or more: a CTA's u units give
    // it ceil(u / 16) whole units unpaired and ceil(u / 8) half units paired (the residual GEMVs, 7 units per
    // CTA: 4 tiles -> 2; in_proj, 21: 8 -> 6; not up||gate, 42: 12 -> 12, nor the lm_head). Measured with
    // exact MTP (same box): residual GEMVs paired +2.0 %, in_proj and qkv too +2.4 % more, up||gate too
    // -5 %. RK_MMVQ_PAIR=1 pairs every 16-warp launch, -1 none.
    const int per_cta = (units + grid - 1) / grid;
    const bool can_pair = W == 16 && mmvq_split(p.n_in >> 10) < (p.n_in >> 10);
    const bool shorter = 2 * ((per_cta + W / 2 - 1) / (W / 2)) <= 3 * ((per_cta + W - 1) / W);
    p.pair = can_pair && (mmvq_env_pair() > 0 || (mmvq_env_pair() == 0 && shorter)) ? 1 : 0;
    const size_t fixed = mmvq_smem_bytes(TYPE, p.n_in, NC, 0, W) + (p.pair ? mmvq_pair_bytes(NC, W) : 0);
    // One CTA per SM (8 warps) with a ring of up to 5 slots: measured best on B200 for config 1 (12288 x
    // 4096, 2 columns: 2.8 vs 2.4-2.6 TB/s) and for a decode step of one GEMV launch per op (2.45 vs
    // 2.59 ms). Two 3-slot CTAs per SM leave the busiest warp 8 tiles where the average is 5 (units are
    // dealt to warps whole), with 16 warps sharing the SM's issue slots, and let the next op's CTAs become
    // resident and start their weight prefetch while this one still runs.
    int stages = (int) (((long long) max_optin - 2048 - (long long) fixed) / (long long) (W * tile));
    if (stages > 5) stages = 5;
    if (mmvq_env_stages() > 0) stages = mmvq_env_stages();
    if (stages < 2 || stages > kMmvqMaxStages) return cudaErrorInvalidValue;
    p.stages = stages;
    const size_t smem = mmvq_smem_bytes(TYPE, p.n_in, NC, stages, W) + (p.pair ? mmvq_pair_bytes(NC, W) : 0);
    if ((int) smem > configured_smem) {
        cudaError_t e = cudaFuncSetAttribute(mmvq_packed_kernel<TYPE, NC, PRO, EPI, W>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return e;
        configured_smem = (int) smem;
    }
    return launch_pdl(mmvq_packed_kernel<TYPE, NC, PRO, EPI, W>, dim3(grid), dim3(W * 32), smem, s, pdl, p);
}
// warps: consumer warps per CTA, 8 (256 threads, 5-slot rings) or 16 (512 threads, 3-4 slots).
// Measured on B200 (same box, alternating): the decode engine's 2-column GEMVs (the MTP verify and draft)
// run 9 % faster with 16 warps (the integer chains of two columns per tile leave 2 warps per scheduler
// idle on dependencies; the MTP decode +5.4 %), single-column ones 6 % slower unpaired (the no-MTP decode
// -5 %; the single-column residual GEMVs gain with 16 paired warps), and a lone repeated 41 MB GEMV 10 %
// slower. RK_MMVQ_WARPS=8|16 overrides.
template <int TYPE, int NC, int PRO, int EPI>
cudaError_t mmvq_launch(MmvqParams p, cudaStream_t s, bool pdl, int warps = kMmvqWarps) {
    if (mmvq_env_warps() == 8 || mmvq_env_warps() == 16) warps = mmvq_env_warps();
    if (warps == 16) return mmvq_launch_w<TYPE, NC, PRO, EPI, 16>(p, s, pdl);
    return mmvq_launch_w<TYPE, NC, PRO, EPI, kMmvqWarps>(p, s, pdl);
}

}  // namespace rk
