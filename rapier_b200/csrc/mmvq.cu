// mmvq.cu — C-ABI for the quantized GEMVs: Q8_1 quantizer, GGUF-layout (drop-in) GEMV, packed-tile
// GEMV (the fast path, mmvq.cuh), the load-time repack, and the integer-sum parity probe.
#include "mmvq.cuh"

namespace rk {
namespace {

constexpr int kMaxNcols = 16;  // the reference's MAX_NCOLS (src/native_mmvq.cu:2316)

// ---------------------------------------------------------------------------------------------------
// Q8_1 quantizer (native_quantize_q8_1_kernel, src/native_mmvq.cu:158-173): one warp per 32-value block.
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quantize_q8_1_kernel(const float* __restrict__ x, uint8_t* __restrict__ y,
                                                            int n_blocks) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= n_blocks) return;  // whole warps only
    const int lane = threadIdx.x & 31;
    q8_1_warp_store(x[(size_t) b * 32 + lane], y + (size_t) b * 36, lane);
}

// ---------------------------------------------------------------------------------------------------
// GGUF-layout GEMV (compat path for rk_mmvq / rk_mmvq_res on unrepacked rows). One warp per row; the
// lanes follow the reference's per-lane mapping (lane iqs of each super-block for Q6_K, q6_q8_dot at
// src/native_mmvq.cu:733-748; two ints of one block per lane for Q8_0, :835-847), with the integer
// sums computed the same way as the packed kernel's (codes dotted unsigned, -32*sum seeded).
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ int ld_b2(const uint8_t* p) {  // two little-endian u16 (2-byte aligned rows)
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
    return (int) ((uint32_t) q[0] | ((uint32_t) q[1] << 16));
}

__host__ __device__ constexpr size_t raw_row_bytes(int type, int n_in) {
    return type == RK_TYPE_Q6_K   ? (size_t) (n_in / 256) * 210
           : type == RK_TYPE_Q5_K ? (size_t) (n_in / 256) * 176
           : type == RK_TYPE_Q4_K ? (size_t) (n_in / 256) * 144
                                  : (size_t) (n_in / 32) * 34;
}

// Q5_K / Q4_K sub-block j's 6-bit (scale, min): ggml's get_scale_min_k4 over the block's 12 scale bytes.
__device__ __forceinline__ void kq_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Thread iqs (even) of a Q5_K / Q4_K block against one Q8_1 column (vec_dot_q5_K_q8_1 / _q4_K_q8_1 as
// src/native_mmvq.cu:191-252 and :543-595 pin them): sub-blocks bq8 and bq8 + 1, 8 values of each. ip
// (optional) receives dot1 * scale and dot2 * min per sub-block; returns d * sumf_d - dmin * sumf_m.
template <int TYPE>
__device__ __forceinline__ float kq_q8_dot(const uint8_t* blk, const uint8_t* x, int iqs, int* ip) {
    constexpr int QS = TYPE == RK_TYPE_Q5_K ? 48 : 16;
    const int bq8 = 2 * ((iqs / 2) / 4), k4 = (iqs / 2) % 4;
    const uint32_t vl0 = *reinterpret_cast<const uint32_t*>(blk + QS + 16 * bq8 + 4 * k4);
    const uint32_t vl1 = *reinterpret_cast<const uint32_t*>(blk + QS + 16 * bq8 + 4 * k4 + 16);
    uint32_t vh0 = 0, vh1 = 0;
    if constexpr (TYPE == RK_TYPE_Q5_K) {
        vh0 = *reinterpret_cast<const uint32_t*>(blk + 16 + 4 * k4) >> bq8;
        vh1 = *reinterpret_cast<const uint32_t*>(blk + 16 + 4 * k4 + 16) >> bq8;
    }
    const uint32_t dm = *reinterpret_cast<const uint32_t*>(blk);
    float sumf_d = 0.0f, sumf_m = 0.0f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        int sc, m;
        kq_scale_min(blk + 4, bq8 + i, sc, m);
        const uint8_t* xb = x + (size_t) (bq8 + i) * 36;
        const int u0 = *reinterpret_cast<const int*>(xb + 4 + 4 * k4), u1 = *reinterpret_cast<const int*>(xb + 20 + 4 * k4);
        int v0 = (int) ((vl0 >> (4 * i)) & 0x0f0f0f0fu), v1 = (int) ((vl1 >> (4 * i)) & 0x0f0f0f0fu);
        int dot1, dot2;
        if constexpr (TYPE == RK_TYPE_Q5_K) {
            v0 |= (int) (((vh0 >> i) << 4) & 0x10101010u);
            v1 |= (int) (((vh1 >> i) << 4) & 0x10101010u);
            dot1 = __dp4a(v0, u0, __dp4a(v1, u1, 0));
            dot2 = __dp4a(0x01010101, u0, __dp4a(0x01010101, u1, 0));
        } else {
            dot1 = __dp4a(v1, u1, __dp4a(v0, u0, 0));
            dot2 = __dp4a(0x01010101, u1, __dp4a(0x01010101, u0, 0));
        }
        if (ip) {
            ip[2 * i] = dot1 * sc;
            ip[2 * i + 1] = dot2 * m;
        }
        const float d8 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(xb));
        sumf_d = __fadd_rn(sumf_d, __fmul_rn(d8, (float) (dot1 * sc)));
        sumf_m = __fadd_rn(sumf_m, __fmul_rn(d8, (float) (dot2 * m)));
    }
    return __fsub_rn(__fmul_rn(half_bits_to_float(dm), sumf_d), __fmul_rn(half_bits_to_float(dm >> 16), sumf_m));
}

template <int TYPE, int NC>
__device__ __forceinline__ void raw_row_dot(const uint8_t* wrow, const uint8_t* xq, size_t xcol, int n_in, int lane,
                                            float (&acc)[NC]) {
    if constexpr (TYPE == RK_TYPE_Q6_K) {
        const int iqs = lane;
        const int bq8 = 4 * (iqs / 16) + (iqs % 16) / 8;
        const int soff = 8 * (iqs / 16) + (iqs % 16) / 4;
        const int vh_shift = 2 * ((iqs % 16) / 8);
        for (int kb = 0; kb < n_in / 256; ++kb) {
            const uint8_t* blk = wrow + (size_t) kb * 210;
            const uint32_t vl = (uint32_t) ld_b2(blk + 4 * iqs);
            const uint32_t vh = (uint32_t) ld_b2(blk + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift;
            const float d = __half2float(*reinterpret_cast<const __half*>(blk + 208));
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                float sumf = 0.0f;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint8_t* xb = xq + c * xcol + (size_t) (kb * 8 + bq8 + 2 * i) * 36;
                    const int u = *reinterpret_cast<const int*>(xb + 4 + 4 * (iqs % 8));
                    const int usum = __dp4a(u, 0x01010101, 0);
                    const int sc = (int) (int8_t) blk[192 + soff + 4 * i];
                    const int vi = (int) (((vl >> (4 * i)) & 0x0f0f0f0fu) | (((vh >> (4 * i)) << 4) & 0x30303030u));
                    const int p = __dp4a(vi, u, -32 * usum) * sc;
                    sumf = __fmaf_rn(half_bits_to_float(*reinterpret_cast<const uint16_t*>(xb)), (float) p, sumf);
                }
                acc[c] = __fmaf_rn(d, sumf, acc[c]);
            }
        }
    } else if constexpr (TYPE == RK_TYPE_Q5_K || TYPE == RK_TYPE_Q4_K) {
        // lanes 0..15: the even blocks, 16..31 the odd ones; thread iqs = 2 * (lane % 16) of each
        const size_t bb = raw_row_bytes(TYPE, 256);
        for (int kb = lane >> 4; kb < n_in / 256; kb += 2) {
            const uint8_t* blk = wrow + (size_t) kb * bb;
#pragma unroll
            for (int c = 0; c < NC; ++c)
                acc[c] = __fadd_rn(acc[c], kq_q8_dot<TYPE>(blk, xq + c * xcol + (size_t) kb * 8 * 36, 2 * (lane & 15), nullptr));
        }
    } else {
        // lane l: ints 2*(l%4), 2*(l%4)+1 of blocks l/4, l/4 + 8, ...
        const int sub = lane >> 2, iqs = 2 * (lane & 3);
        for (int kb = sub; kb < n_in / 32; kb += 8) {
            const uint8_t* blk = wrow + (size_t) kb * 34;
            const int v0 = ld_b2(blk + 2 + 4 * iqs), v1 = ld_b2(blk + 2 + 4 * (iqs + 1));
            const float d0 = __half2float(*reinterpret_cast<const __half*>(blk));
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const uint8_t* xb = xq + c * xcol + (size_t) kb * 36;
                const int* u = reinterpret_cast<const int*>(xb + 4);
                const int s = __dp4a(v1, u[iqs + 1], __dp4a(v0, u[iqs], 0));
                const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(xb));
                acc[c] = __fmaf_rn(__fmul_rn(d0, d1), (float) s, acc[c]);
            }
        }
    }
}

template <int TYPE, int NC, bool RES>
__global__ void __launch_bounds__(128) mmvq_raw_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xq,
                                                       float* y, const float* res, float* __restrict__ partials,
                                                       int n_in, int n_out) {
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + warp;
    const size_t rb = raw_row_bytes(TYPE, n_in);
    const size_t xcol = (size_t) (n_in / 32) * 36;
    float acc[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
    if (row < n_out) raw_row_dot<TYPE, NC>(w + (size_t) row * rb, xq, xcol, n_in, lane, acc);
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[c] = warp_sum(acc[c]);
    if constexpr (!RES) {
        if (row < n_out && lane < NC) {
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if (lane == c) y[(size_t) c * n_out + row] = acc[c];
        }
    } else {
        __shared__ float rows[4];
        if (lane == 0 && row < n_out) {
            const float v = __fadd_rn(acc[0], res[row]);
            y[row] = v;
            rows[warp] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float part = 0.0f;
            for (int i = 0; i < 4 && blockIdx.x * 4 + i < n_out; ++i) part = __fmaf_rn(rows[i], rows[i], part);
            partials[blockIdx.x] = part;
        }
    }
}

// ---------------------------------------------------------------------------------------------------
// Load-time repack GGUF rows <-> packed tiles (the layout defined in mmvq.cuh). One thread per
// (tile, row, group).
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ int q6k_code(const uint8_t* blk, int v) {
    const int h = v >> 7, vv = v & 127, j = vv >> 5, l = vv & 31;
    const uint8_t qlb = blk[64 * h + l + 32 * (j & 1)];
    const int lo = (j >> 1) ? (qlb >> 4) : (qlb & 15);
    const int hi = (blk[128 + 32 * h + l] >> (2 * j)) & 3;
    return lo | (hi << 4);
}

template <int TYPE>
__global__ void pack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int n_in, long long n_items) {
    const long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_items) return;
    const int KC = n_in / 1024;
    const int g = (int) (idx & 31), r = (int) ((idx >> 5) & 3);
    const long long tile = idx >> 7;
    const long long rt = tile / KC;
    const int kc = (int) (tile % KC);
    const long long row = rt * 4 + r;
    if constexpr (TYPE == RK_TYPE_Q6_K) {
        uint8_t* t = dst + (size_t) tile * kQ6Tile;
        const int nb = n_in / 256, sb = 4 * kc + g / 8, gi = g % 8;
        const uint8_t* blk = src + ((size_t) row * nb + sb) * 210;
        int code[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) code[e] = q6k_code(blk, 32 * gi + e);
        // A (16 B): byte 4tt + b = code[4tt + b] (6 bits) | (code[16 + 4tt + b] >> 4) << 6;
        // B (8 B): byte 4u + b = low nibbles of code[16 + 8u + b] | code[20 + 8u + b] << 4 (q6_decode)
        uint8_t* qa = t + (r * 32 + g) * 16;
#pragma unroll
        for (int tt = 0; tt < 4; ++tt)
#pragma unroll
            for (int b = 0; b < 4; ++b)
                qa[4 * tt + b] = (uint8_t) ((code[4 * tt + b] & 63) | ((code[16 + 4 * tt + b] >> 4) << 6));
        uint8_t* qb = t + 2048 + (r * 32 + g) * 8;
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int b = 0; b < 4; ++b)
                qb[4 * u + b] = (uint8_t) ((code[16 + 8 * u + b] & 15) | ((code[20 + 8 * u + b] & 15) << 4));
        t[3072 + (g * 4 + r) * 2 + 0] = blk[192 + 2 * gi];
        t[3072 + (g * 4 + r) * 2 + 1] = blk[192 + 2 * gi + 1];
        if (gi == 0) {
            t[3328 + ((g / 8) * 4 + r) * 2 + 0] = blk[208];
            t[3328 + ((g / 8) * 4 + r) * 2 + 1] = blk[209];
        }
    } else {
        uint8_t* t = dst + (size_t) tile * kQ80Tile;
        const int nb = n_in / 32;
        const uint8_t* blk = src + ((size_t) row * nb + 32 * kc + g) * 34;
        for (int i = 0; i < 16; ++i) {
            t[((r * 2 + 0) * 32 + g) * 16 + i] = blk[2 + i];
            t[((r * 2 + 1) * 32 + g) * 16 + i] = blk[18 + i];
        }
        t[4096 + (g * 4 + r) * 2 + 0] = blk[0];
        t[4096 + (g * 4 + r) * 2 + 1] = blk[1];
    }
}

template <int TYPE>
__global__ void unpack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int n_in, long long n_items) {
    const long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_items) return;
    const int KC = n_in / 1024;
    const int g = (int) (idx & 31), r = (int) ((idx >> 5) & 3);
    const long long tile = idx >> 7;
    const long long rt = tile / KC;
    const int kc = (int) (tile % KC);
    const long long row = rt * 4 + r;
    if constexpr (TYPE == RK_TYPE_Q6_K) {
        const uint8_t* t = src + (size_t) tile * kQ6Tile;
        const int nb = n_in / 256, sb = 4 * kc + g / 8, gi = g % 8;
        uint8_t* blk = dst + ((size_t) row * nb + sb) * 210;
        // this group owns values 32gi..32gi+31: ql bytes 64h + l + 32(j&1) for its (h, j) and qh byte
        // 32h + l bits 2j..2j+1 are shared with other groups of the block, so rebuild whole bytes from
        // the four groups that share them: the group with gi % 4 == 0 of each half writes its half.
        if ((gi & 3) != 0) return;
        const int h = gi >> 2;  // values 128h .. 128h + 127 (groups gi..gi+3)
        const uint8_t* qap[4];
        const uint8_t* qbp[4];
        for (int j = 0; j < 4; ++j) {
            qap[j] = t + (r * 32 + g + j) * 16;
            qbp[j] = t + 2048 + (r * 32 + g + j) * 8;
        }
        auto code_of = [&](int j, int e) {  // group gi + j, value e (the layout pack_kernel writes)
            if (e < 16) return qap[j][e] & 63;
            const int T = (e - 16) >> 2, b = e & 3;
            const int nib = (qbp[j][4 * (T >> 1) + b] >> (4 * (T & 1))) & 15;
            return nib | ((qap[j][4 * T + b] >> 6) << 4);
        };
        for (int l = 0; l < 32; ++l) {
            // ql[64h + l]      : low nibble j=0 (group gi), high nibble j=2 (group gi+2)
            // ql[64h + 32 + l] : low nibble j=1 (group gi+1), high nibble j=3 (group gi+3)
            blk[64 * h + l] = (uint8_t) ((code_of(0, l) & 15) | ((code_of(2, l) & 15) << 4));
            blk[64 * h + 32 + l] = (uint8_t) ((code_of(1, l) & 15) | ((code_of(3, l) & 15) << 4));
            int qhb = 0;
            for (int j = 0; j < 4; ++j) qhb |= ((code_of(j, l) >> 4) & 3) << (2 * j);
            blk[128 + 32 * h + l] = (uint8_t) qhb;
        }
        for (int j = 0; j < 4; ++j) {
            blk[192 + 2 * (gi + j)] = t[3072 + ((g + j) * 4 + r) * 2 + 0];
            blk[192 + 2 * (gi + j) + 1] = t[3072 + ((g + j) * 4 + r) * 2 + 1];
        }
        if (gi == 0) {
            blk[208] = t[3328 + ((g / 8) * 4 + r) * 2 + 0];
            blk[209] = t[3328 + ((g / 8) * 4 + r) * 2 + 1];
        }
    } else {
        const uint8_t* t = src + (size_t) tile * kQ80Tile;
        const int nb = n_in / 32;
        uint8_t* blk = dst + ((size_t) row * nb + 32 * kc + g) * 34;
        for (int i = 0; i < 16; ++i) {
            blk[2 + i] = t[((r * 2 + 0) * 32 + g) * 16 + i];
            blk[18 + i] = t[((r * 2 + 1) * 32 + g) * 16 + i];
        }
        blk[0] = t[4096 + (g * 4 + r) * 2 + 0];
        blk[1] = t[4096 + (g * 4 + r) * 2 + 1];
    }
}

// ---------------------------------------------------------------------------------------------------
// Parity probe: the exact integer sums of the packed kernel, read straight from global memory with the
// same decode and dp4a chain (q6_decode / q6_subsums). One warp per tile, lane = group.
// ---------------------------------------------------------------------------------------------------
template <int TYPE>
__global__ void isums_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xq, int32_t* __restrict__ out,
                             int n_in, int n_out, int ncols) {
    const int KC = n_in / 1024;
    const long long tile = (long long) blockIdx.x * 4 + (threadIdx.x >> 5);
    if (tile >= (long long) (n_out / 4) * KC) return;
    const int lane = threadIdx.x & 31;
    const int rt = (int) (tile / KC), kc = (int) (tile % KC);
    const int g = kc * 32 + lane;  // global group index along n_in
    const size_t xcol = (size_t) (n_in / 32) * 36;
    for (int c = 0; c < ncols; ++c) {
        const int* blk = reinterpret_cast<const int*>(xq + c * xcol + (size_t) g * 36);
        const int4 xa = make_int4(blk[1], blk[2], blk[3], blk[4]);
        const int4 xb = make_int4(blk[5], blk[6], blk[7], blk[8]);
        if constexpr (TYPE == RK_TYPE_Q6_K) {
            const uint8_t* t = w + (size_t) tile * kQ6Tile;
            const int b0 = 32 * __dp4a(xa.x, 0x01010101, __dp4a(xa.y, 0x01010101, __dp4a(xa.z, 0x01010101, __dp4a(xa.w, 0x01010101, 0))));
            const int b1 = 32 * __dp4a(xb.x, 0x01010101, __dp4a(xb.y, 0x01010101, __dp4a(xb.z, 0x01010101, __dp4a(xb.w, 0x01010101, 0))));
            const uint2 scw = *reinterpret_cast<const uint2*>(t + 3072 + lane * 8);
            for (int r = 0; r < 4; ++r) {
                const uint4 ql = *reinterpret_cast<const uint4*>(t + (r * 32 + lane) * 16);
                const uint2 qh = *reinterpret_cast<const uint2*>(t + 2048 + (r * 32 + lane) * 8);
                int v[8];
                q6_decode(ql, qh, v);
                int s0, s1;
                q6_subsums(v, xa, xb, b0, b1, s0, s1);
                const uint32_t sw = r < 2 ? scw.x : scw.y;
                const int sc0 = sext8(sw, 2 * (r & 1)), sc1 = sext8(sw, 2 * (r & 1) + 1);
                int32_t* o = out + ((size_t) c * n_out + rt * 4 + r) * (n_in / 16);
                o[2 * g] = s0 * sc0;
                o[2 * g + 1] = s1 * sc1;
            }
        } else {
            const uint8_t* t = w + (size_t) tile * kQ80Tile;
            for (int r = 0; r < 4; ++r) {
                const int4 w0 = *reinterpret_cast<const int4*>(t + ((r * 2 + 0) * 32 + lane) * 16);
                const int4 w1 = *reinterpret_cast<const int4*>(t + ((r * 2 + 1) * 32 + lane) * 16);
                int s = __dp4a(w0.x, xa.x, 0);
                s = __dp4a(w0.y, xa.y, s);
                s = __dp4a(w0.z, xa.z, s);
                s = __dp4a(w0.w, xa.w, s);
                s = __dp4a(w1.x, xb.x, s);
                s = __dp4a(w1.y, xb.y, s);
                s = __dp4a(w1.z, xb.z, s);
                s = __dp4a(w1.w, xb.w, s);
                out[((size_t) c * n_out + rt * 4 + r) * (n_in / 32) + g] = s;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------
// host validation (the reference's validate_shape / validate_pointer / validate_stream,
// src/native_mmvq.cu:2312-2331)
// ---------------------------------------------------------------------------------------------------
bool type_ok(int type) {  // GGUF rows
    return type == RK_TYPE_Q6_K || type == RK_TYPE_Q8_0 || type == RK_TYPE_Q5_K || type == RK_TYPE_Q4_K;
}
bool packed_ok(int type) { return type == RK_TYPE_Q6_K || type == RK_TYPE_Q8_0; }  // packed tiles
int block_elems(int type) { return type == RK_TYPE_Q8_0 ? 32 : 256; }
bool kquant(int type) { return type == RK_TYPE_Q5_K || type == RK_TYPE_Q4_K; }
int check_ptr(const void* p, const char* what) {
    if (!p || (reinterpret_cast<uintptr_t>(p) & 3u) != 0)
        return set_error(RK_EINVAL, "%s: requires non-null 4-byte aligned device pointers", what);
    return RK_OK;
}
int check_ptr16(const void* p, const char* what) {
    if (!p || (reinterpret_cast<uintptr_t>(p) & 15u) != 0)
        return set_error(RK_EINVAL, "%s: packed weights must be 16-byte aligned", what);
    return RK_OK;
}
int check_stream(void* s, const char* what) {
    if (!s) return set_error(RK_EINVAL, "%s: requires an explicit non-null CUDA stream", what);
    return RK_OK;
}
int check_gemv_shape(int type, int n_in, int n_out, int ncols, const char* what) {
    if (!type_ok(type))
        return set_error(RK_EUNSUPPORTED, "%s: unsupported weight type %d (14 = Q6_K, 13 = Q5_K, 12 = Q4_K, 8 = Q8_0)", what, type);
    if (n_in <= 0 || n_in % block_elems(type) != 0)
        return set_error(RK_EINVAL, "%s: requires n_in > 0 and divisible by its block element count", what);
    if (n_out <= 0) return set_error(RK_EINVAL, "%s: requires n_out > 0", what);
    if (ncols < 1 || ncols > kMaxNcols) return set_error(RK_EINVAL, "%s: requires 1 <= ncols <= 16", what);
    return RK_OK;
}
int check_packed_shape(int type, int n_in, int n_out, int ncols, const char* what) {
    int rc = check_gemv_shape(type, n_in, n_out, ncols, what);
    if (rc) return rc;
    if (!packed_ok(type)) return set_error(RK_EUNSUPPORTED, "%s: type %d has no packed layout (Q6_K and Q8_0 do)", what, type);
    if (n_in % 1024 != 0 || n_out % 4 != 0)
        return set_error(RK_EINVAL, "%s: packed layout requires n_in %% 1024 == 0 and n_out %% 4 == 0", what);
    if (n_in > 32768) return set_error(RK_EINVAL, "%s: packed GEMV supports n_in <= 32768", what);
    return RK_OK;
}

template <int TYPE, bool RES>
cudaError_t raw_launch_cols(const uint8_t* w, const uint8_t* xq, float* y, const float* res, float* partials, int n_in,
                            int n_out, int nc, cudaStream_t s) {
    const dim3 grid((unsigned) ((n_out + 3) / 4));
    if constexpr (RES) return launch_pdl(mmvq_raw_kernel<TYPE, 1, true>, grid, dim3(128), 0, s, true, w, xq, y, res, partials, n_in, n_out);
    switch (nc) {
        case 1: return launch_pdl(mmvq_raw_kernel<TYPE, 1, false>, grid, dim3(128), 0, s, true, w, xq, y, res, partials, n_in, n_out);
        case 2: return launch_pdl(mmvq_raw_kernel<TYPE, 2, false>, grid, dim3(128), 0, s, true, w, xq, y, res, partials, n_in, n_out);
        case 3: return launch_pdl(mmvq_raw_kernel<TYPE, 3, false>, grid, dim3(128), 0, s, true, w, xq, y, res, partials, n_in, n_out);
        default: return launch_pdl(mmvq_raw_kernel<TYPE, 4, false>, grid, dim3(128), 0, s, true, w, xq, y, res, partials, n_in, n_out);
    }
}

template <bool RES>
cudaError_t raw_dispatch(int type, const uint8_t* w, const uint8_t* xq, float* y, const float* res, float* partials,
                         int n_in, int n_out, int nc, cudaStream_t s) {
    switch (type) {
        case RK_TYPE_Q6_K: return raw_launch_cols<RK_TYPE_Q6_K, RES>(w, xq, y, res, partials, n_in, n_out, nc, s);
        case RK_TYPE_Q5_K: return raw_launch_cols<RK_TYPE_Q5_K, RES>(w, xq, y, res, partials, n_in, n_out, nc, s);
        case RK_TYPE_Q4_K: return raw_launch_cols<RK_TYPE_Q4_K, RES>(w, xq, y, res, partials, n_in, n_out, nc, s);
        default: return raw_launch_cols<RK_TYPE_Q8_0, RES>(w, xq, y, res, partials, n_in, n_out, nc, s);
    }
}

// Parity probe for the K-quants on GGUF rows: one thread per (column, row, 32-value sub-block), the sums
// of dot1 * scale and dot2 * min over the four block threads that cover the sub-block (kq_q8_dot).
template <int TYPE>
__global__ void isums_kq_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xq, int32_t* __restrict__ out,
                                int n_in, int n_out, int ncols) {
    const long long nsub = n_in / 32;
    const long long idx = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long) ncols * n_out * nsub) return;
    const int s = (int) (idx % nsub);
    const long long cr = idx / nsub;
    const int r = (int) (cr % n_out), c = (int) (cr / n_out);
    const int kb = s / 8, j = s % 8, p = j / 2, i = j % 2;
    const uint8_t* blk = w + (size_t) r * raw_row_bytes(TYPE, n_in) + (size_t) kb * raw_row_bytes(TYPE, 256);
    const uint8_t* x = xq + (size_t) c * (n_in / 32) * 36 + (size_t) kb * 8 * 36;
    int a = 0, b = 0;
    for (int t = 4 * p; t < 4 * p + 4; ++t) {  // threads iqs = 2t cover sub-blocks 2p, 2p + 1
        int ip[4];
        kq_q8_dot<TYPE>(blk, x, 2 * t, ip);
        a += ip[2 * i];
        b += ip[2 * i + 1];
    }
    out[2 * idx] = a;
    out[2 * idx + 1] = b;
}

template <int TYPE, int EPI>
cudaError_t packed_launch_cols(MmvqParams p, int nc, cudaStream_t s) {
    switch (nc) {
        case 1: return mmvq_launch<TYPE, 1, PRO_Q8, EPI>(p, s, true);
        case 2: return mmvq_launch<TYPE, 2, PRO_Q8, EPI>(p, s, true);
        case 3: return mmvq_launch<TYPE, 3, PRO_Q8, EPI>(p, s, true);
        default: return mmvq_launch<TYPE, 4, PRO_Q8, EPI>(p, s, true);
    }
}

}  // namespace
}  // namespace rk

using namespace rk;

extern "C" {

size_t rk_q8_1_bytes(int n_in, int ncols) {
    if (n_in <= 0 || n_in % 32 != 0 || ncols < 1) return 0;
    return (size_t) ncols * (size_t) (n_in / 32) * 36u;
}

int rk_quantize_q8_1(const float* x, void* x_q8_1, int n_in, int ncols, void* stream) {
    const char* what = "rk_quantize_q8_1";
    if (n_in <= 0 || n_in % 32 != 0) return set_error(RK_EINVAL, "%s: requires n_in > 0 and divisible by 32", what);
    if (ncols < 1 || ncols > kMaxNcols) return set_error(RK_EINVAL, "%s: requires 1 <= ncols <= 16", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(x_q8_1, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const int nb = n_in / 32 * ncols;
    cudaError_t e = launch_pdl(quantize_q8_1_kernel, dim3((unsigned) ((nb + 7) / 8)), dim3(256), 0,
                               (cudaStream_t) stream, true, x, (uint8_t*) x_q8_1, nb);
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

size_t rk_weight_bytes(int type, int n_in, int n_out) {
    if (!type_ok(type) || n_in <= 0 || n_out <= 0 || n_in % block_elems(type) != 0) return 0;
    return raw_row_bytes(type, n_in) * (size_t) n_out;
}

size_t rk_packed_bytes(int type, int n_in, int n_out) {
    if (!packed_ok(type) || n_in <= 0 || n_out <= 0 || n_in % 1024 != 0 || n_out % 4 != 0) return 0;
    return rk_weight_bytes(type, n_in, n_out);
}

int rk_mmvq(int type, const void* weights, const void* x_q8_1, float* y, int n_in, int n_out, int ncols,
            void* stream) {
    const char* what = "rk_mmvq";
    if (int rc = check_gemv_shape(type, n_in, n_out, ncols, what)) return rc;
    if (!weights || (reinterpret_cast<uintptr_t>(weights) & (kquant(type) ? 3u : 1u)))
        return set_error(RK_EINVAL, "%s: requires non-null weights, 2-byte aligned (4-byte for Q5_K / Q4_K)", what);
    if (int rc = check_ptr(x_q8_1, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const size_t xcol = (size_t) (n_in / 32) * 36;
    for (int j = 0; j < ncols; j += 4) {
        const int nc = ncols - j < 4 ? ncols - j : 4;
        const uint8_t* xq = (const uint8_t*) x_q8_1 + (size_t) j * xcol;
        float* yj = y + (size_t) j * n_out;
        cudaError_t e = raw_dispatch<false>(type, (const uint8_t*) weights, xq, yj, nullptr, nullptr, n_in, n_out, nc,
                                            (cudaStream_t) stream);
        if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    return check_launch(what);
}

int rk_mmvq_res(int type, const void* weights, const void* x_q8_1, float* y, const float* res, float* partials,
                int n_in, int n_out, void* stream) {
    const char* what = "rk_mmvq_res";
    if (int rc = check_gemv_shape(type, n_in, n_out, 1, what)) return rc;
    if (!weights || (reinterpret_cast<uintptr_t>(weights) & (kquant(type) ? 3u : 1u)))
        return set_error(RK_EINVAL, "%s: requires non-null weights, 2-byte aligned (4-byte for Q5_K / Q4_K)", what);
    if (int rc = check_ptr(x_q8_1, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_ptr(res, what)) return rc;
    if (int rc = check_ptr(partials, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    cudaError_t e = raw_dispatch<true>(type, (const uint8_t*) weights, (const uint8_t*) x_q8_1, y, res, partials, n_in,
                                       n_out, 1, (cudaStream_t) stream);
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

int rk_pack_weights(int type, const void* src, void* dst, int n_in, int n_out, void* stream) {
    const char* what = "rk_pack_weights";
    if (int rc = check_packed_shape(type, n_in, n_out, 1, what)) return rc;
    if (!src || (reinterpret_cast<uintptr_t>(src) & 1u)) return set_error(RK_EINVAL, "%s: bad source pointer", what);
    if (int rc = check_ptr16(dst, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const long long items = (long long) (n_out / 4) * (n_in / 1024) * 128;
    const unsigned blocks = (unsigned) ((items + 255) / 256);
    if (type == RK_TYPE_Q6_K)
        pack_kernel<RK_TYPE_Q6_K><<<blocks, 256, 0, (cudaStream_t) stream>>>((const uint8_t*) src, (uint8_t*) dst, n_in, items);
    else
        pack_kernel<RK_TYPE_Q8_0><<<blocks, 256, 0, (cudaStream_t) stream>>>((const uint8_t*) src, (uint8_t*) dst, n_in, items);
    return check_launch(what);
}

int rk_unpack_weights(int type, const void* src, void* dst, int n_in, int n_out, void* stream) {
    const char* what = "rk_unpack_weights";
    if (int rc = check_packed_shape(type, n_in, n_out, 1, what)) return rc;
    if (int rc = check_ptr16(src, what)) return rc;
    if (!dst || (reinterpret_cast<uintptr_t>(dst) & 1u)) return set_error(RK_EINVAL, "%s: bad destination pointer", what);
    if (int rc = check_stream(stream, what)) return rc;
    const long long items = (long long) (n_out / 4) * (n_in / 1024) * 128;
    const unsigned blocks = (unsigned) ((items + 255) / 256);
    if (type == RK_TYPE_Q6_K)
        unpack_kernel<RK_TYPE_Q6_K><<<blocks, 256, 0, (cudaStream_t) stream>>>((const uint8_t*) src, (uint8_t*) dst, n_in, items);
    else
        unpack_kernel<RK_TYPE_Q8_0><<<blocks, 256, 0, (cudaStream_t) stream>>>((const uint8_t*) src, (uint8_t*) dst, n_in, items);
    return check_launch(what);
}

int rk_mmvq_packed_ex(int type, const void* packed, const void* x_q8_1, float* y, int n_in, int n_out, int ncols,
                      unsigned flags, void* stream) {
    const char* what = "rk_mmvq_packed";
    if (int rc = check_packed_shape(type, n_in, n_out, ncols, what)) return rc;
    if (int rc = check_ptr16(packed, what)) return rc;
    if (int rc = check_ptr(x_q8_1, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    if (flags & ~RK_FLAG_STATIC_WEIGHTS) return set_error(RK_EINVAL, "%s: unknown flags 0x%x", what, flags);
    const size_t xcol = (size_t) (n_in / 32) * 36;
    for (int j = 0; j < ncols; j += kMmvqMaxCols) {
        const int nc = ncols - j < kMmvqMaxCols ? ncols - j : kMmvqMaxCols;
        MmvqParams p = {};
        p.w = (const uint8_t*) packed;
        p.n_in = n_in;
        p.n_out = n_out;
        p.prefetch_before_wait = (flags & RK_FLAG_STATIC_WEIGHTS) ? 1 : 0;
        p.xq = (const uint8_t*) x_q8_1 + (size_t) j * xcol;
        p.y = y + (size_t) j * n_out;
        p.y_stride = n_out;
        cudaError_t e = type == RK_TYPE_Q6_K ? packed_launch_cols<RK_TYPE_Q6_K, EPI_STORE>(p, nc, (cudaStream_t) stream)
                                             : packed_launch_cols<RK_TYPE_Q8_0, EPI_STORE>(p, nc, (cudaStream_t) stream);
        if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    return check_launch(what);
}

int rk_mmvq_packed(int type, const void* packed, const void* x_q8_1, float* y, int n_in, int n_out, int ncols,
                   void* stream) {
    return rk_mmvq_packed_ex(type, packed, x_q8_1, y, n_in, n_out, ncols, 0u, stream);
}

int rk_mmvq_packed_res(int type, const void* packed, const void* x_q8_1, float* y, const float* res,
                       float* partials, int n_in, int n_out, int ncols, void* stream) {
    const char* what = "rk_mmvq_packed_res";
    if (int rc = check_packed_shape(type, n_in, n_out, ncols, what)) return rc;
    if (int rc = check_ptr16(packed, what)) return rc;
    if (int rc = check_ptr(x_q8_1, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_ptr(res, what)) return rc;
    if (int rc = check_ptr(partials, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const size_t xcol = (size_t) (n_in / 32) * 36;
    for (int j = 0; j < ncols; j += kMmvqMaxCols) {
        const int nc = ncols - j < kMmvqMaxCols ? ncols - j : kMmvqMaxCols;
        MmvqParams p = {};
        p.w = (const uint8_t*) packed;
        p.n_in = n_in;
        p.n_out = n_out;
        p.prefetch_before_wait = 0;
        p.xq = (const uint8_t*) x_q8_1 + (size_t) j * xcol;
        p.y = y + (size_t) j * n_out;
        p.y_stride = n_out;
        p.res = res + (size_t) j * n_out;
        p.res_stride = n_out;
        p.pout = partials + (size_t) j * (n_out / 4);
        p.pout_stride = n_out / 4;
        cudaError_t e = type == RK_TYPE_Q6_K ? packed_launch_cols<RK_TYPE_Q6_K, EPI_RES>(p, nc, (cudaStream_t) stream)
                                             : packed_launch_cols<RK_TYPE_Q8_0, EPI_RES>(p, nc, (cudaStream_t) stream);
        if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    return check_launch(what);
}

int rk_mmvq_isums(int type, const void* packed, const void* x_q8_1, int32_t* out, int n_in, int n_out, int ncols,
                  void* stream) {
    const char* what = "rk_mmvq_isums";
    if (kquant(type)) {  // GGUF rows (the K-quants have no packed layout)
        if (int rc = check_gemv_shape(type, n_in, n_out, ncols, what)) return rc;
        if (int rc = check_ptr(packed, what)) return rc;
        if (int rc = check_ptr(x_q8_1, what)) return rc;
        if (int rc = check_ptr(out, what)) return rc;
        if (int rc = check_stream(stream, what)) return rc;
        const long long items = (long long) ncols * n_out * (n_in / 32);
        const unsigned blocks = (unsigned) ((items + 255) / 256);
        if (type == RK_TYPE_Q5_K)
            isums_kq_kernel<RK_TYPE_Q5_K><<<blocks, 256, 0, (cudaStream_t) stream>>>((const uint8_t*) packed, (const uint8_t*) x_q8_1, out, n_in, n_out, ncols);
        else
            isums_kq_kernel<RK_TYPE_Q4_K><<<blocks, 256, 0, (cudaStream_t) stream>>>((const uint8_t*) packed, (const uint8_t*) x_q8_1, out, n_in, n_out, ncols);
        return check_launch(what);
    }
    if (int rc = check_packed_shape(type, n_in, n_out, ncols, what)) return rc;
    if (int rc = check_ptr16(packed, what)) return rc;
    if (int rc = check_ptr(x_q8_1, what)) return rc;
    if (int rc = check_ptr(out, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const long long tiles = (long long) (n_out / 4) * (n_in / 1024);
    const unsigned blocks = (unsigned) ((tiles + 3) / 4);
    if (type == RK_TYPE_Q6_K)
        isums_kernel<RK_TYPE_Q6_K><<<blocks, 128, 0, (cudaStream_t) stream>>>((const uint8_t*) packed, (const uint8_t*) x_q8_1, out, n_in, n_out, ncols);
    else
        isums_kernel<RK_TYPE_Q8_0><<<blocks, 128, 0, (cudaStream_t) stream>>>((const uint8_t*) packed, (const uint8_t*) x_q8_1, out, n_in, n_out, ncols);
    return check_launch(what);
}

}  // extern "C"
