// gdn.cu — Gated DeltaNet decode kernels (src/fused_gdn.cu of the reference) for sm_100a.
//
//  * rk_gdn_conv_l2           causal conv1d (k = 4) + SiLU + per-head L2 over q/k heads; conv history is a
//                             4-slot ring indexed by position, ring[c*4 + (p & 3)] = input at position p.
//  * rk_gdn_step_norm_silu_q8 the delta-rule state step + RMSNorm * gamma * silu(z) + Q8_1, one cluster of
//                             4 CTAs per v-head (32 state columns per CTA); the head's RMS is reduced over
//                             distributed shared memory.
//  * rk_gdn_fused             the engine's whole recurrence for one layer and 1-2 tokens in one launch: one
//                             cluster of 8 CTAs per k-head kh serves v-heads kh and kh + h_k (the modulo
//                             pairing of src/fused_gdn.cu:57), computes the q/k conv + L2 once per cluster,
//                             steps the state per column (in registers), and writes the state after column 0
//                             to a snapshot for the verify's rollback.
//
// Per-column arithmetic follows the reference kernel's order: 32-row fma chains per row group, row groups
// added 0..3, per-32-column xor trees added quarter 0..3, so the q-scale read-out and both norms see the
// reference's reduction order. A 2-token launch runs column 1 after column 0 with identical code, so each
// column is bitwise equal to a 1-token launch.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace rk {
namespace {

constexpr int S = 128;                              // state size
constexpr float kInvSqrtS = 0.08838834764831845f;   // 1/sqrt(128)

__device__ __forceinline__ float silu_f(float x) { return rk_siluf(x); }
__device__ __forceinline__ float sigmoid_f(float x) { return rk_sigmoidf(x); }
__device__ __forceinline__ float softplus_gate(float alpha, float dt, float ssm_a) {
    return rk_softplus_gate(alpha, dt, ssm_a);
}
__device__ __forceinline__ float pick4(const float4 t, int i) {
    return i == 0 ? t.x : (i == 1 ? t.y : (i == 2 ? t.z : t.w));
}
// conv taps oldest first: sum = v0*w0, then fma(v1,w1), fma(v2,w2), fma(x,w3)
__device__ __forceinline__ float conv4(float v0, float v1, float v2, float x, const float4 w) {
    float s = __fmul_rn(v0, w.x);
    s = __fmaf_rn(v1, w.y, s);
    s = __fmaf_rn(v2, w.z, s);
    return __fmaf_rn(x, w.w, s);
}

// ---------------------------------------------------------------------------------------------------
// rk_gdn_conv_l2: one block per 128-channel head (gdn_conv_l2_kernel, src/fused_gdn.cu:113-133).
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(S) conv_l2_kernel(float* __restrict__ ring, const float* qkv,
                                                    const float* __restrict__ conv_w, float* h, int qk_heads, float eps,
                                                    const int* __restrict__ posp) {
    __shared__ float part[4];
    pdl_trigger();
    pdl_wait();
    const int pos = *posp;
    const int c = blockIdx.x * S + threadIdx.x;
    const float4 taps = reinterpret_cast<const float4*>(ring)[c];
    const float x = qkv[c];
    const float4 w = reinterpret_cast<const float4*>(conv_w)[c];
    const float sum = conv4(pick4(taps, (pos + 1) & 3), pick4(taps, (pos + 2) & 3), pick4(taps, (pos + 3) & 3), x, w);
    ring[(size_t) c * 4 + (pos & 3)] = x;
    float y = silu_f(sum);
    if ((int) blockIdx.x < qk_heads) {
        const float sq = warp_sum(__fmul_rn(y, y));
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
        __syncthreads();
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
        y = __fmul_rn(y, rk_rsqrtf(__fadd_rn(ss, eps)));
    }
    h[c] = y;
}

// ---------------------------------------------------------------------------------------------------
// The state step of one column for this CTA's 32 state columns (thread: col = tid % 32, row group
// rg = tid / 32, rows rg*32 .. rg*32+31 held in s[]). kq: [k (128) | q (128)] in smem. Returns the
// read-out oc (valid in every thread of the column).
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ float state_step(float (&s)[32], const float* kk, const float* qq, float v, float g,
                                            float beta, float (*red_kv)[32], float (*red_o)[32], int col, int rg) {
    float kv = 0.0f;
#pragma unroll
    for (int r = 0; r < 32; ++r) kv = __fmaf_rn(s[r], kk[rg * 32 + r], kv);
    red_kv[rg][col] = kv;
    __syncthreads();
    const float kv_col = __fadd_rn(__fadd_rn(__fadd_rn(red_kv[0][col], red_kv[1][col]), red_kv[2][col]), red_kv[3][col]);
    const float delta = __fmul_rn(__fsub_rn(v, __fmul_rn(g, kv_col)), beta);
    float o = 0.0f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
        s[r] = __fmaf_rn(g, s[r], __fmul_rn(kk[rg * 32 + r], delta));
        o = __fmaf_rn(s[r], qq[rg * 32 + r], o);
    }
    red_o[rg][col] = o;
    __syncthreads();
    return __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(red_o[0][col], red_o[1][col]), red_o[2][col]), red_o[3][col]),
                     kInvSqrtS);
}

// y = oc * rsqrt(ss/128 + eps) * gamma * silu(z), evaluated left to right.
__device__ __forceinline__ float gated_out(float oc, float ss, float eps, float gamma, float z) {
    const float scale = rk_rsqrtf(__fadd_rn(__fdiv_rn(ss, (float) S), eps));
    return __fmul_rn(__fmul_rn(__fmul_rn(oc, scale), gamma), silu_f(z));
}

// ---------------------------------------------------------------------------------------------------
// rk_gdn_step_norm_silu_q8: cluster of 4 CTAs per v-head, 128 threads each.
// ---------------------------------------------------------------------------------------------------
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(128)
    step_norm_kernel(float* __restrict__ state, const float* __restrict__ q, const float* __restrict__ k,
                     const float* __restrict__ v, const float* __restrict__ gate, const float* __restrict__ beta,
                     const float* __restrict__ z, const float* __restrict__ gamma, float eps, float* __restrict__ y,
                     uint8_t* __restrict__ q8, int h_k, int h_v) {
    __shared__ float kq[2 * S];
    __shared__ float red_kv[4][32], red_o[4][32];
    __shared__ float rms_part[4];
    cg::cluster_group cluster = cg::this_cluster();
    pdl_trigger();
    pdl_wait();
    const int head = blockIdx.x >> 2, quarter = (int) cluster.block_rank();
    const int tid = threadIdx.x, col = tid & 31, rg = tid >> 5;
    const int qh = head % h_k;
    kq[tid] = k[qh * S + tid];
    kq[S + tid] = q[qh * S + tid];
    float s[32];
    float* base = state + ((size_t) (rg * 32) * h_v + head) * S + quarter * 32 + col;
    const size_t rs = (size_t) h_v * S;
#pragma unroll
    for (int r = 0; r < 32; ++r) s[r] = base[r * rs];
    __syncthreads();
    const float g = rk_expf(gate[head]);
    const float oc = state_step(s, kq, kq + S, v[head * S + quarter * 32 + col], g, beta[head], red_kv, red_o, col, rg);
#pragma unroll
    for (int r = 0; r < 32; ++r) base[r * rs] = s[r];
    if (rg == 0) {
        const float sq = warp_sum(__fmul_rn(oc, oc));
        if (col == 0)
            for (int dst = 0; dst < 4; ++dst) cluster.map_shared_rank(rms_part, dst)[quarter] = sq;
    }
    cluster.sync();
    if (rg == 0) {
        const float ss = __fadd_rn(__fadd_rn(__fadd_rn(rms_part[0], rms_part[1]), rms_part[2]), rms_part[3]);
        const int j = quarter * 32 + col;
        const float yv = gated_out(oc, ss, eps, gamma[j], z[head * S + j]);
        y[head * S + j] = yv;
        if (q8) q8_1_warp_store(yv, q8 + ((size_t) head * 4 + quarter) * 36, col);
    }
}

// ---------------------------------------------------------------------------------------------------
// rk_gdn_fused: one cluster of 8 CTAs per k-head kh. Rank r: v-head kh + h_k*(r/4), quarter r%4; for
// the conv it owns q/k channels r*32 .. r*32+31 of head kh's [q 128 | k 128] and the 32 v channels of
// its own quarter.
// ---------------------------------------------------------------------------------------------------
template <int NC>
__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(128)
    fused_kernel(const float* __restrict__ proj, int proj_stride, float* __restrict__ ring,
                 const float* __restrict__ conv_w, const float* __restrict__ dt_bias, const float* __restrict__ ssm_a,
                 const float* __restrict__ gamma, float* __restrict__ state, float* __restrict__ snap,
                 const int* __restrict__ rollback, float* __restrict__ y, uint8_t* __restrict__ q8, int h_k, int h_v,
                 const int* __restrict__ posp, float eps) {
    __shared__ float qk_raw[NC][2 * S];   // raw silu(conv) of head kh's q | k (broadcast by all 8 ranks)
    __shared__ float qk_ss[NC][8];        // per-rank sum of squares of its 32 q/k channels
    __shared__ float kq[NC][2 * S];       // normalized [k | q] per column
    __shared__ float vloc[NC][32];
    __shared__ float red_kv[NC][4][32], red_o[NC][4][32];
    __shared__ float rms_part[NC][4];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int) cluster.block_rank();
    const int kh = blockIdx.x >> 3;
    const int head = kh + h_k * (rank >> 2), quarter = rank & 3;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int ch_v0 = 2 * h_k * S;              // first v channel
    const int off_z = ch_v0 + h_v * S;          // z block in the projection output
    const int off_beta = off_z + h_v * S, off_alpha = off_beta + h_v;
    const size_t rs = (size_t) h_v * S;
    float* sbase = state + ((size_t) (wid * 32) * h_v + head) * S + quarter * 32 + lane;
    float* pbase = snap + ((size_t) (wid * 32) * h_v + head) * S + quarter * 32 + lane;
    // The state, conv weights and ring rows do not depend on the upstream kernel's output: warm L2.
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(sbase + r * rs));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(pbase + r * rs));
    }
    pdl_trigger();
    pdl_wait();
    const int pos = *posp;
    const bool from_snap = *rollback != 0;

    // ---- conv + silu for this rank's 32 q/k channels (warp 0) and 32 v channels (warp 1) ----
    if (wid < 2) {
        int ch;
        if (wid == 0) {
            const int j = rank * 32 + lane;  // 0..255 within [q | k] of head kh
            ch = j < S ? kh * S + j : h_k * S + kh * S + (j - S);
        } else {
            ch = ch_v0 + head * S + quarter * 32 + lane;
        }
        const float4 taps = reinterpret_cast<const float4*>(ring)[ch];
        const float4 w = reinterpret_cast<const float4*>(conv_w)[ch];
        float x[NC], yv[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) x[c] = proj[(size_t) c * proj_stride + ch];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            // inputs at positions pos+c-3 .. pos+c-1: from the ring below pos, else from this launch
            float in[3];
#pragma unroll
            for (int t = 0; t < 3; ++t) {
                const int d = c - 3 + t;  // position pos + d
                in[t] = d < 0 ? pick4(taps, (pos + d) & 3) : x[d < 0 ? 0 : d];
            }
            yv[c] = silu_f(conv4(in[0], in[1], in[2], x[c], w));
        }
        // ring writes (after this thread's reads): every q/k channel of head kh has exactly one owner
        // rank in the cluster, every v channel its own CTA, so no two CTAs touch the same ring row
#pragma unroll
        for (int c = 0; c < NC; ++c) ring[(size_t) ch * 4 + ((pos + c) & 3)] = x[c];
        if (wid == 0) {
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float sq = warp_sum(__fmul_rn(yv[c], yv[c]));
#pragma unroll
                for (int dst = 0; dst < 8; ++dst) {
                    float* rq = cluster.map_shared_rank(&qk_raw[c][0], dst);
                    rq[rank * 32 + lane] = yv[c];
                    if (lane == 0) cluster.map_shared_rank(&qk_ss[c][0], dst)[rank] = sq;
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < NC; ++c) vloc[c][lane] = yv[c];
        }
    }
    cluster.sync();

    // ---- L2-normalize q (ranks 0-3's partials) and k (ranks 4-7's) per column ----
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const float ssq = __fadd_rn(__fadd_rn(__fadd_rn(qk_ss[c][0], qk_ss[c][1]), qk_ss[c][2]), qk_ss[c][3]);
        const float ssk = __fadd_rn(__fadd_rn(__fadd_rn(qk_ss[c][4], qk_ss[c][5]), qk_ss[c][6]), qk_ss[c][7]);
        kq[c][S + tid] = __fmul_rn(qk_raw[c][tid], rk_rsqrtf(__fadd_rn(ssq, eps)));       // q
        kq[c][tid] = __fmul_rn(qk_raw[c][S + tid], rk_rsqrtf(__fadd_rn(ssk, eps)));       // k
    }
    // ---- the state step, column by column, state in registers ----
    float s[32];
    const float* src = from_snap ? pbase : sbase;
#pragma unroll
    for (int r = 0; r < 32; ++r) s[r] = src[r * rs];
    __syncthreads();
    float oc[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const float* pc = proj + (size_t) c * proj_stride;
        const float beta = sigmoid_f(pc[off_beta + head]);
        const float g = rk_expf(softplus_gate(pc[off_alpha + head], dt_bias[head], ssm_a[head]));
        oc[c] = state_step(s, kq[c], kq[c] + S, vloc[c][lane], g, beta, red_kv[c], red_o[c], lane, wid);
        if (NC > 1 && c == 0) {
#pragma unroll
            for (int r = 0; r < 32; ++r) pbase[r * rs] = s[r];
        }
    }
#pragma unroll
    for (int r = 0; r < 32; ++r) sbase[r * rs] = s[r];
    // ---- gated RMSNorm over the head's 128 outputs (the 4 CTAs of this head) ----
    if (wid == 0) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float sq = warp_sum(__fmul_rn(oc[c], oc[c]));
            if (lane == 0)
                for (int d = 0; d < 4; ++d) cluster.map_shared_rank(&rms_part[c][0], (rank & 4) + d)[quarter] = sq;
        }
    }
    cluster.sync();
    if (wid == 0) {
        const int j = quarter * 32 + lane;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float ss = __fadd_rn(__fadd_rn(__fadd_rn(rms_part[c][0], rms_part[c][1]), rms_part[c][2]), rms_part[c][3]);
            const float yv = gated_out(oc[c], ss, eps, gamma[j], proj[(size_t) c * proj_stride + off_z + head * S + j]);
            y[(size_t) c * h_v * S + head * S + j] = yv;
            q8_1_warp_store(yv, q8 + ((size_t) c * h_v * 4 + head * 4 + quarter) * 36, lane);
        }
    }
}

int check_ptr(const void* p, const char* what) {
    if (!p || (reinterpret_cast<uintptr_t>(p) & 3u) != 0)
        return set_error(RK_EINVAL, "%s: requires non-null 4-byte aligned device pointers", what);
    return RK_OK;
}
int check_ptr16(const void* p, const char* what) {
    if (!p || (reinterpret_cast<uintptr_t>(p) & 15u) != 0)
        return set_error(RK_EINVAL, "%s: ring and conv weights must be 16-byte aligned", what);
    return RK_OK;
}
int check_stream(void* s, const char* what) {
    if (!s) return set_error(RK_EINVAL, "%s: requires an explicit non-null CUDA stream", what);
    return RK_OK;
}

}  // namespace

cudaError_t gdn_fused_launch(const float* proj, int proj_stride, float* ring, const float* conv_w, const float* dt_bias,
                             const float* ssm_a, const float* gamma, float* state, float* snap, const int* rollback,
                             float* y, uint8_t* q8, int h_k, int h_v, int ncols, const int* pos, float eps,
                             cudaStream_t s, bool pdl) {
    const dim3 grid((unsigned) (h_k * 8)), block(128);
    if (ncols == 1)
        return launch_pdl(fused_kernel<1>, grid, block, 0, s, pdl, proj, proj_stride, ring, conv_w, dt_bias, ssm_a,
                          gamma, state, snap, rollback, y, q8, h_k, h_v, pos, eps);
    return launch_pdl(fused_kernel<2>, grid, block, 0, s, pdl, proj, proj_stride, ring, conv_w, dt_bias, ssm_a, gamma,
                      state, snap, rollback, y, q8, h_k, h_v, pos, eps);
}

}  // namespace rk

using namespace rk;

extern "C" {

int rk_gdn_conv_l2(float* ring, const float* qkv, const float* conv_w, float* h, int channels, int qk_heads,
                   float eps, const int* pos, void* stream) {
    const char* what = "rk_gdn_conv_l2";
    if (channels <= 0 || channels % S != 0 || qk_heads < 0 || qk_heads > channels / S)
        return set_error(RK_EINVAL, "%s: invalid arguments (channels %% 128 == 0, 0 <= qk_heads <= channels/128)", what);
    if (int rc = check_ptr16(ring, what)) return rc;
    if (int rc = check_ptr16(conv_w, what)) return rc;
    if (int rc = check_ptr(qkv, what)) return rc;
    if (int rc = check_ptr(h, what)) return rc;
    if (int rc = check_ptr(pos, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    cudaError_t e = launch_pdl(conv_l2_kernel, dim3((unsigned) (channels / S)), dim3(S), 0, (cudaStream_t) stream, true,
                               ring, qkv, conv_w, h, qk_heads, eps, pos);
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

int rk_gdn_step_norm_silu_q8(float* state, const float* q, const float* k, const float* v, const float* gate,
                             const float* beta, const float* z, const float* gamma, float eps, float* y, void* q8,
                             int h_k, int h_v, void* stream) {
    const char* what = "rk_gdn_step_norm_silu_q8";
    if (h_k <= 0 || h_v <= 0 || h_v % h_k) return set_error(RK_EINVAL, "%s: invalid arguments (h_v %% h_k == 0)", what);
    const void* ptrs[] = {state, q, k, v, gate, beta, z, gamma, y};
    for (const void* p : ptrs)
        if (int rc = check_ptr(p, what)) return rc;
    if (q8 && (reinterpret_cast<uintptr_t>(q8) & 3u)) return set_error(RK_EINVAL, "%s: q8 must be 4-byte aligned", what);
    if (int rc = check_stream(stream, what)) return rc;
    cudaError_t e = launch_pdl(step_norm_kernel, dim3((unsigned) (h_v * 4)), dim3(128), 0, (cudaStream_t) stream, true,
                               state, q, k, v, gate, beta, z, gamma, eps, y, (uint8_t*) q8, h_k, h_v);
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

int rk_gdn_fused(const float* proj, int proj_stride, float* ring, const float* conv_w, const float* dt_bias,
                 const float* ssm_a, const float* gamma, float* state, float* snap, const int* rollback, float* y,
                 void* q8, int h_k, int h_v, int ncols, const int* pos, float eps, void* stream) {
    const char* what = "rk_gdn_fused";
    if (h_k <= 0 || h_v != 2 * h_k) return set_error(RK_EINVAL, "%s: requires h_v == 2 * h_k", what);
    if (ncols < 1 || ncols > 2) return set_error(RK_EINVAL, "%s: requires 1 <= ncols <= 2", what);
    if (proj_stride < 2 * h_k * S + 2 * h_v * S + 2 * h_v)
        return set_error(RK_EINVAL, "%s: proj_stride smaller than one projection column", what);
    const void* ptrs[] = {proj, dt_bias, ssm_a, gamma, state, snap, rollback, y, q8, pos};
    for (const void* p : ptrs)
        if (int rc = check_ptr(p, what)) return rc;
    if (int rc = check_ptr16(ring, what)) return rc;
    if (int rc = check_ptr16(conv_w, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    cudaError_t e = gdn_fused_launch(proj, proj_stride, ring, conv_w, dt_bias, ssm_a, gamma, state, snap, rollback, y,
                                     (uint8_t*) q8, h_k, h_v, ncols, pos, eps, (cudaStream_t) stream, true);
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

}  // extern "C"
