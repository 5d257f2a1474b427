// elementwise.cu — norms, fused quantizers, gates and argmax of the decode step
// (src/qwythos.cpp:602-715 and :70-84 of the reference), C-ABI entry points.
#include "mmvq.cuh"

namespace rk {
namespace {

// row_sum_partials_kernel (:616-623): partials[b] = sum over rows 4b..4b+3 of x^2, in row order.
__global__ void row_sumsq_kernel(const float* __restrict__ x, float* __restrict__ partials, int n) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= (n + 3) / 4) return;
    float p = 0.0f;
    for (int i = 4 * b; i < 4 * b + 4 && i < n; ++i) p = __fmaf_rn(x[i], x[i], p);
    partials[b] = p;
}

// add_partials_1024_kernel (:602-614): x += o, then the partials of the new x.
__global__ void add_partials_kernel(float* __restrict__ x, const float* __restrict__ o, float* __restrict__ partials,
                                    int n) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= (n + 3) / 4) return;
    float p = 0.0f;
    for (int i = 4 * b; i < 4 * b + 4 && i < n; ++i) {
        const float v = __fadd_rn(x[i], o[i]);
        x[i] = v;
        p = __fmaf_rn(v, v, p);
    }
    partials[b] = p;
}

// rms_quant_apply_kernel (:627-655) / rms_norm_out_kernel (:658-672): blockIdx.y = column; every
// block reduces the column's partials with the fixed 256-thread tree, then warps walk 32-value blocks.
template <bool QUANT>
__global__ void __launch_bounds__(256) rms_apply_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                        const float* __restrict__ partials, void* __restrict__ out,
                                                        int cols, float eps) {
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.y;
    const float inv = rms_inv(block256_partials_sum(partials + (size_t) c * (cols / 4), cols / 4, red), cols, eps);
    const int lane = threadIdx.x & 31;
    const int nblk = cols >> 5;
    for (int blk = blockIdx.x * 8 + (threadIdx.x >> 5); blk < nblk; blk += gridDim.x * 8) {
        const int i = (blk << 5) + lane;
        const float v = rms_value(x[(size_t) c * cols + i], w[i], inv);
        if constexpr (QUANT)
            q8_1_warp_store(v, static_cast<uint8_t*>(out) + ((size_t) c * nblk + blk) * 36, lane);
        else
            static_cast<float*>(out)[(size_t) c * cols + i] = v;
    }
}

// swiglu_quant_kernel (:676-689) and sig_mul_quant_kernel (:692-704): one warp per 32-value block.
template <int KIND>
__global__ void __launch_bounds__(256) gate_quant_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                         uint8_t* __restrict__ y, int n) {
    pdl_trigger();
    pdl_wait();
    const int blk = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (blk >= n / 32) return;
    const int lane = threadIdx.x & 31;
    const int i = blk * 32 + lane;
    const float v = KIND == 0 ? swiglu_value(a[i], b[i]) : sigmul_value(a[i], b[i]);
    q8_1_warp_store(v, y + (size_t) blk * 36, lane);
}

// beta_gate_kernel (:707-715).
__device__ __forceinline__ float softplus_gate(float alpha, float dt, float ssm_a) {
    return rk_softplus_gate(alpha, dt, ssm_a);
}
__device__ __forceinline__ float sigmoidf_(float x) { return rk_sigmoidf(x); }

__global__ void beta_gate_kernel(float* __restrict__ beta, const float* __restrict__ alpha, const float* __restrict__ dt,
                                 const float* __restrict__ ssm_a, float* __restrict__ gate, int n) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    beta[i] = sigmoidf_(beta[i]);
    gate[i] = softplus_gate(alpha[i], dt[i], ssm_a[i]);
}

// The exactly specified transcendentals of common.cuh, one value per thread (a parity probe).
__global__ void math_probe_kernel(int fn, const float* __restrict__ x, float* __restrict__ y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = x[i];
    float r;
    switch (fn) {
        case 0: r = rk_expf(v); break;
        case 1: r = rk_logf(v); break;
        case 2: r = rk_log1pf(v); break;
        case 3: r = rk_sigmoidf(v); break;
        case 4: r = rk_siluf(v); break;
        case 5: r = rk_rsqrtf(v); break;
        default: r = expf(v); break;  // the CUDA library's expf, for the error-bound comparison only
    }
    y[i] = r;
}

// rms_norm_weighted (Strata; written definition): per row, ss by each thread's strided fma partial,
// xor tree per warp, warps added in order; x = x * rsqrt(ss/cols + eps) * w.
__global__ void __launch_bounds__(128) rms_rows_kernel(float* __restrict__ x, const float* __restrict__ w, int cols,
                                                       float eps) {
    __shared__ float red[4];
    pdl_trigger();
    pdl_wait();
    float* p = x + (size_t) blockIdx.x * cols;
    float part = 0.0f;
    for (int i = threadIdx.x; i < cols; i += 128) part = __fmaf_rn(p[i], p[i], part);
    part = warp_sum(part);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
    __syncthreads();
    const float ss = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
    const float inv = rk_rsqrtf(__fadd_rn(__fdiv_rn(ss, (float) cols), eps));
    for (int i = threadIdx.x; i < cols; i += 128) p[i] = __fmul_rn(__fmul_rn(p[i], inv), w[i]);
}

// Greedy argmax, one block per column: strict-greater scan per thread (lowest index within a thread),
// then the packed (value, ~index) maximum, which keeps the lowest index among equal values. NaN never wins.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int n, int* __restrict__ out) {
    __shared__ unsigned long long red[32];
    pdl_trigger();
    pdl_wait();
    const float* col = x + (size_t) blockIdx.x * n;
    float best = 0.0f;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = col[i];
        if (v == v && (bi < 0 || v > best)) {
            best = v;
            bi = i;
        }
    }
    unsigned long long key = bi >= 0 ? argmax_key(best, bi) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long k = red[0];
        for (int i = 1; i < (int) (blockDim.x >> 5); ++i) k = red[i] > k ? red[i] : k;
        out[blockIdx.x] = k ? argmax_key_row(k) : 0;
    }
}

int check_ptr(const void* p, const char* what) {
    if (!p || (reinterpret_cast<uintptr_t>(p) & 3u) != 0)
        return set_error(RK_EINVAL, "%s: requires non-null 4-byte aligned device pointers", what);
    return RK_OK;
}
int check_stream(void* s, const char* what) {
    if (!s) return set_error(RK_EINVAL, "%s: requires an explicit non-null CUDA stream", what);
    return RK_OK;
}
int launched(cudaError_t e, const char* what) {
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

}  // namespace
}  // namespace rk

using namespace rk;

extern "C" {

int rk_row_sumsq_partials(const float* x, float* partials, int n, void* stream) {
    const char* what = "rk_row_sumsq_partials";
    if (n <= 0) return set_error(RK_EINVAL, "%s: requires n > 0", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(partials, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const int slots = (n + 3) / 4;
    return launched(launch_pdl(row_sumsq_kernel, dim3((slots + 255) / 256), dim3(256), 0, (cudaStream_t) stream, true,
                               x, partials, n),
                    what);
}

int rk_add_partials(float* x, const float* o, float* partials, int n, void* stream) {
    const char* what = "rk_add_partials";
    if (n <= 0) return set_error(RK_EINVAL, "%s: requires n > 0", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(o, what)) return rc;
    if (int rc = check_ptr(partials, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const int slots = (n + 3) / 4;
    return launched(launch_pdl(add_partials_kernel, dim3((slots + 255) / 256), dim3(256), 0, (cudaStream_t) stream,
                               true, x, o, partials, n),
                    what);
}

static int rms_common(const float* x, const float* w, const float* partials, void* out, int cols, int ncols,
                      const char* what, void* stream) {
    if (cols <= 0 || cols % 32 != 0) return set_error(RK_EINVAL, "%s: requires cols > 0 and divisible by 32", what);
    if (ncols < 1 || ncols > 16) return set_error(RK_EINVAL, "%s: requires 1 <= ncols <= 16", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(w, what)) return rc;
    if (int rc = check_ptr(partials, what)) return rc;
    if (int rc = check_ptr(out, what)) return rc;
    return check_stream(stream, what);
}

int rk_rms_quant_q8_1(const float* x, const float* w, const float* partials, void* y, int cols, int ncols, float eps,
                      void* stream) {
    const char* what = "rk_rms_quant_q8_1";
    if (int rc = rms_common(x, w, partials, y, cols, ncols, what, stream)) return rc;
    const int gx = (cols / 32 + 7) / 8 < 16 ? (cols / 32 + 7) / 8 : 16;
    return launched(launch_pdl(rms_apply_kernel<true>, dim3(gx, ncols), dim3(256), 0, (cudaStream_t) stream, true, x, w,
                               partials, y, cols, eps),
                    what);
}

int rk_rms_norm_out(const float* x, const float* w, const float* partials, float* out, int cols, int ncols, float eps,
                    void* stream) {
    const char* what = "rk_rms_norm_out";
    if (int rc = rms_common(x, w, partials, out, cols, ncols, what, stream)) return rc;
    const int gx = (cols / 32 + 7) / 8 < 16 ? (cols / 32 + 7) / 8 : 16;
    return launched(launch_pdl(rms_apply_kernel<false>, dim3(gx, ncols), dim3(256), 0, (cudaStream_t) stream, true, x,
                               w, partials, (void*) out, cols, eps),
                    what);
}

int rk_swiglu_q8_1(const float* up, const float* gate, void* y, int n, void* stream) {
    const char* what = "rk_swiglu_q8_1";
    if (n <= 0 || n % 32 != 0) return set_error(RK_EINVAL, "%s: requires n > 0 and divisible by 32", what);
    if (int rc = check_ptr(up, what)) return rc;
    if (int rc = check_ptr(gate, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(launch_pdl(gate_quant_kernel<0>, dim3((n / 32 + 7) / 8), dim3(256), 0, (cudaStream_t) stream, true,
                               up, gate, (uint8_t*) y, n),
                    what);
}

int rk_sigmul_q8_1(const float* o, const float* g, void* y, int n, void* stream) {
    const char* what = "rk_sigmul_q8_1";
    if (n <= 0 || n % 32 != 0) return set_error(RK_EINVAL, "%s: requires n > 0 and divisible by 32", what);
    if (int rc = check_ptr(o, what)) return rc;
    if (int rc = check_ptr(g, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(launch_pdl(gate_quant_kernel<1>, dim3((n / 32 + 7) / 8), dim3(256), 0, (cudaStream_t) stream, true,
                               o, g, (uint8_t*) y, n),
                    what);
}

int rk_beta_gate(float* beta, const float* alpha, const float* dt, const float* ssm_a, float* gate, int n,
                 void* stream) {
    const char* what = "rk_beta_gate";
    if (n <= 0) return set_error(RK_EINVAL, "%s: requires n > 0", what);
    if (int rc = check_ptr(beta, what)) return rc;
    if (int rc = check_ptr(alpha, what)) return rc;
    if (int rc = check_ptr(dt, what)) return rc;
    if (int rc = check_ptr(ssm_a, what)) return rc;
    if (int rc = check_ptr(gate, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(launch_pdl(beta_gate_kernel, dim3((n + 255) / 256), dim3(256), 0, (cudaStream_t) stream, true, beta,
                               alpha, dt, ssm_a, gate, n),
                    what);
}

int rk_math_probe(int fn, const float* x, float* y, int n, void* stream) {
    const char* what = "rk_math_probe";
    if (n <= 0 || fn < 0 || fn > 6) return set_error(RK_EINVAL, "%s: requires n > 0 and 0 <= fn <= 6", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(y, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    math_probe_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t) stream>>>(fn, x, y, n);
    return check_launch(what);
}

int rk_rms_norm_rows(float* x, const float* w, int rows, int cols, float eps, void* stream) {
    const char* what = "rk_rms_norm_rows";
    if (rows <= 0 || cols <= 0) return set_error(RK_EINVAL, "%s: requires rows > 0 and cols > 0", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(w, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(launch_pdl(rms_rows_kernel, dim3(rows), dim3(128), 0, (cudaStream_t) stream, true, x, w, cols, eps),
                    what);
}

int rk_argmax(const float* x, int n, int ncols, int* out, void* stream) {
    const char* what = "rk_argmax";
    if (n <= 0 || ncols < 1) return set_error(RK_EINVAL, "%s: requires n > 0 and ncols >= 1", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(out, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(launch_pdl(argmax_kernel, dim3(ncols), dim3(1024), 0, (cudaStream_t) stream, true, x, n, out), what);
}

}  // extern "C"
