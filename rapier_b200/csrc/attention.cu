// attention.cu — the GQA attention layer's decode kernels (src/qwythos.cpp:320-442 of the reference):
// split q/gate, per-head RMSNorm, partial RoPE, fp16 KV store, and split-L flash-decode attention.
//
// KV cache layout: fp16 [n_kv][max_ctx][hd] (head-major, so one head's token chunk is contiguous).
//
// Flash decode: the tokens are cut into fixed chunks of kChunk = 256 starting at token 0; one CTA per
// (chunk, kv head) scores the chunk against the kv head's n_head/n_kv query heads for every query column,
// takes the chunk's max and exp-sum, and accumulates its weighted V; a combine kernel merges the chunks
// of each (head, column) in chunk order. Column c attends tokens 0..pos+c; its chunk partition and every
// reduction depend only on its own position, so a 2-column launch gives each column the bits of a
// 1-column launch at that position.
#include <mutex>

#include "mmvq.cuh"

namespace rk {
namespace {

constexpr int kChunk = 256;
constexpr int kHd = 256;

// ---- split_qg_kernel (:320-327) ----
__global__ void split_qg_kernel(const float* __restrict__ qg, float* __restrict__ q, float* __restrict__ g, int heads,
                                int hd) {
    pdl_trigger();
    pdl_wait();
    const int h = blockIdx.x;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        q[(size_t) h * hd + i] = qg[(size_t) h * 2 * hd + i];
        g[(size_t) h * hd + i] = qg[(size_t) h * 2 * hd + hd + i];
    }
}

// ---- RoPE (Strata native_rope_apply; written definition): NEOX rotate-half over the first n_rot dims,
// cos/sin from a host-built table. out = (x0*c - x1*s, x0*s + x1*c), each product rounded separately.
__device__ __forceinline__ void rope_pair(float& a, float& b, float c, float s) {
    const float x0 = a, x1 = b;
    a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    b = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}
__global__ void rope_kernel(float* __restrict__ x, int hd, int n_rot, const float* __restrict__ table, int max_pos,
                            const int* __restrict__ posp) {
    pdl_trigger();
    pdl_wait();
    const int pos = *posp, half = n_rot / 2;
    if (pos < 0 || pos >= max_pos) {
        if (threadIdx.x == 0) atomicOr(&g_rk_status, kStatusBadIndex);
        return;
    }
    float* p = x + (size_t) blockIdx.x * hd;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float c = table[((size_t) pos * half + i) * 2 + 0], s = table[((size_t) pos * half + i) * 2 + 1];
        rope_pair(p[i], p[i + half], c, s);
    }
}

// ---- store_kv2_kernel (:340-345), fp16 head-major caches ----
__global__ void store_kv_kernel(__half* __restrict__ kc, __half* __restrict__ vc, const float* __restrict__ k,
                                const float* __restrict__ v, const int* __restrict__ posp, int n_kv, int hd,
                                int max_ctx) {
    pdl_trigger();
    pdl_wait();
    const int pos = *posp;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_kv * hd) return;
    if (pos < 0 || pos >= max_ctx) {
        if (i == 0) atomicOr(&g_rk_status, kStatusBadIndex);
        return;
    }
    const int h = i / hd, d = i - h * hd;
    const size_t dst = ((size_t) h * max_ctx + pos) * hd + d;
    kc[dst] = __float2half_rn(k[i]);
    vc[dst] = __float2half_rn(v[i]);
}

// ---- flash-decode chunk kernel ----
// grid (chunks, n_kv), 256 threads. q: [NC][n_head][256] fp32. Partials: o [n_head][NC][max_chunks][256],
// m / l [n_head][NC][max_chunks].
template <int NC, int G>
__global__ void __launch_bounds__(256) gqa_chunk_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                                                        const __half* __restrict__ vc, float* __restrict__ part_o,
                                                        float* __restrict__ part_ml, int n_head, int max_ctx,
                                                        int max_chunks, const int* __restrict__ posp, float scale) {
    __shared__ float sc[G][NC][kChunk];
    __shared__ float mstat[G][NC];
    pdl_trigger();
    pdl_wait();
    const int pos = *posp;
    if (pos < 0 || pos + NC > max_ctx) {  // out of the cache: record and do nothing
        if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicOr(&g_rk_status, kStatusBadIndex);
        return;
    }
    const int chunk = blockIdx.x, kvh = blockIdx.y;
    const int t0 = chunk * kChunk;
    if (t0 > pos + NC - 1) return;  // beyond every column
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const __half* kbase = kc + ((size_t) kvh * max_ctx + t0) * kHd;
    const __half* vbase = vc + ((size_t) kvh * max_ctx + t0) * kHd;
    const int ntok = min(kChunk, pos + NC - t0);  // tokens any column may read in this chunk

    // this lane's 8 query dims for every (group head, column)
    float qr[G][NC][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float4* qp = reinterpret_cast<const float4*>(q + ((size_t) c * n_head + kvh * G + g) * kHd + lane * 8);
            const float4 a = qp[0], b = qp[1];
            qr[g][c][0] = a.x; qr[g][c][1] = a.y; qr[g][c][2] = a.z; qr[g][c][3] = a.w;
            qr[g][c][4] = b.x; qr[g][c][5] = b.y; qr[g][c][6] = b.z; qr[g][c][7] = b.w;
        }
    // phase 1: scores, one warp per token, lanes over 8-dim slices, xor tree per (head, column)
    for (int t = warp; t < ntok; t += 8) {
        const uint4 kraw = *reinterpret_cast<const uint4*>(kbase + (size_t) t * kHd + lane * 8);
        const __half2* kh2 = reinterpret_cast<const __half2*>(&kraw);
        float kf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(kh2[i]);
            kf[2 * i] = f.x;
            kf[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                float d = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) d = __fmaf_rn(qr[g][c][i], kf[i], d);
                d = warp_sum(d);
                if (lane == 0) sc[g][c][t] = (t0 + t <= pos + c) ? __fmul_rn(d, scale) : -INFINITY;
            }
    }
    __syncthreads();
    // phase 2: per (head, column) the chunk max and the exponentials, one warp per pair
    for (int pair = warp; pair < G * NC; pair += 8) {
        const int g = pair / NC, c = pair % NC;
        float m = -INFINITY;
        for (int t = lane; t < ntok; t += 32) m = fmaxf(m, sc[g][c][t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < ntok; t += 32) {
            const float e = m == -INFINITY ? 0.0f : rk_expf(__fsub_rn(sc[g][c][t], m));  // masked: exp(-inf) = 0
            sc[g][c][t] = e;
            l = __fadd_rn(l, e);
        }
        l = warp_sum(l);
        if (lane == 0) {
            mstat[g][c] = m;
            float* ml = part_ml + (((size_t) (kvh * G + g) * NC + c) * max_chunks + chunk) * 2;
            ml[0] = m;
            ml[1] = l;
        }
    }
    __syncthreads();
    // phase 3: weighted V, thread = output dim
    float acc[G][NC];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < NC; ++c) acc[g][c] = 0.0f;
    for (int t = 0; t < ntok; ++t) {
        const float vv = __half2float(vbase[(size_t) t * kHd + tid]);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int c = 0; c < NC; ++c) acc[g][c] = __fmaf_rn(sc[g][c][t], vv, acc[g][c]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < NC; ++c)
            part_o[(((size_t) (kvh * G + g) * NC + c) * max_chunks + chunk) * kHd + tid] = acc[g][c];
    (void) mstat;
}

// ---- combine: grid (n_head, NC), 256 threads (thread = dim). Chunks merged in order. With gate/q8 set it
// also writes the Q8_1 blocks of o * sigmoid(gate) (sig_mul_quant_kernel, src/qwythos.cpp:692-704; one
// warp = one 32-dim block). ----
template <int NC>
__global__ void __launch_bounds__(256) gqa_combine_kernel(const float* __restrict__ part_o,
                                                          const float* __restrict__ part_ml, float* __restrict__ o,
                                                          int n_head, int max_chunks, const int* __restrict__ posp,
                                                          const float* __restrict__ gate, uint8_t* __restrict__ q8) {
    pdl_trigger();
    pdl_wait();
    const int h = blockIdx.x, c = blockIdx.y, d = threadIdx.x;
    const int pos = *posp;
    if (pos < 0 || pos + NC > max_chunks * kChunk) return;  // recorded by the chunk kernel
    const int nchunks = (pos + c) / kChunk + 1;
    const float* ml = part_ml + ((size_t) h * NC + c) * max_chunks * 2;
    const float* po = part_o + ((size_t) h * NC + c) * max_chunks * kHd;
    float M = -INFINITY;
    for (int k = 0; k < nchunks; ++k) M = fmaxf(M, ml[2 * k]);
    float num = 0.0f, den = 0.0f;
    for (int k = 0; k < nchunks; ++k) {
        const float w = rk_expf(__fsub_rn(ml[2 * k], M));
        num = __fmaf_rn(w, po[(size_t) k * kHd + d], num);
        den = __fmaf_rn(w, ml[2 * k + 1], den);
    }
    const float ov = __fdiv_rn(num, den);
    const size_t oi = ((size_t) c * n_head + h) * kHd + d;
    o[oi] = ov;
    if (q8 != nullptr)
        q8_1_warp_store(sigmul_value(ov, gate[oi]), q8 + (((size_t) c * n_head + h) * (kHd / 32) + (d >> 5)) * 36, d & 31);
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

size_t gqa_scratch_bytes(int n_head, int ncols, int max_ctx) {
    const size_t chunks = (size_t) (max_ctx + kChunk - 1) / kChunk;
    return (size_t) n_head * ncols * chunks * (kHd + 2) * sizeof(float);
}

// Launch the chunk + combine kernels (the engine calls this directly with PDL).
cudaError_t gqa_launch(const float* q, const __half* kc, const __half* vc, float* o, int n_head, int n_kv, int ncols,
                       const int* pos, int max_ctx, float scale, float* scratch, cudaStream_t s, bool pdl,
                       const float* gate, uint8_t* q8) {
    const int max_chunks = (max_ctx + kChunk - 1) / kChunk;
    float* part_o = scratch;
    float* part_ml = scratch + (size_t) n_head * ncols * max_chunks * kHd;
    const dim3 grid((unsigned) max_chunks, (unsigned) n_kv);
    cudaError_t e;
    if (n_head / n_kv != 4) return cudaErrorInvalidValue;
    if (ncols == 1)
        e = launch_pdl(gqa_chunk_kernel<1, 4>, grid, dim3(256), 0, s, pdl, q, kc, vc, part_o, part_ml, n_head, max_ctx,
                       max_chunks, pos, scale);
    else
        e = launch_pdl(gqa_chunk_kernel<2, 4>, grid, dim3(256), 0, s, pdl, q, kc, vc, part_o, part_ml, n_head, max_ctx,
                       max_chunks, pos, scale);
    if (e != cudaSuccess) return e;
    if (ncols == 1)
        return launch_pdl(gqa_combine_kernel<1>, dim3((unsigned) n_head, 1), dim3(256), 0, s, pdl, part_o, part_ml, o,
                          n_head, max_chunks, pos, gate, q8);
    return launch_pdl(gqa_combine_kernel<2>, dim3((unsigned) n_head, 2), dim3(256), 0, s, pdl, part_o, part_ml, o, n_head,
                      max_chunks, pos, gate, q8);
}

}  // namespace rk

using namespace rk;

extern "C" {

int rk_split_qg(const float* qg, float* q, float* g, int heads, int hd, void* stream) {
    const char* what = "rk_split_qg";
    if (heads <= 0 || hd <= 0) return set_error(RK_EINVAL, "%s: requires heads > 0 and hd > 0", what);
    if (int rc = check_ptr(qg, what)) return rc;
    if (int rc = check_ptr(q, what)) return rc;
    if (int rc = check_ptr(g, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(launch_pdl(split_qg_kernel, dim3(heads), dim3(256), 0, (cudaStream_t) stream, true, qg, q, g, heads, hd),
                    what);
}

int rk_rope(float* x, int heads, int hd, int n_rot, const float* table, int max_pos, const int* pos, void* stream) {
    const char* what = "rk_rope";
    if (heads <= 0 || hd <= 0 || n_rot <= 0 || n_rot > hd || n_rot % 2)
        return set_error(RK_EINVAL, "%s: requires 0 < n_rot <= hd, n_rot even", what);
    if (int rc = check_ptr(x, what)) return rc;
    if (int rc = check_ptr(table, what)) return rc;
    if (int rc = check_ptr(pos, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    if (max_pos <= 0) return set_error(RK_EINVAL, "%s: requires max_pos > 0", what);
    return launched(launch_pdl(rope_kernel, dim3(heads), dim3(64), 0, (cudaStream_t) stream, true, x, hd, n_rot, table,
                               max_pos, pos),
                    what);
}

int rk_store_kv_f16(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v, const int* pos, int n_kv,
                    int hd, int max_ctx, void* stream) {
    const char* what = "rk_store_kv_f16";
    if (n_kv <= 0 || hd <= 0 || max_ctx <= 0) return set_error(RK_EINVAL, "%s: requires n_kv, hd, max_ctx > 0", what);
    if (!kcache || !vcache || (reinterpret_cast<uintptr_t>(kcache) & 1u) || (reinterpret_cast<uintptr_t>(vcache) & 1u))
        return set_error(RK_EINVAL, "%s: requires non-null 2-byte aligned caches", what);
    if (int rc = check_ptr(k, what)) return rc;
    if (int rc = check_ptr(v, what)) return rc;
    if (int rc = check_ptr(pos, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    const int n = n_kv * hd;
    return launched(launch_pdl(store_kv_kernel, dim3((n + 255) / 256), dim3(256), 0, (cudaStream_t) stream, true,
                               (__half*) kcache, (__half*) vcache, k, v, pos, n_kv, hd, max_ctx),
                    what);
}

size_t rk_gqa_scratch_bytes(int n_head, int ncols, int max_ctx) {
    if (n_head <= 0 || ncols < 1 || max_ctx <= 0) return 0;
    return gqa_scratch_bytes(n_head, ncols, max_ctx);
}

int rk_gqa_decode_f16(const float* q, const uint16_t* kcache, const uint16_t* vcache, float* o, int n_head, int n_kv,
                      int hd, int ncols, const int* pos, int max_ctx, float scale, void* scratch, size_t scratch_bytes,
                      void* stream) {
    const char* what = "rk_gqa_decode_f16";
    if (hd != kHd) return set_error(RK_EINVAL, "%s: requires hd == 256", what);
    if (n_kv <= 0 || n_head != 4 * n_kv) return set_error(RK_EINVAL, "%s: requires n_head == 4 * n_kv", what);
    if (ncols < 1 || ncols > 2) return set_error(RK_EINVAL, "%s: requires 1 <= ncols <= 2", what);
    if (max_ctx <= 0) return set_error(RK_EINVAL, "%s: requires max_ctx > 0", what);
    if (scratch_bytes < gqa_scratch_bytes(n_head, ncols, max_ctx))
        return set_error(RK_EINVAL, "%s: scratch smaller than rk_gqa_scratch_bytes()", what);
    if (!q || (reinterpret_cast<uintptr_t>(q) & 15u)) return set_error(RK_EINVAL, "%s: q must be 16-byte aligned", what);
    if (!kcache || !vcache || (reinterpret_cast<uintptr_t>(kcache) & 15u) || (reinterpret_cast<uintptr_t>(vcache) & 15u))
        return set_error(RK_EINVAL, "%s: caches must be 16-byte aligned", what);
    if (int rc = check_ptr(o, what)) return rc;
    if (int rc = check_ptr(pos, what)) return rc;
    if (int rc = check_ptr(scratch, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    return launched(gqa_launch(q, (const __half*) kcache, (const __half*) vcache, o, n_head, n_kv, ncols, pos, max_ctx,
                               scale, (float*) scratch, (cudaStream_t) stream, true, nullptr, nullptr),
                    what);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------
// Allocation-free attention for callers that cannot allocate device memory themselves: for example a
// plugin loaded into an application that hands all device memory to its own pool and forbids raw
// cudaMalloc, or a decode loop that cannot afford the device-wide synchronization cudaMalloc / cudaFree
// imply. The chunk partials live in the file-scope array below instead of a caller buffer. Every GPU that
// loads this library holds the array (16 MiB) until the process exits.
//
// Set-up: the first call on each device looks up the array's device address with cudaGetSymbolAddress
// (with that device current) and caches it; make that first call before any stream capture. Host code
// never hands the symbol itself to a kernel: on the host it is only a stand-in, not a device address.
//
// Sharing: all calls on a device use the same array and it keeps the last call's contents. Nothing in it
// has to start at zero (the chunk kernel writes every partial the combine reads in the same call), but
// calls whose kernels overlap on the GPU (other streams, other host threads) race on the array and must
// be serialized by the caller.
// ---------------------------------------------------------------------------------------------------
namespace rk {
namespace {
constexpr size_t kNoAllocScratchBytes = (size_t) 16 << 20;
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};
}  // namespace
}  // namespace rk

static __device__ __align__(256) float g_gqa_noalloc_scratch[rk::kNoAllocScratchBytes / sizeof(float)];

extern "C" int rk_gqa_decode_f16_noalloc(const float* q, const uint16_t* kcache, const uint16_t* vcache, float* o,
                                         int n_head, int n_kv, int hd, int ncols, const int* pos, int max_ctx,
                                         float scale, void* stream) {
    const char* what = "rk_gqa_decode_f16_noalloc";
    if (hd != kHd) return set_error(RK_EINVAL, "%s: requires hd == 256", what);
    if (n_kv <= 0 || n_head != 4 * n_kv) return set_error(RK_EINVAL, "%s: requires n_head == 4 * n_kv", what);
    if (ncols < 1 || ncols > 2) return set_error(RK_EINVAL, "%s: requires 1 <= ncols <= 2", what);
    if (max_ctx <= 0) return set_error(RK_EINVAL, "%s: requires max_ctx > 0", what);
    const size_t need = gqa_scratch_bytes(n_head, ncols, max_ctx);
    if (need > kNoAllocScratchBytes)
        return set_error(RK_EINVAL,
                         "%s: n_head %d x ncols %d x max_ctx %d needs %zu bytes of partials, above the built-in %zu "
                         "(use rk_gqa_decode_f16 with a caller buffer)",
                         what, n_head, ncols, max_ctx, need, kNoAllocScratchBytes);
    if (!q || (reinterpret_cast<uintptr_t>(q) & 15u)) return set_error(RK_EINVAL, "%s: q must be 16-byte aligned", what);
    if (!kcache || !vcache || (reinterpret_cast<uintptr_t>(kcache) & 15u) || (reinterpret_cast<uintptr_t>(vcache) & 15u))
        return set_error(RK_EINVAL, "%s: caches must be 16-byte aligned", what);
    if (int rc = check_ptr(o, what)) return rc;
    if (int rc = check_ptr(pos, what)) return rc;
    if (int rc = check_stream(stream, what)) return rc;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(RK_ECUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
    if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(RK_EINVAL, "%s: device %d out of range", what, dev);
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_gqa_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return set_error(RK_ECUDA, "%s: cudaGetSymbolAddress: %s", what, cudaGetErrorString(e));
            g_noalloc_ptr[dev] = p;
        }
        scratch = g_noalloc_ptr[dev];
    }
    return launched(gqa_launch(q, (const __half*) kcache, (const __half*) vcache, o, n_head, n_kv, ncols, pos, max_ctx,
                               scale, static_cast<float*>(scratch), (cudaStream_t) stream, true, nullptr, nullptr),
                    what);
}
