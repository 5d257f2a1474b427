// common.cuh — shared device helpers for the rapier_b200 sm_100a kernels: block formats, warp
// reductions, the Q8_1 block rules, PTX wrappers for mbarriers / bulk copies / programmatic dependent
// launch, bounded waits, and the host-side error plumbing of the C-ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <utility>

#include "../../include/rapier_b200.h"

namespace rk {

constexpr int WARP = 32;
constexpr int kQ6Tile = 3360;   // packed Q6_K tile: 4 rows x 1024 values
constexpr int kQ80Tile = 4352;  // packed Q8_0 tile: 4 rows x 1024 values

// ---------------------------------------------------------------------------------------------
// Error plumbing: every C-ABI entry returns 0 or a negative RK_E* code and records a message that
// rk_last_error() returns (thread-local). Device-side bounded waits that give up set a bit in a
// per-module device word that rk_device_status() reads.
// ---------------------------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
void clear_error();

// ---------------------------------------------------------------------------------------------
// warp reductions (xor butterfly, offsets 16..1: every lane ends with the same value)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Warp sums of M values (a power of two) per lane as a reduce-scatter: at xor offsets 16, 8, ... each lane
// keeps half of its values and adds the partner's copy of that half; once one value is left, plain
// butterfly steps. Every step adds the same two partial sums that warp_sum adds for that value (fp32
// addition is commutative), so each sum is bitwise warp_sum's, for M - 1 shuffles (M <= 32) instead of 5 M.
// Afterwards v[0 .. R), R = max(M / 32, 1), hold sums: v[i] on lane l is the sum of value i + R * l when
// M >= 32, and of value l >> (5 - log2 M) when M < 32 (the 32 / M lanes of a value agree).
template <int M>
__device__ __forceinline__ void rs_step(float* v, int lane, int o) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < M / 2; ++i) {
        const float send = hi ? v[i] : v[i + M / 2];
        const float keep = hi ? v[i + M / 2] : v[i];
        v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
}
template <int M, int O>
__device__ __forceinline__ void rs_level(float* v, int lane) {
    if constexpr (O > 0) {
        if constexpr (M > 1) {
            rs_step<M>(v, lane, O);
            rs_level<M / 2, O / 2>(v, lane);
        } else {
            v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], O));
            rs_level<1, O / 2>(v, lane);
        }
    }
}
template <int M>
__device__ __forceinline__ void warp_reduce_scatter(float (&v)[M], int lane) {
    static_assert(M >= 1 && (M & (M - 1)) == 0, "a power of two");
    rs_level<M, 16>(v, lane);
}

// ---------------------------------------------------------------------------------------------
// Transcendentals with an exactly specified operation sequence. Every step is one IEEE-754 fp32
// operation rounded to nearest even (or an exact bit manipulation), so the CPU oracle, which writes the
// same sequence in C, gets the same bits. The reference computes these with the vendor library's expf /
// __expf / log1pf / rsqrtf, whose last-ulp behaviour is not specified; these stay within ~1 ulp of the
// true value (tests compare with float64).
//
// rk_expf: Cody-Waite argument reduction and a Taylor polynomial (W. J. Cody, W. Waite, "Software
// Manual for the Elementary Functions", 1980, ch. 6): n = rint(x * log2 e); r = x - n * C1 - n * C2
// with C1 = 355/512 (9 significant bits, so n * C1 is exact inside the fma) and C2 = ln 2 - C1;
// exp(r) = sum_{k<=7} r^k / k! by Horner's rule with fused multiply-adds (|r| <= 0.35: the first
// omitted term is below 6e-9 relative); the result is p * 2^n, applied as two exact power-of-two
// factors 2^(n/2) and 2^(n - n/2) so that overflow gives inf and underflow rounds once.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float rk_pow2i(int e) { return __int_as_float((e + 127) << 23); }  // -126 <= e <= 127
__device__ __forceinline__ float rk_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return __int_as_float(0x7f800000);
    if (x < -104.0f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269502f));
    float r = __fmaf_rn(-n, 0.693359375f, x);
    r = __fmaf_rn(-n, -2.12194440e-4f, r);
    float p = 1.98412698e-4f;
    p = __fmaf_rn(p, r, 1.38888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333e-3f);
    p = __fmaf_rn(p, r, 4.16666667e-2f);
    p = __fmaf_rn(p, r, 1.66666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int) n, n1 = ni / 2;
    return __fmul_rn(__fmul_rn(p, rk_pow2i(n1)), rk_pow2i(ni - n1));
}
// rk_logf for x > 0 finite: x = m * 2^e with m in [sqrt(1/2), sqrt(2)); s = (m - 1) / (m + 1);
// log m = 2 s (1 + s^2/3 + s^4/5 + ... + s^10/11) (the atanh series, |s| <= 0.172); log x = e * ln2 + log m
// with ln 2 split in two parts. Subnormal x is scaled by 2^24 first.
__device__ __forceinline__ float rk_logf(float x) {
    int bias = 0;
    if (x < 1.17549435e-38f) {
        x = __fmul_rn(x, 16777216.0f);
        bias = -24;
    }
    const int bits = __float_as_int(x);
    int e = ((bits >> 23) & 0xff) - 127;
    float m = __int_as_float((bits & 0x007fffff) | 0x3f800000);
    if (m > 1.41421354f) {
        m = __fmul_rn(m, 0.5f);
        e += 1;
    }
    e += bias;
    const float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    const float s2 = __fmul_rn(s, s);
    float q = 9.09090909e-2f;
    q = __fmaf_rn(q, s2, 1.11111111e-1f);
    q = __fmaf_rn(q, s2, 1.42857143e-1f);
    q = __fmaf_rn(q, s2, 2.00000000e-1f);
    q = __fmaf_rn(q, s2, 3.33333333e-1f);
    const float lm = __fmaf_rn(__fmul_rn(__fmul_rn(2.0f, s), s2), q, __fmul_rn(2.0f, s));
    const float fe = (float) e;
    return __fmaf_rn(fe, 0.693359375f, __fmaf_rn(fe, -2.12194440e-4f, lm));
}
// rk_log1pf for t >= 0 (softplus only feeds it exp values): u = 1 + t; t when u == 1, else
// log(u) * t / (u - 1), which cancels the rounding error of 1 + t (D. Goldberg, "What every computer
// scientist should know about floating-point arithmetic", 1991, Theorem 4).
__device__ __forceinline__ float rk_log1pf(float t) {
    if (t != t || t == __int_as_float(0x7f800000)) return t;
    const float u = __fadd_rn(1.0f, t);
    if (u == 1.0f) return t;
    return __fdiv_rn(__fmul_rn(rk_logf(u), t), __fsub_rn(u, 1.0f));
}
// 1 / sqrt(x), two correctly rounded operations (the reference uses rsqrtf, an approximation).
__device__ __forceinline__ float rk_rsqrtf(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }
__device__ __forceinline__ float rk_sigmoidf(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, rk_expf(-x))); }
__device__ __forceinline__ float rk_siluf(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, rk_expf(-x))); }
// The GDN decay input softplus(alpha + dt) * ssm_a, softplus passing v through above 20 (beta_gate_kernel,
// src/qwythos.cpp:707-715).
__device__ __forceinline__ float rk_softplus_gate(float alpha, float dt, float ssm_a) {
    const float v = __fadd_rn(alpha, dt);
    return __fmul_rn(v > 20.0f ? v : rk_log1pf(rk_expf(v)), ssm_a);
}

// ---------------------------------------------------------------------------------------------
// Q8_1 block rules (the reference's q8_1_finite / q8_1_quant / q8_1_ds are out of its tree; this is
// the written definition the CPU oracle restates):
//   d = amax / 127, clamped to 65504 when NaN, infinite or above the fp16 maximum;
//   q = 0 for an all-zero block, else roundf(x / d) clamped to [-127, 127];
//   stored {half(d), half(sum clamped to +-65504, NaN -> 0)}.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float q8_finite_d(float d) { return (d <= 65504.0f) ? d : 65504.0f; }
__device__ __forceinline__ int q8_quant(float x, float d, float amax) {
    if (amax == 0.0f) return 0;
    float q = roundf(__fdiv_rn(x, d));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    return (int) q;
}
__device__ __forceinline__ float q8_ds_sum(float s) {
    if (s != s) return 0.0f;
    return fminf(fmaxf(s, -65504.0f), 65504.0f);
}
// Quantize one value per lane of a full warp as one Q8_1 block (lane l owns value l): returns lane l's
// int8 code and sets `ds` to the packed half2 {d, sum} word (the same on every lane).
__device__ __forceinline__ int q8_1_warp_code(float v, uint32_t& ds) {
    const float amax = warp_max(fabsf(v));
    const float sum = warp_sum(v);
    const float d = q8_finite_d(__fdiv_rn(amax, 127.0f));
    const __half2 h = __halves2half2(__float2half_rn(d), __float2half_rn(q8_ds_sum(sum)));
    ds = *reinterpret_cast<const uint32_t*>(&h);
    return q8_quant(v, d, amax);
}
// The same block written to global memory in the 36-byte layout (blk = the block's first byte).
__device__ __forceinline__ void q8_1_warp_store(float v, uint8_t* blk, int lane) {
    uint32_t ds;
    const int code = q8_1_warp_code(v, ds);
    reinterpret_cast<int8_t*>(blk + 4)[lane] = (int8_t) code;
    if (lane == 0) *reinterpret_cast<uint32_t*>(blk) = ds;
}

// ---------------------------------------------------------------------------------------------
// PTX wrappers (sm_90+ forms, valid on sm_100a)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on an mbarrier. No multicast.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
// Barrier over threads 0..255 (named barrier 1). The 256-thread op bodies and GEMV prologues use it so they
// also run on the first 8 warps of the persistent decode kernel's 512-thread CTA; in a 256-thread block
// it is __syncthreads.
__device__ __forceinline__ void block_sync256() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Programmatic dependent launch: wait for the upstream grid's memory, and let the downstream grid launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Device status word (one per translation unit; rk_device_status() ORs and clears them all):
// bit 0 = an mbarrier wait gave up (a bulk copy did not land within the bound), bit 1 = a cluster
// handshake gave up, bit 2 = an index a kernel was handed was out of range, bit 3 = a grid barrier of
// the persistent decode kernel gave up.
static __device__ unsigned int g_rk_status = 0;
constexpr unsigned kStatusWaitTimeout = 1u;
constexpr unsigned kStatusClusterTimeout = 2u;
constexpr unsigned kStatusBadIndex = 4u;
constexpr unsigned kStatusGridTimeout = 8u;
typedef unsigned (*StatusReader)(bool clear);
void register_status_reader(StatusReader r);
namespace {
unsigned read_status_this_tu(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_rk_status, sizeof v) != cudaSuccess) return 0x80000000u;
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_rk_status, &z, sizeof z);
    }
    return v;
}
struct StatusRegistrar {
    StatusRegistrar() { register_status_reader(&read_status_this_tu); }
};
static StatusRegistrar g_status_registrar;
}  // namespace
// Bounded mbarrier wait: try_wait suspends for a hardware-defined slice per call; 1<<22 calls is far
// beyond any legal copy latency. On giving up it records the status bit and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (uint32_t it = 0; it < (1u << 22); ++it)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(&g_rk_status, kStatusWaitTimeout);
    return false;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// ---------------------------------------------------------------------------------------------
// Host-side launch helper: cudaLaunchKernelEx with the programmatic-stream-serialization attribute
// (the kernel may start while the previous kernel on the stream finishes; it calls pdl_wait() before
// touching that kernel's outputs).
// ---------------------------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int num_sms();

}  // namespace rk
