// persistent.cuh — the two executors of a decode op program (decode_ops.cuh).
//
// * op_kernel<NC>: one launch per non-GEMV op (grid = the op's largest item count, one item per block,
//   blocks past the op's live item count return); GEMV ops launch mmvq_packed_kernel. The engine
//   captures the launches of a program in a CUDA graph.
// * persistent_kernel<NC>: the whole program in one cooperative launch, one 256-thread CTA per SM. Ops
//   run in program order separated by grid barriers; the items of a non-GEMV op are dealt to CTAs
//   round-robin. The weight tiles of every GEMV stream through per-warp rings of `stages` 3360-B slots
//   (one 1-D bulk copy and one mbarrier per slot, lane 0 issuing) whose producer cursor walks the
//   program's GEMV sequence ahead of the consumer: the slots a warp frees at the end of one GEMV are
//   refilled with the next GEMV's tiles, so HBM keeps streaming through the op's tail, the grid barrier,
//   the next prologue and the non-GEMV ops in between. With `until` > 0 the program repeats while
//   ctrl->n_emitted < until, at most `max_iters` times (a whole generation in one launch), and the
//   producer wraps around to the program's first GEMV.
//
// A GEMV's work split (contiguous unit ranges per CTA, units dealt to warps round-robin) and its per-row
// arithmetic are those of mmvq_packed_kernel, so both executors write the same bits.
//
// Failure handling: every mbarrier wait and grid-barrier spin is bounded. A CTA that gives up sets the
// sticky `abort` word and a status bit; every CTA then skips the rest of the program, waits (bounded)
// for its own bulk copies still in flight and exits. The last CTA to exit resets the barrier counter,
// so each launch starts from zero.
#pragma once

#include "decode_ops.cuh"

namespace rk {

struct PSync {
    unsigned long long arrive;  // grid-barrier arrivals of the running launch
    unsigned exits;             // CTAs of the running launch that have finished
    unsigned abort;             // sticky give-up flag, cleared by the host
};

constexpr unsigned long long kGridSpinNs = 1000000000ull;  // a grid barrier gives up after 1 s

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p) {
    return *reinterpret_cast<const volatile unsigned*>(p);
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Grid barrier: the counter starts at 0 in every launch and every barrier adds gridDim.x arrivals.
// Returns false when the program must stop (abort seen, or this spin gave up).
__device__ __forceinline__ bool grid_sync(PSync* sync, unsigned long long& target, int* flag) {
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&sync->arrive, 1ull);
        int good = 1;
        unsigned long long t0 = 0;
        for (uint32_t it = 0; ld_acquire_u64(&sync->arrive) < target; ++it) {
            if (ld_volatile_u32(&sync->abort)) {
                good = 0;
                break;
            }
            if ((it & 63u) == 0u) {
                const unsigned long long now = globaltimer_ns();
                if (it == 0u) {
                    t0 = now;
                } else if (now - t0 > kGridSpinNs) {
                    atomicOr(&g_rk_status, kStatusGridTimeout);
                    atomicExch(&sync->abort, 1u);
                    good = 0;
                    break;
                }
            }
            __nanosleep(32);
        }
        if (good && ld_volatile_u32(&sync->abort)) good = 0;
        __threadfence();
        *flag = good;
    }
    __syncthreads();
    return *flag != 0;
}

// ---------------------------------------------------------------------------------------------------
// Per-warp weight ring. All lanes keep the same cursor state; lane 0 issues the copies.
// ---------------------------------------------------------------------------------------------------
struct WarpPipe {
    uint32_t bar0, ring0;  // shared-memory addresses of the warp's first mbarrier and first slot
    const uint8_t* ring;
    int stages;
    int cs;         // consumer slot
    uint32_t cpar;  // consumer phase parity
    int ps;         // producer slot
    int inflight;   // tiles issued and not yet consumed
    int pj, pu, puend, pkc, pKC;  // producer cursor: op (-1: none left), unit, unit end, k-chunk, k-chunks
    const uint8_t* pw;
    uint64_t pol;
    int wrap;
};

// Point the producer at the first GEMV op at or after `from` (wrapping once when w.wrap) that has units
// for this warp.
__device__ __forceinline__ void pipe_seek(WarpPipe& w, const POp* prog, int nops, int from, int warp) {
    for (int n = 0; n < nops; ++n) {
        int j = from + n;
        if (j >= nops) {
            if (!w.wrap) break;
            j -= nops;
        }
        const POp& op = prog[j];
        if (op.kind != POP_GEMV) continue;
        const int units = op.g.n_out >> 2;
        const int ubeg = (int) (((long long) blockIdx.x * units) / gridDim.x);
        const int uend = (int) (((long long) (blockIdx.x + 1) * units) / gridDim.x);
        if (ubeg + warp < uend) {
            w.pj = j;
            w.pu = ubeg + warp;
            w.puend = uend;
            w.pkc = 0;
            w.pKC = op.g.n_in >> 10;
            w.pw = op.g.w;
            return;
        }
    }
    w.pj = -1;
}

__device__ __forceinline__ void pipe_issue(WarpPipe& w, const POp* prog, int nops, int warp, int lane) {
    if (w.pj < 0) return;
    if (lane == 0) {
        const uint32_t bar = w.bar0 + 8u * (uint32_t) w.ps;
        mbar_arrive_expect_tx(bar, kQ6Tile);
        bulk_g2s(w.ring0 + (uint32_t) (w.ps * kQ6Tile), w.pw + ((size_t) w.pu * w.pKC + w.pkc) * kQ6Tile, kQ6Tile, bar,
                 w.pol);
    }
    if (++w.ps == w.stages) w.ps = 0;
    ++w.inflight;
    if (++w.pkc == w.pKC) {
        w.pkc = 0;
        w.pu += kMmvqWarps;
        if (w.pu >= w.puend) pipe_seek(w, prog, nops, w.pj + 1, warp);
    }
}

__device__ __forceinline__ bool pipe_wait(const WarpPipe& w) {
    const bool landed = mbar_wait_bounded(w.bar0 + 8u * (uint32_t) w.cs, w.cpar);
    return __all_sync(0xffffffffu, landed);
}

// The warp is done reading the current slot: hand it back to the async proxy and refill it.
__device__ __forceinline__ void pipe_release(WarpPipe& w, const POp* prog, int nops, int warp, int lane) {
    __syncwarp();
    if (lane == 0) fence_proxy_async_smem();
    --w.inflight;
    if (++w.cs == w.stages) {
        w.cs = 0;
        w.cpar ^= 1u;
    }
    pipe_issue(w, prog, nops, warp, lane);
}

// Wait (bounded) for every copy still in flight, so no copy lands after the CTA has exited.
__device__ __forceinline__ void pipe_drain(WarpPipe& w) {
    int s = w.cs;
    uint32_t par = w.cpar;
    for (int k = 0; k < w.inflight; ++k) {
        mbar_wait_bounded(w.bar0 + 8u * (uint32_t) s, par);
        if (++s == w.stages) {
            s = 0;
            par ^= 1u;
        }
    }
    w.inflight = 0;
}

// One GEMV op: the prologue builds the staged activations, then every unit of this CTA's range that
// belongs to this warp is accumulated tile by tile from the ring (mmvq_packed_kernel's loop).
template <int NC, int PRO, int EPI>
__device__ __forceinline__ bool p_gemv(const MmvqParams& p, uint8_t* xsm, float* red, WarpPipe& w, const POp* prog,
                                       int nops) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    mmvq_build_x<NC, PRO>(p, xsm, red);
    __syncthreads();
    const int KC = p.n_in >> 10, ng = p.n_in >> 5;
    const int units = p.n_out >> 2;
    const int ubeg = (int) (((long long) blockIdx.x * units) / gridDim.x);
    const int uend = (int) (((long long) (blockIdx.x + 1) * units) / gridDim.x);
    unsigned long long best[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) best[c] = 0ull;
    bool ok = true;
    for (int unit = ubeg + warp; unit < uend && ok; unit += kMmvqWarps) {
        float acc[NC][4];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[c][r] = 0.0f;
        for (int kc = 0; kc < KC; ++kc) {
            if (!pipe_wait(w)) {
                ok = false;
                break;
            }
            const uint8_t* t = w.ring + (size_t) w.cs * kQ6Tile;
            int4 xa[NC], xb[NC];
            float4 xm[NC];
            const int g = (kc << 5) + lane;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const XStage xs = xstage_col(xsm, ng, c);
                xa[c] = xs.lo[g];
                xb[c] = xs.hi[g];
                xm[c] = xs.meta[g];
            }
            q6_tile<NC>(t, lane, xa, xb, xm, acc);
            pipe_release(w, prog, nops, warp, lane);
        }
        if (ok) mmvq_epilogue<NC, EPI>(p, unit, lane, acc, best);
    }
    if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
        for (int c = 0; c < NC; ++c)
            if (lane == c && best[c] != 0ull) atomicMax(p.amax + c, best[c]);
    }
    return ok;
}

// The prologue / epilogue pairs the engine's programs use (checked when a program is built).
__host__ __device__ __forceinline__ bool gemv_combo_supported(int pro, int epi) {
    return (pro == PRO_RMS && (epi == EPI_STORE || epi == EPI_SWIGLU || epi == EPI_ARGMAX)) ||
           (pro == PRO_Q8 && (epi == EPI_RES || epi == EPI_STORE_P));
}

template <int NC>
__device__ __forceinline__ bool p_gemv_dispatch(const POp& op, uint8_t* xsm, float* red, WarpPipe& w, const POp* prog,
                                                int nops) {
    const MmvqParams& p = op.g;
    if (op.pro == PRO_RMS) {
        if (op.epi == EPI_STORE) return p_gemv<NC, PRO_RMS, EPI_STORE>(p, xsm, red, w, prog, nops);
        if (op.epi == EPI_SWIGLU) return p_gemv<NC, PRO_RMS, EPI_SWIGLU>(p, xsm, red, w, prog, nops);
        return p_gemv<NC, PRO_RMS, EPI_ARGMAX>(p, xsm, red, w, prog, nops);
    }
    if (op.epi == EPI_RES) return p_gemv<NC, PRO_Q8, EPI_RES>(p, xsm, red, w, prog, nops);
    return p_gemv<NC, PRO_Q8, EPI_STORE_P>(p, xsm, red, w, prog, nops);
}

// Shared memory of the persistent kernel: mbarriers | region (staged activations or op scratch) | rings.
inline size_t persistent_smem_bytes(int region_bytes, int stages) {
    return (size_t) kMmvqWarps * kMmvqMaxStages * 8 + (size_t) region_bytes + (size_t) kMmvqWarps * stages * kQ6Tile;
}

template <int NC>
__global__ void __launch_bounds__(256, 1)
    persistent_kernel(const POp* __restrict__ prog, int nops, Ctrl* ctrl, PSync* sync, int stages, int region_bytes,
                      int until, int max_iters) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[8];
    __shared__ int flag;
    __shared__ __align__(16) POp op_sm;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* region = smem + kMmvqWarps * kMmvqMaxStages * 8;
    WarpPipe w;
    w.bar0 = smem_u32(smem) + (uint32_t) (warp * kMmvqMaxStages * 8);
    w.ring = region + region_bytes + (size_t) warp * stages * kQ6Tile;
    w.ring0 = smem_u32(w.ring);
    w.stages = stages;
    w.cs = 0;
    w.cpar = 0u;
    w.ps = 0;
    w.inflight = 0;
    w.pj = -1;
    w.pu = w.puend = w.pkc = w.pKC = 0;
    w.pw = nullptr;
    w.pol = policy_evict_first();
    w.wrap = until > 0;
    if (lane == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(w.bar0 + 8u * (uint32_t) s, 1);
        fence_mbar_init();
    }
    __syncwarp();
    unsigned long long target = 0ull;
    bool alive = ld_volatile_u32(&sync->abort) == 0u;
    if (alive) {
        pipe_seek(w, prog, nops, 0, warp);
        for (int k = 0; k < stages; ++k) pipe_issue(w, prog, nops, warp, lane);
    }
    for (int iter = 1; alive; ++iter) {
        for (int j = 0; j < nops && alive; ++j) {
            {
                const int* src = reinterpret_cast<const int*>(prog + j);
                int* dst = reinterpret_cast<int*>(&op_sm);
                for (int i = threadIdx.x; i < (int) (sizeof(POp) / 4); i += blockDim.x) dst[i] = src[i];
            }
            __syncthreads();
            bool ok = true;
            if (op_sm.kind == POP_GEMV) {
                ok = p_gemv_dispatch<NC>(op_sm, region, red, w, prog, nops);
            } else {
                const int pos = ld_cg(op_sm.draft ? &ctrl->dpos : &ctrl->pos);
                const int rb = ld_cg(&ctrl->rollback);
                const int items = pop_items<NC>(op_sm, pos);
                for (int it = (int) blockIdx.x; it < items; it += (int) gridDim.x)
                    run_item<NC>(op_sm, ctrl, it, pos, rb, reinterpret_cast<float*>(region), red);
            }
            if (!ok && lane == 0) atomicExch(&sync->abort, 1u);
            if (j + 1 < nops || until > 0) alive = grid_sync(sync, target, &flag);
        }
        if (!alive || until <= 0 || iter >= max_iters) break;
        if (ld_cg(&ctrl->n_emitted) >= until) break;
    }
    pipe_drain(w);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&sync->exits, 1u) == gridDim.x - 1) {
            volatile PSync* v = sync;
            v->arrive = 0ull;
            v->exits = 0u;
            __threadfence();
        }
    }
}

// One non-GEMV op as its own launch (graph mode).
template <int NC>
__global__ void __launch_bounds__(256) op_kernel(const POp op, Ctrl* ctrl) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();
    const int pos = ld_cg(op.draft ? &ctrl->dpos : &ctrl->pos);
    const int rb = ld_cg(&ctrl->rollback);
    if ((int) blockIdx.x >= pop_items<NC>(op, pos)) return;
    run_item<NC>(op, ctrl, (int) blockIdx.x, pos, rb, reinterpret_cast<float*>(smem), red);
}

}  // namespace rk
