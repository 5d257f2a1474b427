// persistent.cuh — the two executors of a decode op program (decode_ops.cuh).
//
// * Graph executor: one launch per op, captured in a CUDA graph. GEMV ops launch mmvq_packed_kernel; the GDN
//   step, the flash-decode chunks and the attention combine have kernels of their own (gdn_kernel,
//   attn_kernel, combine_kernel: each compiled for its body alone, so its register count allows several
//   blocks per SM and its code stays small); the remaining small ops (embedding, draft input, control) run
//   in op_kernel<NC> (grid = the op's largest item count, blocks past the live item count return).
// * persistent_kernel<NC>: the whole program in one cooperative launch, one 512-thread CTA per SM. Ops
//   run in program order separated by grid barriers. All 16 warps consume GEMV tiles (16 warps per SM
//   hide the latency of the tile decode) against one staged copy of the activations; the 256-thread
//   GEMV prologue and the non-GEMV op bodies run on warps 0..7 (named barrier 1), whose items are dealt
//   to CTAs round-robin.
//   Weight streaming runs ahead of the op boundaries: each warp walks the program's sequence of GEMV
//   tiles (its units of every GEMV, in order, from a GEMV table in shared memory) with a cursor that
//   fills a private ring of `stages` 3360-B shared-memory slots by 1-D bulk copies (one mbarrier per
//   slot). A slot freed by the consumer is refilled at once, so at the end of one GEMV the ring already
//   holds the next GEMV's first tiles, and HBM keeps streaming through the op's tail, the grid barrier,
//   the next prologue and the non-GEMV ops in between. Further ahead, when an op starts each CTA asks L2
//   for the first `l2pf` bytes of its (contiguous) share of the next GEMV's weights with one bulk L2
//   prefetch, so that GEMV's ring refills find their tiles in L2. With `until` > 0 the program repeats while
//   ctrl->n_emitted < until, at most `max_iters` times (a whole generation in one launch), and the cursor
//   wraps around to the program's first GEMV.
//
// A GEMV's work split (contiguous unit ranges per CTA, units dealt to warps round-robin) and its per-row
// arithmetic are those of mmvq_packed_kernel, so both executors write the same bits.
//
// Tracing: with a non-null `trace`, CTA 0 records four globaltimer stamps per op of the first pass (op
// start, prologue done, its own work done, barrier passed) and every CTA its op start and work-done
// stamps; ncu sees a persistent launch only as a whole.
//
// Failure handling: every mbarrier wait and grid-barrier spin is bounded. A CTA that gives up sets the
// sticky `abort` word and a status bit; every CTA then skips the rest of the program, waits (bounded)
// for its own bulk copies still in flight and exits. The last CTA to exit resets the barrier counter,
// so each launch starts from zero.
#pragma once

#include "decode_ops.cuh"

namespace rk {

// One GEMV of a program, as the weight cursors see it (built by the host in program order).
struct GemvEnt {
    const uint8_t* w;  // packed tiles
    int units;         // n_out / 4
    int KC;            // n_in / 1024: tiles per unit
};
static_assert(sizeof(GemvEnt) == 16, "GemvEnt is copied in 16-byte chunks");
constexpr int kMaxGemvOps = 256;
constexpr int kPWarps = 16;  // warps of a persistent CTA; all consume GEMV tiles

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Grid barrier: the counter starts at 0 in every launch and every barrier adds gridDim.x arrivals. A CTA
// that failed (any thread's `failed`) arrives with kAbortArrive more, so every waiter of this barrier and
// of all later ones sees the failure in the same load that ends its wait; the sticky abort word (set by the
// failing CTA for the host) is polled only every 64 spins, for a CTA that gave up without arriving.
// Returns false when the program must stop (a failed arrival, abort seen, or this spin gave up).
constexpr unsigned long long kAbortArrive = 1ull << 40;
__device__ __forceinline__ bool grid_sync(PSync* sync, unsigned long long& target, int* flag, bool failed) {
    const int any_failed = __syncthreads_or(failed ? 1 : 0);
    target += gridDim.x;
    if (threadIdx.x == 0) {
        // release: this CTA's writes (ordered before by the bar.red above) become visible with the arrival
        const unsigned long long add = any_failed ? kAbortArrive + 1ull : 1ull;
        asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(&sync->arrive), "l"(add) : "memory");
        int good = 1;
        unsigned long long t0 = 0, v = 0;
        for (uint32_t it = 0;; ++it) {
            v = ld_acquire_u64(&sync->arrive);
            if (v >= target) break;
            if ((it & 63u) == 0u) {
                const unsigned long long now = globaltimer_ns();
                if (it == 0u) {
                    t0 = now;
                } else if (ld_volatile_u32(&sync->abort) || now - t0 > kGridSpinNs) {
                    if (!ld_volatile_u32(&sync->abort)) atomicOr(&g_rk_status, kStatusGridTimeout);
                    atomicExch(&sync->abort, 1u);
                    good = 0;
                    break;
                }
            }
            if (it >= 256u) __nanosleep(32);
        }
        if (v >= kAbortArrive) good = 0;
        *flag = good;
    }
    // the acquire above and this bar.sync order the whole CTA's later reads after every arrival
    __syncthreads();
    return *flag != 0;
}

// ---------------------------------------------------------------------------------------------------
// Weight cursors: position in a warp's tile sequence (GEMV table index gi, -1 when none is left; unit u
// of the CTA's range [.., uend); k-chunk kc).
// ---------------------------------------------------------------------------------------------------
struct Cursor {
    int gi, u, uend, kc;
};

__device__ __forceinline__ void cur_seek(Cursor& c, const GemvEnt* gt, int ng, int from, int warp, bool wrap) {
    for (int n = 0; n < ng; ++n) {
        int i = from + n;
        if (i >= ng) {
            if (!wrap) break;
            i -= ng;
        }
        const int units = gt[i].units;
        const int ubeg = (int) (((long long) blockIdx.x * units) / gridDim.x);
        const int uend = (int) (((long long) (blockIdx.x + 1) * units) / gridDim.x);
        if (ubeg + warp < uend) {
            c.gi = i;
            c.u = ubeg + warp;
            c.uend = uend;
            c.kc = 0;
            return;
        }
    }
    c.gi = -1;
}
__device__ __forceinline__ void cur_next(Cursor& c, const GemvEnt* gt, int ng, int warp, bool wrap) {
    if (++c.kc == gt[c.gi].KC) {
        c.kc = 0;
        c.u += kPWarps;
        if (c.u >= c.uend) cur_seek(c, gt, ng, c.gi + 1, warp, wrap);
    }
}
__device__ __forceinline__ const uint8_t* cur_src(const Cursor& c, const GemvEnt* gt) {
    return gt[c.gi].w + ((size_t) c.u * gt[c.gi].KC + c.kc) * kQ6Tile;
}

// Per-warp ring state, the same in every lane (lane 0 issues the copies).
struct WarpPipe {
    uint32_t bar0, ring0;  // shared-memory addresses of the warp's first mbarrier and first slot
    const uint8_t* ring;
    int stages;
    int cs;         // consumer slot
    uint32_t cpar;  // consumer phase parity
    int ps;         // producer slot
    int inflight;   // tiles issued and not yet consumed
    uint64_t pol;
    bool wrap;
    Cursor pc;  // ring cursor
    const GemvEnt* gt;
    int ng;
};

// The cursor's next tile into the free slot.
__device__ __forceinline__ void pipe_issue(WarpPipe& w, int warp, int lane) {
    if (w.pc.gi < 0) return;
    if (lane == 0) {
        const uint32_t bar = w.bar0 + 8u * (uint32_t) w.ps;
        mbar_arrive_expect_tx(bar, kQ6Tile);
        bulk_g2s(w.ring0 + (uint32_t) (w.ps * kQ6Tile), cur_src(w.pc, w.gt), kQ6Tile, bar, w.pol);
    }
    if (++w.ps == w.stages) w.ps = 0;
    ++w.inflight;
    cur_next(w.pc, w.gt, w.ng, warp, w.wrap);
}

// Place the cursor at the start and fill the ring.
__device__ __forceinline__ void pipe_start(WarpPipe& w, int warp, int lane) {
    cur_seek(w.pc, w.gt, w.ng, 0, warp, w.wrap);
    for (int k = 0; k < w.stages; ++k) pipe_issue(w, warp, lane);
}

// Wait (bounded) for the tile `ahead` slots past the consumer's.
__device__ __forceinline__ bool pipe_wait(const WarpPipe& w, int ahead) {
    int s = w.cs + ahead;
    uint32_t par = w.cpar;
    if (s >= w.stages) {
        s -= w.stages;
        par ^= 1u;
    }
    const bool landed = mbar_wait_bounded(w.bar0 + 8u * (uint32_t) s, par);
    return __all_sync(0xffffffffu, landed);
}
__device__ __forceinline__ const uint8_t* pipe_tile(const WarpPipe& w, int ahead) {
    int s = w.cs + ahead;
    if (s >= w.stages) s -= w.stages;
    return w.ring + (size_t) s * kQ6Tile;
}

// The warp is done reading the current slot: hand it back to the async proxy and refill it.
__device__ __forceinline__ void pipe_release(WarpPipe& w, int warp, int lane) {
    __syncwarp();
    if (lane == 0) fence_proxy_async_smem();
    --w.inflight;
    if (++w.cs == w.stages) {
        w.cs = 0;
        w.cpar ^= 1u;
    }
    pipe_issue(w, warp, lane);
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
// An L2 prefetch request (the next GEMV's share of this CTA; bytes 0: none).
struct L2Pf {
    const void* ptr;
    uint32_t bytes;
};

template <int NC, int PRO, int EPI>
__device__ __forceinline__ bool p_gemv(const MmvqParams& p, uint8_t* xsm, float* red, WarpPipe& w,
                                       unsigned long long* tp, unsigned long long& xep, PSync* sync,
                                       const L2Pf& pf) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // EPI_XRES: this exchange's epoch and this rank's partial buffer (by epoch parity)
    unsigned long long ep = 0ull;
    size_t yoff = 0;  // this rank's slot in every rank's partial buffer for this exchange
    if constexpr (EPI == EPI_XRES) {
        ep = ++xep;
        yoff = xres_offset(p.xch, ep);
    }
    mmvq_build_x<NC, PRO>(p, xsm, red);
    __syncthreads();
    if (tp != nullptr && threadIdx.x == 0) *tp = globaltimer_ns();
    // the next GEMV's L2 prefetch goes out only now, behind this prologue's loads
    if (threadIdx.x == 256 && pf.bytes > 0) prefetch_l2(pf.ptr, pf.bytes);
    const int KC = p.n_in >> 10, ng = p.n_in >> 5;
    const int units = p.n_out >> 2;
    const int ubeg = (int) (((long long) blockIdx.x * units) / gridDim.x);
    const int uend = (int) (((long long) (blockIdx.x + 1) * units) / gridDim.x);
    unsigned long long best[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) best[c] = 0ull;
    bool ok = true;
    int unit = ubeg + warp;
    for (; unit < uend; unit += kPWarps) {
        float acc[NC][4];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[c][r] = 0.0f;
        float resv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mmvq_res_prefetch<NC, EPI>(p, unit, lane, resv);
        float lo[NC][4];  // the first half's chains (an even chunk count runs two chains, mmvq_packed_kernel)
        const int split = mmvq_split(KC);
        for (int kc = 0; kc < KC; ++kc) {
            if (kc == split) mmvq_stash_half<NC>(acc, lo);
            if (!pipe_wait(w, 0)) {
                ok = false;
                break;
            }
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
            q6_tile<NC>(pipe_tile(w, 0), lane, xa, xb, xm, acc);
            pipe_release(w, warp, lane);
        }
        if (!ok) break;
        if (split < KC) mmvq_join_halves<NC>(acc, lo);
        if constexpr (EPI == EPI_XRES) {  // this rank's partial rows, pushed to every rank
            xres_push<NC>(p.xch, yoff, ep, unit, lane, acc);
        } else {
            mmvq_epilogue<NC, EPI>(p, unit, lane, acc, best, resv);
        }
    }
    if constexpr (EPI == EPI_XRES) return xres_finish<NC>(p, ubeg, uend, ep, sync) && ok;
    if constexpr (EPI == EPI_SWIGLU) mmvq_swiglu_finish<NC>(p, ubeg + warp, kPWarps, unit, lane);
    if constexpr (EPI == EPI_ARGMAX) mmvq_argmax_flush<NC>(p, lane, best);
    return ok;
}

// The prologue / epilogue pairs the engine's programs use (checked when a program is built).
__host__ __device__ __forceinline__ bool gemv_combo_supported(int pro, int epi) {
    return (pro == PRO_RMS && (epi == EPI_STORE || epi == EPI_SWIGLU || epi == EPI_ARGMAX)) ||
           (pro == PRO_Q8 && (epi == EPI_RES || epi == EPI_STORE_P || epi == EPI_XRES));
}

template <int NC>
__device__ __forceinline__ bool p_gemv_dispatch(const POp& op, uint8_t* xsm, float* red, WarpPipe& w,
                                                unsigned long long* tp, unsigned long long& xep, PSync* sync,
                                                const L2Pf& pf) {
    const MmvqParams& p = op.g;
    if (op.pro == PRO_RMS) {
        if (op.epi == EPI_STORE) return p_gemv<NC, PRO_RMS, EPI_STORE>(p, xsm, red, w, tp, xep, sync, pf);
        if (op.epi == EPI_SWIGLU) return p_gemv<NC, PRO_RMS, EPI_SWIGLU>(p, xsm, red, w, tp, xep, sync, pf);
        return p_gemv<NC, PRO_RMS, EPI_ARGMAX>(p, xsm, red, w, tp, xep, sync, pf);
    }
    if (op.epi == EPI_RES) return p_gemv<NC, PRO_Q8, EPI_RES>(p, xsm, red, w, tp, xep, sync, pf);
    if constexpr (NC <= 2)  // the exchange buffers hold two columns (tensor parallelism has no prefill program)
        if (op.epi == EPI_XRES) return p_gemv<NC, PRO_Q8, EPI_XRES>(p, xsm, red, w, tp, xep, sync, pf);
    return p_gemv<NC, PRO_Q8, EPI_STORE_P>(p, xsm, red, w, tp, xep, sync, pf);
}

// Asynchronous copy of op record j into shared memory (16-byte cp.async chunks, one per thread), so the
// next op's record arrives while the current op runs.
__device__ __forceinline__ void op_fetch(const POp* prog, int j, POp* dst) {
    constexpr int kChunks = (int) (sizeof(POp) / 16);
    if ((int) threadIdx.x < kChunks) {
        const uint32_t d = smem_u32(dst) + 16u * threadIdx.x;
        const char* src = reinterpret_cast<const char*>(prog + j) + 16 * threadIdx.x;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared memory of the persistent kernel: mbarriers | region (staged activations or op scratch) | rings.
inline size_t persistent_smem_bytes(int region_bytes, int stages) {
    return (size_t) kPWarps * kMmvqMaxStages * 8 + (size_t) region_bytes + (size_t) kPWarps * stages * kQ6Tile;
}

template <int NC>
__global__ void __launch_bounds__(kPWarps * 32, 1)
    persistent_kernel(const POp* __restrict__ prog, int nops, const GemvEnt* __restrict__ gtab, int ngemv, Ctrl* ctrl,
                      PSync* sync, int stages, int region_bytes, int l2pf, int until, int max_iters,
                      unsigned long long* trace) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[kRedCols * 8];
    __shared__ int flag;
    __shared__ POp op_sm[2];  // the running op's record and the next one's (fetched while the op runs)
    __shared__ GemvEnt gt_sm[kMaxGemvOps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* region = smem + kPWarps * kMmvqMaxStages * 8;
    // the GEMV table and the first op record
    for (int i = (int) threadIdx.x; i < ngemv; i += (int) blockDim.x) {
        const uint32_t d = smem_u32(&gt_sm[i]);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gtab + i) : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    op_fetch(prog, 0, &op_sm[0]);
    WarpPipe w;
    w.bar0 = smem_u32(smem) + (uint32_t) (warp * kMmvqMaxStages * 8);
    w.ring = region + region_bytes + (size_t) warp * stages * kQ6Tile;
    w.ring0 = smem_u32(w.ring);
    w.stages = stages;
    w.cs = 0;
    w.cpar = 0u;
    w.ps = 0;
    w.inflight = 0;
    w.pol = policy_evict_first();
    w.wrap = until > 0;
    w.pc.gi = -1;
    w.gt = gt_sm;
    w.ng = ngemv;
    if (lane == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(w.bar0 + 8u * (uint32_t) s, 1);
        fence_mbar_init();
    }
    cp_async_wait_all();
    __syncthreads();
    unsigned long long target = 0ull;
    unsigned long long xep = *reinterpret_cast<volatile unsigned long long*>(&sync->xepoch);
    bool alive = ld_volatile_u32(&sync->abort) == 0u;
    if (alive) pipe_start(w, warp, lane);
    int k = 0;  // ops started; op_sm[k & 1] holds the running op
    for (int iter = 1; alive; ++iter) {
        for (int j = 0; j < nops && alive; ++j, ++k) {
            const POp& op = op_sm[k & 1];
            const int next = j + 1 < nops ? j + 1 : (until > 0 ? 0 : -1);
            if (next >= 0) op_fetch(prog, next, &op_sm[(k + 1) & 1]);
            // this CTA's share of the next GEMV into L2 (thread 256; a GEMV issues it after its prologue)
            L2Pf pf = {nullptr, 0u};
            if (threadIdx.x == 256 && l2pf > 0 && op.next_gemv >= 0) {
                const GemvEnt& e = gt_sm[op.next_gemv];
                const int ubeg = (int) (((long long) blockIdx.x * e.units) / gridDim.x);
                const int uend = (int) (((long long) (blockIdx.x + 1) * e.units) / gridDim.x);
                const size_t bytes = (size_t) (uend - ubeg) * e.KC * kQ6Tile;
                pf.ptr = e.w + (size_t) ubeg * e.KC * kQ6Tile;
                pf.bytes = (uint32_t) (bytes < (size_t) l2pf ? bytes : (size_t) l2pf);
                if (op.kind != POP_GEMV && pf.bytes > 0) prefetch_l2(pf.ptr, pf.bytes);
            }
            // op trace (CTA 0, first pass): start, prologue done, this CTA's work done, barrier passed;
            // per CTA (first pass): start, work done
            unsigned long long* tr = trace != nullptr && blockIdx.x == 0 && iter == 1 ? trace + 4 * j : nullptr;
            unsigned long long* tc =
                trace != nullptr && iter == 1 ? trace + 4 * (size_t) nops + ((size_t) j * gridDim.x + blockIdx.x) * 2 : nullptr;
            if (threadIdx.x == 0) {
                if (tr != nullptr) tr[0] = tr[1] = globaltimer_ns();
                if (tc != nullptr) tc[0] = globaltimer_ns();
            }
            bool ok = true;
            if (op.kind == POP_GEMV) {
                ok = p_gemv_dispatch<NC>(op, region, red, w, tr != nullptr ? tr + 1 : nullptr, xep, sync, pf);
            } else if (op.kind == POP_XARGMAX) {
                const unsigned long long ep = ++xep;
                if constexpr (NC <= 2)
                    if (blockIdx.x == 0 && threadIdx.x == 0)
                        ok = xch_argmax<NC>(op.xa.xch, op.draft ? ctrl->damax : ctrl->amax, ep, sync);
            } else {
                const int pos = ld_cg(op.draft ? &ctrl->dpos : &ctrl->pos);
                const int rb = ld_cg(&ctrl->rollback);
                const int items = pop_items<NC>(op, pos);
                if (warp < 8)
                    for (int it = (int) blockIdx.x; it < items; it += (int) gridDim.x)
                        run_item<NC>(op, ctrl, it, pos, rb, reinterpret_cast<float*>(region), red);
            }
            if (!ok && lane == 0) atomicExch(&sync->abort, 1u);  // for the host; the barrier carries it too
            if (tc != nullptr) {
                __syncthreads();
                if (threadIdx.x == 0) {
                    const unsigned long long t = globaltimer_ns();
                    tc[1] = t;
                    if (tr != nullptr) tr[2] = t;
                }
            }
            cp_async_wait_all();  // the next record has landed (made visible by the barrier's bar.sync)
            if (j + 1 < nops || until > 0) alive = grid_sync(sync, target, &flag, !ok);
            else if (!ok) alive = false;
            if (tr != nullptr && threadIdx.x == 0) tr[3] = globaltimer_ns();
        }
        if (!alive || until <= 0 || iter >= max_iters) break;
        if (ld_cg(&ctrl->n_emitted) >= until || ld_cg(&ctrl->stop)) break;
    }
    pipe_drain(w);
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<volatile unsigned long long*>(&sync->xepoch) = xep;
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

// The flash-decode chunk items of an attention op as their own launch (graph mode). op_kernel's register
// allocation covers every op body and leaves one CTA per SM; the chunk body alone keeps kAttnCtas CTAs per
// SM resident, which the long-context chunk loop (memory latency bound) needs.
template <int NC>
constexpr int kAttnCtas = NC == 1 ? 3 : NC == 2 ? 2 : 1;  // 80 / 127 / 255 registers, no spills
template <int NC, int G = kGqa>
__global__ void __launch_bounds__(256, kAttnCtas<NC>) attn_kernel(const POp op, Ctrl* ctrl) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    if (threadIdx.x == 0) {
        // The K rows of this block's first chunk (all but the new positions written long before) head for
        // L2 while the projection GEMV upstream still runs; the position as it reads now is only a hint
        // for this prefetch, bounds-checked like the body's.
        const int ph = ld_cg(op.draft ? &ctrl->dpos : &ctrl->pos);
        const AttnArgs& a = op.at;
        if (ph >= 0 && ph + NC <= a.max_ctx && (int) blockIdx.x < pop_items<NC>(op, ph)) {
            const int chunk = (int) blockIdx.x / a.n_kv, kvh = (int) blockIdx.x % a.n_kv;
            const int t0 = chunk * a.chunk_len;
            const int tend = min(t0 + a.chunk_len, ph + NC);
            if (chunk < a.max_chunks && t0 < tend) {
                const uint32_t bytes = (uint32_t) (tend - t0) * kHdA * 2;
                const size_t row0 = ((size_t) kvh * a.max_ctx + t0) * kHdA;
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.kc + row0), "r"(bytes) : "memory");
            }
        }
    }
    pdl_wait();
    const int pos = ld_cg(op.draft ? &ctrl->dpos : &ctrl->pos);
    const int items = pop_items<NC>(op, pos);
    for (int it = (int) blockIdx.x; it < items; it += (int) gridDim.x)  // uniform over the block
        attn_chunk_impl<NC, G>(op.at, pos, it / op.at.n_kv, it % op.at.n_kv, reinterpret_cast<float*>(smem));
}

// The GDN op as its own launch (graph mode): a kernel of its own instead of the generic op kernel, whose
// code covers every op body (instruction-cache misses) and whose register allocation is the largest body's.
template <int NC>
__global__ void __launch_bounds__(256) gdn_kernel(const POp op, Ctrl* ctrl) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    // The state slice this block steps was written by the same layer's GDN op one step earlier, long
    // complete; its lines are asked of L2 now, while the projection GEMV upstream still runs (from the
    // snapshot when the rollback flag, as it reads now, says so). A prefetch only warms L2: the loads
    // after the wait read the current values from wherever the flag then points.
    if (threadIdx.x < 128 && (int) blockIdx.x < op.gd.hv * 4) {
        const int head = (int) blockIdx.x >> 2, quarter = (int) blockIdx.x & 3;
        const size_t off = ((size_t) ((threadIdx.x >> 5) * 32) * op.gd.hv + head) * kSsm + quarter * 32 + (threadIdx.x & 31);
        const size_t rs = (size_t) op.gd.hv * kSsm;
        const float* src = (ld_cg(&ctrl->rollback) != 0 ? op.gd.snap : op.gd.state) + off;
#pragma unroll 8
        for (int r = 0; r < 32; ++r) asm volatile("prefetch.global.L2 [%0];" ::"l"(src + r * rs));
    }
    pdl_wait();
    const int pos = ld_cg(op.draft ? &ctrl->dpos : &ctrl->pos);
    const int rb = ld_cg(&ctrl->rollback);
    const int items = pop_items<NC>(op, pos);
    for (int it = (int) blockIdx.x; it < items; it += (int) gridDim.x)  // uniform over the block
        gdn_quarter_impl<NC>(op.gd, it >> 2, it & 3, pos, rb != 0, reinterpret_cast<float*>(smem));
}

// The attention combine as its own launch (graph mode): n_head x NC x 8 items of 32 dims, small enough per
// block that they run in one wave (the generic op kernel's registers leave one block per SM).
template <int NC>
__global__ void __launch_bounds__(256, 2) combine_kernel(const POp op, Ctrl* ctrl) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    pdl_wait();
    const int pos = ld_cg(op.draft ? &ctrl->dpos : &ctrl->pos);
    const int items = pop_items<NC>(op, pos);
    for (int it = (int) blockIdx.x; it < items; it += (int) gridDim.x)  // uniform over the block
        combine_impl<NC>(op.at, pos, it / (NC * 8), (it / 8) % NC, it % 8, reinterpret_cast<float*>(smem));
}

// Tensor parallelism, graph mode: the global argmax after an lm_head over this rank's vocabulary shard
// (one thread; the keys exchange of xch_argmax on the argmax flag slot, whose epoch counter it advances).
template <int NC>
__global__ void __launch_bounds__(32) xargmax_kernel(const POp op, Ctrl* ctrl) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    const XchDesc* x = op.xa.xch;
    const int slot = x->slots - 1;
    const unsigned long long ep = xch_epoch_next(x, slot);
    if (!xch_argmax<NC>(x, op.draft ? ctrl->damax : ctrl->amax, ep, x->sync)) atomicExch(&x->sync->abort, 1u);
    xch_epoch_done(x, slot, ep);
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
    const int items = pop_items<NC>(op, pos);
    for (int it = (int) blockIdx.x; it < items; it += (int) gridDim.x)  // uniform over the block
        run_item<NC>(op, ctrl, it, pos, rb, reinterpret_cast<float*>(smem), red);
}

}  // namespace rk
