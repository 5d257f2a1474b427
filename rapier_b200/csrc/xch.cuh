// xch.cuh — the tensor-parallel exchange over NVLink peer memory, shared by both decode executors: the
// persistent kernel (persistent.cuh) and the one-kernel-per-op graph executor (mmvq_packed_kernel's
// EPI_XRES epilogue, xargmax_kernel).
//
// Every rank's exchange memory is mapped into this rank's address space (CUDA IPC over NVLink).
//
// Row-parallel partial sums travel as self-validating 8-byte words, (exchange epoch << 32) | fp32 bits: a
// CTA stores each of its rows' partials into its own source slot of every rank's buffer with one 64-bit
// store, and the same CTA of every rank (same grid, same split: the same rows) polls the words of its rows
// in its own memory until each carries the exchange's epoch. A 64-bit store is seen whole, so a word with
// the right epoch holds that exchange's value: no fence and no separate flag. Epochs only grow (a resync
// clears them together with the buffers), and the buffers alternate by epoch parity: a rank writes epoch
// e + 2 into a slot only after it has read the peers' epoch e + 1 words of the same rows, which the peers'
// same CTA wrote after it had read epoch e, so no word is overwritten before it is read.
//
// The argmax exchange (one per lm_head) keeps a flag protocol: each rank writes its keys into every rank's
// key array, fences at system scope and release-stores the epoch into every peer's flag slot, then acquires
// all the peers' flags before it reads the keys.
//
// Epochs: the persistent kernel counts all of a launch's exchanges in one register (carried between
// launches in PSync::xepoch); the graph executor keeps one counter per slot (a GEMV CTA index, or the
// argmax) in this rank's own exchange memory (`ep`), which the CTA owning the slot reads at its start and
// writes back at its end. Either way the same slot of every rank sees the same epoch sequence.
#pragma once

#include "common.cuh"

namespace rk {

struct PSync {
    unsigned long long arrive;  // grid-barrier arrivals of the running launch
    unsigned exits;             // CTAs of the running launch that have finished
    unsigned abort;             // sticky give-up flag, cleared by the host
    unsigned long long xepoch;  // tensor parallelism: exchanges done so far (monotonic, never cleared)
};

constexpr int kMaxRanks = 8;
struct XchDesc {
    int rank, n;  // this rank, number of ranks
    int rows;     // rows of a partial column (the hidden size)
    int slots;    // epoch slots: one per GEMV CTA (its rows' exchanges) + one for the argmax exchange
    unsigned long long wait_ns;            // a cross-rank wait gives up after this long
    unsigned long long* buf[kMaxRanks];    // per rank: partial words [2 parity][kMaxRanks source][2 columns][rows]
    unsigned long long* flags[kMaxRanks];  // per rank: [slots][kMaxRanks] epochs, written by the peers
    unsigned long long* keys[kMaxRanks];   // per rank: argmax keys [2 parity][kMaxRanks][2 columns]
    unsigned long long* ep;                // graph executor: this rank's epoch counter per flag slot
    PSync* sync;                           // this rank's sticky abort word (both executors)
};

constexpr unsigned long long kGridSpinNs = 1000000000ull;  // a grid barrier gives up after 1 s
constexpr unsigned long long kPeerSpinNs = 5000000000ull;  // default cross-rank wait bound (a peer's host may lag)

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
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    return *reinterpret_cast<const volatile unsigned long long*>(p);
}
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
    *reinterpret_cast<volatile unsigned long long*>(p) = v;
}
__device__ __forceinline__ unsigned long long xch_word(unsigned long long epoch, float v) {
    return ((unsigned long long) (uint32_t) epoch << 32) | (unsigned long long) __float_as_uint(v);
}

// One partial word: waits until the word at `p` carries epoch `epoch` and returns its value in `v`. The wait
// gives up after x->wait_ns (status bit, abort), or at once once the abort word is set.
__device__ __forceinline__ bool xch_poll(const unsigned long long* p, unsigned long long epoch, const XchDesc* x,
                                         PSync* sync, float& v) {
    const uint32_t e32 = (uint32_t) epoch;
    unsigned long long w = ld_volatile_u64(p);
    if ((uint32_t) (w >> 32) != e32) {
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t it = 1;; ++it) {
            if (it >= 64u) __nanosleep(32);
            w = ld_volatile_u64(p);
            if ((uint32_t) (w >> 32) == e32) break;
            if ((it & 63u) == 0u) {
                if (ld_volatile_u32(&sync->abort)) return false;
                if (globaltimer_ns() - t0 > x->wait_ns) {
                    atomicOr(&g_rk_status, kStatusGridTimeout);
                    atomicExch(&sync->abort, 1u);
                    return false;
                }
            }
        }
    }
    v = __uint_as_float((uint32_t) w);
    return true;
}

// One thread: signal flag slot `slot` of every peer with `epoch` (after a system-scope fence that makes
// this CTA's preceding writes visible), then wait until every peer has signalled this rank's slot. The
// wait gives up after x->wait_ns (status bit, abort), or at once once the abort word is set. Returns false
// when the step must stop.
static __device__ __noinline__ bool xch_signal_wait(const XchDesc* x, int slot, unsigned long long epoch, PSync* sync) {
    const int me = x->rank, n = x->n;
    __threadfence_system();
    for (int q = 0; q < n; ++q)
        if (q != me) st_release_sys_u64(x->flags[q] + (size_t) slot * kMaxRanks + me, epoch);
    const unsigned long long* mine = x->flags[me] + (size_t) slot * kMaxRanks;
    const unsigned long long t0 = globaltimer_ns();
    for (int q = 0; q < n; ++q) {
        if (q == me) continue;
        for (uint32_t it = 0; ld_acquire_sys_u64(mine + q) < epoch; ++it) {
            if (ld_volatile_u32(&sync->abort)) return false;
            if ((it & 63u) == 63u && globaltimer_ns() - t0 > x->wait_ns) {
                atomicOr(&g_rk_status, kStatusGridTimeout);
                atomicExch(&sync->abort, 1u);
                return false;
            }
            if (it >= 256u) __nanosleep(32);
        }
    }
    return true;
}

// The global argmax of the ranks' vocabulary shards (one thread): every rank's per-column keys
// (value, ~global row) go to every rank, and the maximum replaces this rank's slot, so all ranks continue
// with the same token.
template <int NC>
__device__ __noinline__ bool xch_argmax(const XchDesc* x, unsigned long long* slots, unsigned long long epoch,
                                        PSync* sync) {
    const int me = x->rank, n = x->n, par = (int) (epoch & 1ull);
    volatile unsigned long long* vs = slots;
    unsigned long long mine[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) mine[c] = vs[c];
    for (int q = 0; q < n; ++q)
#pragma unroll
        for (int c = 0; c < NC; ++c) x->keys[q][((size_t) par * kMaxRanks + me) * 2 + c] = mine[c];
    if (!xch_signal_wait(x, x->slots - 1, epoch, sync)) return false;
    const volatile unsigned long long* k = x->keys[me] + (size_t) par * kMaxRanks * 2;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        unsigned long long best = 0ull;
        for (int q = 0; q < n; ++q) best = k[q * 2 + c] > best ? k[q * 2 + c] : best;
        vs[c] = best;
    }
    __threadfence();
    return true;
}

// The graph executor's epoch for flag slot `slot` (the counter is written back by xch_epoch_done).
__device__ __forceinline__ unsigned long long xch_epoch_next(const XchDesc* x, int slot) {
    return *reinterpret_cast<const volatile unsigned long long*>(x->ep + slot) + 1ull;
}
__device__ __forceinline__ void xch_epoch_done(const XchDesc* x, int slot, unsigned long long ep) {
    *reinterpret_cast<volatile unsigned long long*>(x->ep + slot) = ep;
}

}  // namespace rk
