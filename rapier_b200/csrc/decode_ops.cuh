// decode_ops.cuh — the decode engine's op program format and its per-op device bodies.
//
// An engine step (one token, one MTP verify round, one draft) is a program: a list of POp records
// (GEMV, embedding, GDN layer, attention chunks, attention combine, draft input, control). Each body
// below does one work item of its op with the whole 256-thread block. The same bodies run either as one
// kernel per op inside a CUDA graph (op_kernel) or back to back inside one persistent kernel per step
// (persistent.cuh), so both execution modes compute the same bits.
//
// Data written earlier in the same step is read with ld.global.cg (L2, not L1): inside the persistent
// kernel another SM may have rewritten a line this SM still holds in L1.
#pragma once

#include "mmvq.cuh"

namespace rk {

constexpr int kHdA = 256;     // attention head dim
constexpr int kSubA = 256;    // tokens scored per pass inside a flash-decode chunk (shared-memory scores)
constexpr int kMaxChunksA = 512;  // flash-decode chunks per kv head the chunk length aims for (see attn_chunk_len)
constexpr int kGqa = 4;       // query heads per kv head
constexpr int kDraftParts = 16;  // work items per column of the draft-input op
constexpr int kSsm = 128;     // GDN head size
constexpr float kInvSqrtSsm = 0.08838834764831845f;  // 1/sqrt(128)
constexpr int kRingSlots = 8;  // conv history per channel: the input at position p sits in slot p & 7

// ------------------------------------------------------------------------------------------------
// Device control block of the engine.
// ------------------------------------------------------------------------------------------------
struct Ctrl {
    int pos;       // trunk position of column 0
    int tok[4];    // trunk input tokens (tok[1] = the draft candidate in a verify round; 4 in a prefill pass)
    int dpos;      // draft position of column 0
    int dtok[2];   // draft input tokens
    int rollback;  // GDN state from the snapshot (the previous verify's draft was rejected)
    int accept;    // the last round accepted its draft
    int n_emitted;
    int steps, accepted, singles;
    int bad;       // a token id outside the vocabulary reached a kernel
    int eos1;      // end-of-sequence token id + 1 (0: none); emitting it stops the generation
    int stop;      // the generation emitted eos1 - 1 (the persistent loop ends after the pass)
    int pad;
    unsigned long long amax[2];   // trunk argmax keys per column
    unsigned long long damax[2];  // draft argmax keys per column
};
constexpr int kCtrlHostFields = 10;  // pos, tok[4], dpos, dtok[2], rollback, accept: written by the host
constexpr int kMaxCols = 4;          // columns of a step program: 1 (decode), 2 (verify), 4 (prefill)

__device__ __forceinline__ int ld_cg(const int* p) { return __ldcg(p); }
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

// ------------------------------------------------------------------------------------------------
// Op records
// ------------------------------------------------------------------------------------------------
enum : int { POP_GEMV = 1, POP_EMBED, POP_GDN, POP_ATTN, POP_COMBINE, POP_DRAFT_PREP, POP_CTRL, POP_XARGMAX };
enum : int { CTRL_SINGLE = 1, CTRL_ACCEPT, CTRL_ROUND, CTRL_DRAFT1 };

struct EmbedArgs {
    const uint8_t* emb;  // GGUF Q6_K rows
    int H, V;
    float* x;
    float* xp;
};
struct GdnArgs {
    const float* proj;  // [c][proj_stride]: q | k | v | z | beta | alpha
    int proj_stride;
    float* ring;  // [C][8]
    const float *conv_w, *dt, *ssm_a, *gamma;
    float *state, *snap;
    float* o_scr;   // [2][hv][128] read-outs before the norm
    float* ss_scr;  // [2][hv][4] per-quarter sums of squares
    unsigned* cnt;  // [hv] last-arriver counters (left zeroed)
    float* y;       // optional fp32 output [c][hv*128]
    uint8_t* q8;
    int hk, hv;
    float eps;
};
struct AttnArgs {
    const float* proj;  // [c][proj_stride]: n_head x (q 256 | gate 256), k n_kv x 256, v n_kv x 256
    int proj_stride;
    const float *qn, *kn, *rope;
    int n_rot, n_head, n_kv, max_ctx, max_chunks;
    int chunk_len;  // tokens per flash-decode chunk (attn_chunk_len of max_ctx)
    float eps, scale;
    __half *kc, *vc;
    float *part_o, *part_ml;
    float* o;      // optional fp32 attention output (combine)
    uint8_t* q8;   // Q8_1 of o * sigmoid(gate) (combine)
};
struct DraftPrepArgs {
    const uint8_t* emb;
    int H, V;
    const float *enorm, *hnorm, *hsave, *hsave_p;
    float eps;
    uint8_t* eh_q8;
};
struct CtrlArgs {
    int kind;
    int* out;
    int max_out;
    const int* force;  // forced draft candidate per position (-1: the draft's own argmax); a test hook
    int n_force;
};
struct XArgmaxArgs {  // tensor parallelism: the global argmax over the ranks' vocabulary shards
    const XchDesc* xch;
};
struct alignas(16) POp {  // 16-byte multiple: fetched into shared memory by 16-byte cp.async chunks
    int kind;
    int pro, epi;  // POP_GEMV: prologue / epilogue
    int draft;     // reads the draft position / tokens (ctrl->dpos, ctrl->dtok)
    int next_gemv; // persistent executor: GEMV-table index of the first GEMV after this op (-1: none)
    int pad_[3];
    union {
        MmvqParams g;
        EmbedArgs em;
        GdnArgs gd;
        AttnArgs at;
        DraftPrepArgs dp;
        CtrlArgs ct;
        XArgmaxArgs xa;
    };
};
static_assert(sizeof(POp) % 16 == 0 && sizeof(POp) / 16 <= 256, "op records are copied in 16-byte chunks");

// Tokens per flash-decode chunk of an engine with cache capacity max_ctx: the smallest of 32, 64, 128, 256
// (kSubA) that splits the whole cache into at most kMaxChunksA chunks (256 beyond 131072 positions), so a
// chunk is one pass of at most kSubA tokens and short contexts spread over many CTAs (17 chunks of 32 at
// 512 tokens when max_ctx <= 16384). The length depends on the engine only, never on the position or the
// column count: column c of a multi-column step is chunked exactly as a single-token step at position
// pos + c, which keeps the MTP verify bitwise equal to single-token decoding at every position.
__host__ __device__ __forceinline__ int attn_chunk_len(int max_ctx) {
    int len = 32;
    while ((max_ctx + len - 1) / len > kMaxChunksA && len < kSubA) len <<= 1;
    return len;
}

// Work items of a non-GEMV op at position pos (column 0). Blocks or persistent CTAs take items
// i = first, first + stride, ...
template <int NC>
__host__ __device__ __forceinline__ int pop_items(const POp& op, int pos) {
    switch (op.kind) {
        case POP_EMBED: return NC;
        case POP_GDN: return op.gd.hv * 4;
        case POP_ATTN: {  // positions outside the cache are refused by the body; bound the count
            const int p = pos < 0 ? 0 : (pos > op.at.max_ctx - NC ? op.at.max_ctx - NC : pos);
            return ((p + NC - 1) / op.at.chunk_len + 1) * op.at.n_kv;
        }
        case POP_COMBINE: return op.at.n_head * NC * (kHdA / 32);
        case POP_DRAFT_PREP: return NC * kDraftParts;
        case POP_CTRL: return 1;
        default: return 0;
    }
}

// Shared-memory scratch (bytes) of the non-GEMV bodies.
__host__ __device__ constexpr int gdn_scratch_floats(int nc) { return nc * (256 + 32 + 128 + 128 + 8) + 4; }
__host__ __device__ constexpr int attn_scratch_floats(int nc) {
    // (max, sum) pairs, then q + scores + the RoPE rows, or the [8][4][256] warp sums of the merge
    return 64 + (kGqa * nc * (kHdA + kSubA) + 8 * kHdA > 8 * 4 * kHdA ? kGqa * nc * (kHdA + kSubA) + 8 * kHdA : 8 * 4 * kHdA);
}
inline size_t op_scratch_bytes(int nc, int H) {
    size_t b = (size_t) gdn_scratch_floats(nc) * 4;
    const size_t a = (size_t) attn_scratch_floats(nc) * 4, d = (size_t) (H + H / 4) * 4;
    if (a > b) b = a;
    if (d > b) b = d;
    return (b + 127) & ~(size_t) 127;
}

// ------------------------------------------------------------------------------------------------
// Shared helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float silu_dev(float x) { return rk_siluf(x); }
__device__ __forceinline__ float sigmoid_dev(float x) { return rk_sigmoidf(x); }
__device__ __forceinline__ float softplus_gate_dev(float alpha, float dt, float ssm_a) {
    return rk_softplus_gate(alpha, dt, ssm_a);
}
// conv taps oldest first: sum = v0*w0, then fma(v1,w1), fma(v2,w2), fma(x,w3)
__device__ __forceinline__ float conv4_dev(float v0, float v1, float v2, float x, const float4 w) {
    float s = __fmul_rn(v0, w.x);
    s = __fmaf_rn(v1, w.y, s);
    s = __fmaf_rn(v2, w.z, s);
    return __fmaf_rn(x, w.w, s);
}
__device__ __forceinline__ float pick8(const float4 lo, const float4 hi, int i) {
    const float4 t = i < 4 ? lo : hi;
    const int j = i & 3;
    return j == 0 ? t.x : (j == 1 ? t.y : (j == 2 ? t.z : t.w));
}
__device__ __forceinline__ int read_token(Ctrl* ctrl, int draft, int c, int V) {
    int tok = ld_cg(draft ? &ctrl->dtok[c] : &ctrl->tok[c]);
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) {
            atomicOr(&g_rk_status, kStatusBadIndex);
            ctrl->bad = 1;
        }
        tok = 0;
    }
    return tok;
}
// dequantize_row_q6_K of one GGUF row, y = (d * scale) * (code - 32); thread t owns 16-value sub-blocks
// t, t+256, ...; also the row's 4-value sum-of-squares partials.
__device__ __forceinline__ void dequant_row(const uint8_t* row, int H, float* x, float* xp) {
    for (int sub = threadIdx.x; sub < H / 16; sub += 256) {
        const uint8_t* blk = row + (size_t) (sub >> 4) * 210;
        const float d = __half2float(*reinterpret_cast<const __half*>(blk + 208));
        const float ds = __fmul_rn(d, (float) (int8_t) blk[192 + (sub & 15)]);
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int v = ((sub & 15) << 4) + i;
            const int h = v >> 7, vv = v & 127, j = vv >> 5, l = vv & 31;
            const uint8_t qlb = blk[64 * h + l + 32 * (j & 1)];
            const int code = ((j >> 1) ? (qlb >> 4) : (qlb & 15)) | (((blk[128 + 32 * h + l] >> (2 * j)) & 3) << 4);
            const float y = __fmul_rn(ds, (float) (code - 32));
            x[sub * 16 + i] = y;
            part[i >> 2] = __fmaf_rn(y, y, part[i >> 2]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) xp[sub * 4 + k] = part[k];
    }
}

// ------------------------------------------------------------------------------------------------
// Bodies (one work item each, called by threads 0..255 of a block; block_sync256 is their barrier)
// ------------------------------------------------------------------------------------------------
// Token embedding of column c (the reference copies a host-dequantized row, src/qwythos.cpp:1782-1789).
// The trunk embedding also clears the argmax slots the lm_head fills.
__device__ __noinline__ void embed_body(const EmbedArgs& a, Ctrl* ctrl, int draft, int c) {
    const int tok = read_token(ctrl, draft, c, a.V);
    if (!draft && c == 0 && threadIdx.x == 0) {
        ctrl->amax[0] = 0ull;
        ctrl->amax[1] = 0ull;
    }
    const size_t rb = (size_t) (a.H / 256) * 210;
    dequant_row(a.emb + (size_t) tok * rb, a.H, a.x + (size_t) c * a.H, a.xp + (size_t) c * (a.H / 4));
}

// One GDN layer for quarter `quarter` (state columns quarter*32 .. +31) of v-head `head` and NC tokens
// at positions pos .. pos+NC-1: the reference's beta_gate + fused_gdn_conv_l2 +
// fused_gdn_step_norm_silu_q8 (src/qwythos.cpp:707-715, src/fused_gdn.cu:39-133).
//  * conv + SiLU + L2 of the paired k-head's q and k (head % hk, the modulo pairing of
//    src/fused_gdn.cu:57; every quarter of both v-heads of a k-head computes the same values, the block
//    of v-head kh < hk, quarter 0 writes their history) and of this quarter's 32 v channels;
//  * the 128 x 32 state slice stepped in registers column by column (threads 0..127: column = lane,
//    row group = warp), the state after column 0 kept in `snap` when NC == 2 (the verify's rollback);
//  * the gated RMSNorm over the head's 128 outputs and the Q8_1 epilogue by the head's last quarter
//    to finish (a per-head arrival counter).
// Reduction order of the reference kernel: 32-row fma chains per row group, groups added 0..3, per-32
// channel xor trees added in order. History: 8 slots per channel; this launch writes slots pos, pos+1
// and reads pos-3 .. pos-1 (mod 8), so no write of any block can meet a read of another.
template <int NC>
__device__ __forceinline__ void gdn_quarter_impl(const GdnArgs& a, int head, int quarter, int pos, bool from_snap,
                                                 float* sm) {
    constexpr int S = kSsm;
    float* kq = sm;                     // [NC][256]: normalized k (0..127) | q (128..255)
    float* vloc = kq + NC * 256;        // [NC][32]
    float* red_kv = vloc + NC * 32;     // [NC][4][32]
    float* red_o = red_kv + NC * 128;   // [NC][4][32]
    float* qk_part = red_o + NC * 128;  // [NC][8]
    int* last = reinterpret_cast<int*>(qk_part + NC * 8);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int hk = a.hk, hv = a.hv, kh = head % hk;
    const int C = 2 * hk * S + hv * S;
    const int off_z = C, off_beta = C + hv * S, off_alpha = off_beta + hv;
    block_sync256();  // scratch reuse across items
    // Loads that do not depend on the conv go out first: the state slice (threads 0..127: column = lane,
    // row group = warp), the gate inputs and z.
    const bool stepper = tid < 128;
    const int col = lane, rg = wid & 3;
    const size_t rs = (size_t) hv * S;
    float* sbase = a.state + ((size_t) (rg * 32) * hv + head) * S + quarter * 32 + col;
    float* pbase = a.snap + ((size_t) (rg * 32) * hv + head) * S + quarter * 32 + col;
    float s[32];
    float beta_in[NC], alpha_in[NC], z_in[NC];
    if (stepper) {
        const float* src = from_snap ? pbase : sbase;
#pragma unroll
        for (int r = 0; r < 32; ++r) s[r] = ld_cg(src + r * rs);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float* pc = a.proj + (size_t) c * a.proj_stride;
            beta_in[c] = ld_cg(pc + off_beta + head);
            alpha_in[c] = ld_cg(pc + off_alpha + head);
            z_in[c] = ld_cg(pc + off_z + head * S + wid * 32 + lane);  // column this thread normalizes if last
        }
    }
    auto conv = [&](int ch, float (&x)[NC], float (&yv)[NC]) {
        const float4* rp = reinterpret_cast<const float4*>(a.ring + (size_t) ch * kRingSlots);
        const float4 lo = __ldcg(rp), hi = __ldcg(rp + 1);
        const float4 w = reinterpret_cast<const float4*>(a.conv_w)[ch];
#pragma unroll
        for (int c = 0; c < NC; ++c) x[c] = ld_cg(a.proj + (size_t) c * a.proj_stride + ch);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            float in[3];
#pragma unroll
            for (int t = 0; t < 3; ++t) {
                const int d = c - 3 + t;  // the input at position pos + d
                in[t] = d < 0 ? pick8(lo, hi, (pos + d) & 7) : x[d < 0 ? 0 : d];
            }
            yv[c] = silu_dev(conv4_dev(in[0], in[1], in[2], x[c], w));
        }
    };
    {  // thread j: channel j of head kh's [q 128 | k 128]
        const int j = tid;
        const int ch = j < S ? kh * S + j : hk * S + kh * S + (j - S);
        float x[NC], yv[NC];
        conv(ch, x, yv);
        if (head < hk && quarter == 0) {
#pragma unroll
            for (int c = 0; c < NC; ++c) a.ring[(size_t) ch * kRingSlots + ((pos + c) & 7)] = x[c];
        }
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float sq = warp_sum(__fmul_rn(yv[c], yv[c]));
            if (lane == 0) qk_part[c * 8 + wid] = sq;
            kq[c * 256 + (j < S ? S + j : j - S)] = yv[c];
        }
    }
    if (wid == 0) {  // this quarter's v channels
        const int ch = 2 * hk * S + head * S + quarter * 32 + lane;
        float x[NC], yv[NC];
        conv(ch, x, yv);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            a.ring[(size_t) ch * kRingSlots + ((pos + c) & 7)] = x[c];
            vloc[c * 32 + lane] = yv[c];
        }
    }
    block_sync256();
#pragma unroll
    for (int c = 0; c < NC; ++c) {  // L2 norms: q from warps 0-3' partials, k from warps 4-7'
        const float* p = qk_part + c * 8;
        const float ssq = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), p[2]), p[3]);
        const float ssk = __fadd_rn(__fadd_rn(__fadd_rn(p[4], p[5]), p[6]), p[7]);
        const int idx = tid < S ? S + tid : tid - S;
        kq[c * 256 + idx] = __fmul_rn(kq[c * 256 + idx], rk_rsqrtf(__fadd_rn(tid < S ? ssq : ssk, a.eps)));
    }
    // ---- the state step ----
    block_sync256();
    float oc[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const float* kk = kq + c * 256;
        const float* qq = kk + S;
        float* rk = red_kv + c * 128;
        float* ro = red_o + c * 128;
        float beta = 0.0f, g = 0.0f;
        if (stepper) {
            beta = sigmoid_dev(beta_in[c]);
            g = rk_expf(softplus_gate_dev(alpha_in[c], a.dt[head], a.ssm_a[head]));
            float kv = 0.0f;
#pragma unroll
            for (int r = 0; r < 32; ++r) kv = __fmaf_rn(s[r], kk[rg * 32 + r], kv);
            rk[rg * 32 + col] = kv;
        }
        block_sync256();
        if (stepper) {
            const float kv_col = __fadd_rn(__fadd_rn(__fadd_rn(rk[col], rk[32 + col]), rk[64 + col]), rk[96 + col]);
            const float delta = __fmul_rn(__fsub_rn(vloc[c * 32 + col], __fmul_rn(g, kv_col)), beta);
            float o = 0.0f;
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                s[r] = __fmaf_rn(g, s[r], __fmul_rn(kk[rg * 32 + r], delta));
                o = __fmaf_rn(s[r], qq[rg * 32 + r], o);
            }
            ro[rg * 32 + col] = o;
        }
        block_sync256();
        oc[c] = 0.0f;
        if (stepper) {
            oc[c] = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(ro[col], ro[32 + col]), ro[64 + col]), ro[96 + col]),
                              kInvSqrtSsm);
            if (NC == 2 && c == 0) {  // the verify's rollback point
#pragma unroll
                for (int r = 0; r < 32; ++r) pbase[r * rs] = s[r];
            }
        }
    }
    if (stepper) {
#pragma unroll
        for (int r = 0; r < 32; ++r) sbase[r * rs] = s[r];
    }
    // ---- read-outs and sums of squares to the head's scratch; the last quarter normalizes ----
    if (wid == 0) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            a.o_scr[((size_t) c * hv + head) * S + quarter * 32 + lane] = oc[c];
            const float sq = warp_sum(__fmul_rn(oc[c], oc[c]));
            if (lane == 0) a.ss_scr[((size_t) c * hv + head) * 4 + quarter] = sq;
        }
        __threadfence();
    }
    block_sync256();
    if (tid == 0) *last = atomicAdd(a.cnt + head, 1u) == 3u;
    block_sync256();
    if (*last) {
        __threadfence();
        if (tid < S) {  // warp w: quarter w of the head
            const int j = wid * 32 + lane;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float* q4 = a.ss_scr + ((size_t) c * hv + head) * 4;
                const float ss = __fadd_rn(__fadd_rn(__fadd_rn(ld_cg(q4), ld_cg(q4 + 1)), ld_cg(q4 + 2)), ld_cg(q4 + 3));
                const float ocj = ld_cg(a.o_scr + ((size_t) c * hv + head) * S + j);
                const float z = z_in[c];
                const float scale = rk_rsqrtf(__fadd_rn(__fdiv_rn(ss, (float) S), a.eps));
                const float yv = __fmul_rn(__fmul_rn(__fmul_rn(ocj, scale), a.gamma[j]), silu_dev(z));
                if (a.y) a.y[(size_t) c * hv * S + head * S + j] = yv;
                q8_1_warp_store(yv, a.q8 + ((size_t) c * hv * 4 + head * 4 + wid) * 36, lane);
            }
        }
        if (tid == 0) a.cnt[head] = 0u;
    }
}

// The GDN item as a call (the op kernel and the persistent kernel); gdn_kernel inlines the impl.
template <int NC>
__device__ __noinline__ void gdn_quarter_body(const GdnArgs& a, int head, int quarter, int pos, bool from_snap,
                                                 float* sm) {
    gdn_quarter_impl<NC>(a, head, quarter, pos, from_snap, sm);
}

// Flash-decode chunk `chunk` of kv head kvh for NC query columns (gqa_head_kernel, src/qwythos.cpp:380-442,
// split over chunks of a.chunk_len <= kSubA tokens), with the attention prologue of the tokens it needs
// folded in: split of q / gate (split_qg_kernel, :320-327), per-head RMSNorm, NEOX RoPE over n_rot dims from
// the cos / sin table, and the fp16 K/V store (store_kv2_kernel, :340-345) of the new positions inside this
// chunk (each position has exactly one owning chunk). Column c attends tokens <= pos + c. One pass: scores
// of every (head, column, token) into shared memory, the chunk's max and exponential sum per (head,
// column), then the weighted V rows, warp w summing tokens [32 w, 32 w + 32) with lane l on dims 8 l ..
// 8 l + 7, and the eight warp sums added in warp order. The token-to-warp split does not depend on NC, so a
// column's partial is the same for any column count. Partials: o [n_head][NC][max_chunks][256],
// (m, l) [n_head][NC][max_chunks].
template <int NC, int G = kGqa>
__device__ __forceinline__ void attn_chunk_impl(const AttnArgs& a, int pos, int chunk, int kvh, float* sm) {
    static_assert(G == 2 || G == 4, "2 or 4 q heads per kv head");
    constexpr int GC = G * NC;
    if (pos < 0 || pos + NC > a.max_ctx) {  // uniform over the block
        if (threadIdx.x == 0) atomicOr(&g_rk_status, kStatusBadIndex);
        return;
    }
    const int len = a.chunk_len;
    const int t0 = chunk * len;
    if (t0 > pos + NC - 1 || chunk >= a.max_chunks) return;  // beyond every column (uniform over the block)
    const int tend = min(t0 + len, pos + NC);                  // tokens [t0, tend) some column may read
    if (threadIdx.x == 0) {  // the chunk's K rows (contiguous per kv head) head for L2 now; V after the scores
        const uint32_t bytes = (uint32_t) (tend - t0) * kHdA * 2;
        const size_t row0 = ((size_t) kvh * a.max_ctx + t0) * kHdA;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.kc + row0), "r"(bytes) : "memory");
    }
    float* mlc = sm;                    // [GC][2]: the chunk's max and exponential sum (64 floats reserved)
    float* qs = sm + 64;                // [GC][256]
    float* scb = qs + GC * kHdA;        // [GC][kSubA]: scores, then their exponentials
    float* rot = scb + GC * kSubA;      // [8 warps][256]
    float* wacc = sm + 64;              // [8 warps][4][256]: warp sums in the merge (aliases qs / scb / rot)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    block_sync256();  // scratch reuse across items
    // ---- prologue: one warp per head vector (lane holds dims j*32 + lane), the block256 order ----
    for (int job = warp; job < G * NC + NC; job += 8) {
        const bool is_q = job < G * NC;
        const int g = is_q ? job / NC : 0;
        const int c = is_q ? job % NC : job - G * NC;
        const int pc = pos + c;
        if (!is_q && (pc < t0 || pc >= t0 + len)) continue;  // a key this chunk does not own
        const float* col = a.proj + (size_t) c * a.proj_stride;
        const float* src = is_q ? col + (kvh * G + g) * 2 * kHdA : col + a.n_head * 2 * kHdA + kvh * kHdA;
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = ld_cg(src + j * 32 + lane);
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float pj = warp_sum(__fmul_rn(x[j], x[j]));
            ss = j == 0 ? pj : __fadd_rn(ss, pj);
        }
        const float inv = rk_rsqrtf(__fadd_rn(__fdiv_rn(ss, (float) kHdA), a.eps));
        const float* nw = is_q ? a.qn : a.kn;
        float* r = rot + warp * kHdA;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            x[j] = __fmul_rn(__fmul_rn(x[j], inv), nw[j * 32 + lane]);
            r[j * 32 + lane] = x[j];
        }
        __syncwarp();
        const int half = a.n_rot / 2;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int d = j * 32 + lane;
            if (d < a.n_rot) {
                const int i = d < half ? d : d - half;
                const float cs = a.rope[((size_t) pc * half + i) * 2 + 0];
                const float sn = a.rope[((size_t) pc * half + i) * 2 + 1];
                const float x0 = r[i], x1 = r[i + half];
                x[j] = d < half ? __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
            }
        }
        __syncwarp();  // `r` is rewritten by this warp's next job
        if (is_q) {
#pragma unroll
            for (int j = 0; j < 8; ++j) qs[(g * NC + c) * kHdA + j * 32 + lane] = x[j];
        } else {
            const size_t dst = ((size_t) kvh * a.max_ctx + pc) * kHdA;
            const float* vsrc = col + a.n_head * 2 * kHdA + a.n_kv * kHdA + kvh * kHdA;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                a.kc[dst + j * 32 + lane] = __float2half_rn(x[j]);
                a.vc[dst + j * 32 + lane] = __float2half_rn(ld_cg(vsrc + j * 32 + lane));
            }
        }
    }
    block_sync256();  // q in smem; this block's K/V stores visible to its threads
    const __half* kbase = a.kc + (size_t) kvh * a.max_ctx * kHdA;
    const __half* vbase = a.vc + (size_t) kvh * a.max_ctx * kHdA;
    const int ntok = tend - t0;  // <= kSubA
    // phase 1: scores, a warp per 4 consecutive tokens (their K rows loaded together), lanes over 8-dim
    // slices; the G * NC * 4 dot products are summed over the lanes by one reduce-scatter (the sums
    // warp_sum gives), after which each value's lane stores it
    for (int tb = warp * 4; tb < ntok; tb += 32) {
        float kf[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            uint4 kraw = make_uint4(0u, 0u, 0u, 0u);
            if (tb + u < ntok) kraw = __ldcg(reinterpret_cast<const uint4*>(kbase + (size_t) (t0 + tb + u) * kHdA + lane * 8));
            const __half2* kh2 = reinterpret_cast<const __half2*>(&kraw);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(kh2[i]);
                kf[u][2 * i] = f.x;
                kf[u][2 * i + 1] = f.y;
            }
        }
        constexpr int M = GC * 4;  // value j = (g * NC + c) * 4 + u
        float dv[M];
#pragma unroll
        for (int gc = 0; gc < GC; ++gc) {
            const float4* qp = reinterpret_cast<const float4*>(qs + gc * kHdA + lane * 8);
            const float4 q0 = qp[0], q1 = qp[1];
            const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float d = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) d = __fmaf_rn(qv[i], kf[u][i], d);
                dv[gc * 4 + u] = d;
            }
        }
        warp_reduce_scatter<M>(dv, lane);
        constexpr int R = M >= 32 ? M / 32 : 1;
        constexpr int SH = M >= 32 ? 0 : (M == 16 ? 1 : 2);
        if ((lane & ((1 << SH) - 1)) == 0) {
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const int j = M >= 32 ? R * lane + i : lane >> SH;
                const int gc = j >> 2, t = tb + (j & 3), c = gc % NC;
                if (t < ntok) scb[gc * kSubA + t] = (t0 + t <= pos + c) ? __fmul_rn(dv[i], a.scale) : -INFINITY;
            }
        }
    }
    block_sync256();
    if (threadIdx.x == 0) {  // V rows head for L2 only now: fewer prefetched lines wait (and get evicted) in L2
        const uint32_t bytes = (uint32_t) (tend - t0) * kHdA * 2;
        const size_t row0 = ((size_t) kvh * a.max_ctx + t0) * kHdA;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.vc + row0), "r"(bytes) : "memory");
    }
    // this warp's first V rows go out now, so their round trip overlaps phase 2
    constexpr int kVB = 4;  // V rows per batch (16 B per lane each)
    const int tw0 = warp * 32, tw1 = min(tw0 + 32, ntok);
    uint4 vr[kVB];
    auto load_v = [&](int tb) {
#pragma unroll
        for (int u = 0; u < kVB; ++u)
            vr[u] = tb + u < tw1 ? __ldcg(reinterpret_cast<const uint4*>(vbase + (size_t) (t0 + tb + u) * kHdA + lane * 8))
                                 : make_uint4(0u, 0u, 0u, 0u);
    };
    load_v(tw0);
    // phase 2: per (head, column) the chunk's max, the exponentials (masked: 0) and their sum; a warp per pair
    for (int pair = warp; pair < GC; pair += 8) {
        float* sp = scb + pair * kSubA;
        float m = -INFINITY;
        for (int t = lane; t < ntok; t += 32) m = fmaxf(m, sp[t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < ntok; t += 32) {
            const float e = m == -INFINITY ? 0.0f : rk_expf(__fsub_rn(sp[t], m));
            sp[t] = e;
            l = __fadd_rn(l, e);
        }
        l = warp_sum(l);
        if (lane == 0) {
            mlc[pair * 2 + 0] = m;
            mlc[pair * 2 + 1] = l;
        }
    }
    block_sync256();
    // phase 3: weighted V rows, this warp's tokens in order
    float acc[GC][8];
#pragma unroll
    for (int gc = 0; gc < GC; ++gc)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[gc][i] = 0.0f;
    for (int tb = tw0; tb < tw1; tb += kVB) {
        if (tb > tw0) load_v(tb);
#pragma unroll
        for (int u = 0; u < kVB; ++u)
            if (tb + u < tw1) {
                const __half2* vh2 = reinterpret_cast<const __half2*>(&vr[u]);
                float vf[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __half22float2(vh2[i]);
                    vf[2 * i] = f.x;
                    vf[2 * i + 1] = f.y;
                }
#pragma unroll
                for (int gc = 0; gc < GC; ++gc) {
                    const float pw = scb[gc * kSubA + tb + u];
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[gc][i] = __fmaf_rn(pw, vf[i], acc[gc][i]);
                }
            }
    }
    // merge: up to 4 (head, column) pairs per round, warp sums added in warp order by thread d = dim
    constexpr int QR = GC < 4 ? GC : 4;
#pragma unroll
    for (int r0 = 0; r0 < GC; r0 += QR) {
        block_sync256();  // wacc aliases the scores (first round) and the previous round
#pragma unroll
        for (int q = 0; q < QR; ++q) {
            float4* dst = reinterpret_cast<float4*>(wacc + (warp * 4 + q) * kHdA + lane * 8);
            dst[0] = make_float4(acc[r0 + q][0], acc[r0 + q][1], acc[r0 + q][2], acc[r0 + q][3]);
            dst[1] = make_float4(acc[r0 + q][4], acc[r0 + q][5], acc[r0 + q][6], acc[r0 + q][7]);
        }
        block_sync256();
#pragma unroll
        for (int q = 0; q < QR; ++q) {
            float o = wacc[q * kHdA + tid];
#pragma unroll
            for (int w = 1; w < 8; ++w) o = __fadd_rn(o, wacc[(w * 4 + q) * kHdA + tid]);
            const size_t slot = ((size_t) kvh * GC + r0 + q) * a.max_chunks + chunk;
            a.part_o[slot * kHdA + tid] = o;
        }
    }
    if (tid < GC) {
        const size_t slot = ((size_t) kvh * GC + tid) * a.max_chunks + chunk;
        a.part_ml[slot * 2 + 0] = mlc[tid * 2 + 0];
        a.part_ml[slot * 2 + 1] = mlc[tid * 2 + 1];
    }
}

// The chunk body as a call (the op kernel and the persistent kernel); attn_kernel inlines the impl.
template <int NC>
__device__ __noinline__ void attn_chunk_body(const AttnArgs& a, int pos, int chunk, int kvh, float* sm) {
    if (a.n_head == 2 * a.n_kv) attn_chunk_impl<NC, 2>(a, pos, chunk, kvh, sm);  // 8-way tensor parallelism
    else attn_chunk_impl<NC>(a, pos, chunk, kvh, sm);
}

// Combine of head h, column c, dims [32 slice, 32 slice + 32), then that dims' Q8_1 block of
// o * sigmoid(gate) (sig_mul_quant_kernel, src/qwythos.cpp:692-704; one warp = one 32-dim block). Warp w
// merges chunks [w n / 8, (w + 1) n / 8) (lane = one dim, 16 chunks' rows in flight), then warp 0 merges
// the eight warp partials in warp order: the same merge for any column count and any slicing, so a dim's
// result does not depend on which item computed it. sm: 8 x 32 + 16 floats.
template <int NC>
__device__ __forceinline__ void combine_impl(const AttnArgs& a, int pos, int h, int c, int slice, float* sm) {
    constexpr int kU = 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (pos < 0 || pos + NC > a.max_ctx) return;  // recorded by the chunk body
    float* wnum = sm;         // [8][32]
    float* wm = sm + 8 * 32;  // [8] warp maxima (-inf: the warp had no chunk)
    float* wden = wm + 8;     // [8]
    block_sync256();          // scratch reuse across items
    const int n = (pos + c) / a.chunk_len + 1;
    const int d = slice * 32 + lane;
    const float* ml = a.part_ml + ((size_t) h * NC + c) * a.max_chunks * 2;
    const float* po = a.part_o + ((size_t) h * NC + c) * a.max_chunks * kHdA + d;
    const int k0 = warp * n / 8, k1 = (warp + 1) * n / 8;
    float m = -INFINITY;
    for (int k = k0 + lane; k < k1; k += 32) m = fmaxf(m, ld_cg(ml + 2 * k));
    m = warp_max(m);
    float num = 0.0f, den = 0.0f;
    for (int k = k0; k < k1; k += kU) {
        float mk[kU], lk[kU], ok[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (k + u < k1) {
                mk[u] = ld_cg(ml + 2 * (k + u));
                lk[u] = ld_cg(ml + 2 * (k + u) + 1);
                ok[u] = ld_cg(po + (size_t) (k + u) * kHdA);
            }
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (k + u < k1) {
                const float w = rk_expf(__fsub_rn(mk[u], m));
                num = __fmaf_rn(w, ok[u], num);
                den = __fmaf_rn(w, lk[u], den);
            }
    }
    wnum[warp * 32 + lane] = num;
    if (lane == 0) {
        wm[warp] = k1 > k0 ? m : -INFINITY;
        wden[warp] = den;
    }
    block_sync256();
    if (warp != 0) return;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w]);
    float nu = 0.0f, de = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w)
        if (wm[w] != -INFINITY) {
            const float sw = rk_expf(__fsub_rn(wm[w], M));
            nu = __fmaf_rn(sw, wnum[w * 32 + lane], nu);
            de = __fmaf_rn(sw, wden[w], de);
        }
    const float ov = __fdiv_rn(nu, de);
    const size_t oi = ((size_t) c * a.n_head + h) * kHdA + d;
    if (a.o) a.o[oi] = ov;
    const float gate = ld_cg(a.proj + (size_t) c * a.proj_stride + h * 2 * kHdA + kHdA + d);
    q8_1_warp_store(sigmul_value(ov, gate), a.q8 + (((size_t) c * a.n_head + h) * (kHdA / 32) + slice) * 36, lane);
}

// The combine item as a call (the op kernel and the persistent kernel); combine_kernel inlines the impl.
template <int NC>
__device__ __noinline__ void combine_body(const AttnArgs& a, int pos, int h, int c, int slice, float* sm) {
    combine_impl<NC>(a, pos, h, c, slice, sm);
}

// MTP draft input of column c: Q8_1 of [enorm(emb(dtok)) | hnorm(h)] (src/qwythos.cpp:1316-1334); the
// draft's argmax slots are cleared here. Item `part` (kDraftParts per column) quantizes 32-value blocks
// [part * H / 256, (part + 1) * H / 256): parts 0..7 the embedding half (each dequantizes the whole row
// for its RMS), parts 8..15 the hidden half; the scales are those of one whole-row pass. sm: H + H/4 floats.
__device__ __noinline__ void draft_prep_body(const DraftPrepArgs& a, Ctrl* ctrl, int c, int part, float* sm,
                                             float* red) {
    const int H = a.H;
    float* e = sm;
    float* ep = sm + H;
    block_sync256();  // scratch reuse across items
    if (c == 0 && part == 0 && threadIdx.x == 0) {
        ctrl->damax[0] = 0ull;
        ctrl->damax[1] = 0ull;
    }
    const bool emb_half = part < kDraftParts / 2;  // uniform over the block
    float inv;
    if (emb_half) {
        const int tok = read_token(ctrl, 1, c, a.V);
        dequant_row(a.emb + (size_t) tok * ((size_t) (H / 256) * 210), H, e, ep);
        block_sync256();
        inv = rms_inv(block256_partials_sum<true>(ep, H / 4, red), H, a.eps);
    } else {
        inv = rms_inv(block256_partials_sum(a.hsave_p + (size_t) c * (H / 4), H / 4, red), H, a.eps);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = (2 * H / 32) / kDraftParts;
    const float* hc = a.hsave + (size_t) c * H;
    uint8_t* out = a.eh_q8 + (size_t) c * (2 * H / 32) * 36;
    for (int blk = part * nb + warp; blk < (part + 1) * nb; blk += 8) {
        const int i = blk * 32 + lane;
        const float v = i < H ? rms_value(e[i], a.enorm[i], inv) : rms_value(ld_cg(hc + i - H), a.hnorm[i - H], inv);
        q8_1_warp_store(v, out + (size_t) blk * 36, lane);
    }
}

// Control ops (thread 0 of one block).
__device__ __noinline__ void ctrl_body(const CtrlArgs& a, Ctrl* ctrl) {
    volatile Ctrl* v = ctrl;
    if (a.kind == CTRL_SINGLE) {
        // emit the trunk argmax and advance (src/qwythos.cpp:1803-1811, :3184-3192)
        const int id = argmax_key_row(v->amax[0]);
        const int n = v->n_emitted;
        if (n < a.max_out) a.out[n] = id;
        v->n_emitted = n + 1;
        if (id + 1 == v->eos1) v->stop = 1;  // emitted, never ingested
        v->tok[0] = id;
        v->dtok[0] = id;
        v->dpos = v->pos + 1;
        v->pos = v->pos + 1;
        v->rollback = 0;
        v->singles = v->singles + 1;
    } else if (a.kind == CTRL_ACCEPT) {
        // greedy acceptance (src/qwythos.cpp:3196-3238): c0 = argmax of column 0; accepted iff c0 == the
        // candidate; emit c0 (and c1 when accepted); the draft then runs on (c0 at pos+1, c1 at pos+2)
        const int c0 = argmax_key_row(v->amax[0]), c1 = argmax_key_row(v->amax[1]);
        int n = v->n_emitted;
        if (n < a.max_out) a.out[n] = c0;
        ++n;
        if (c0 + 1 == v->eos1) {
            // emitted and not ingested: the state keeps column 0 only (the snapshot), whatever the draft was
            v->n_emitted = n;
            v->stop = 1;
            v->dtok[0] = c0;
            v->dtok[1] = c1;
            v->dpos = v->pos + 1;
            v->pos = v->pos + 1;
            v->rollback = 1;
            v->accept = 0;
            v->steps = v->steps + 1;
            __threadfence();
            return;
        }
        const int acc = c0 == v->tok[1];
        if (acc && c1 + 1 == v->eos1) v->stop = 1;  // c1 is emitted below and stays pending
        if (acc) {
            if (n < a.max_out) a.out[n] = c1;
            ++n;
        }
        v->n_emitted = n;
        v->dtok[0] = c0;
        v->dtok[1] = c1;
        v->dpos = v->pos + 1;
        v->tok[0] = acc ? c1 : c0;
        v->pos = v->pos + 1 + acc;
        v->rollback = !acc;
        v->accept = acc;
        v->steps = v->steps + 1;
        v->accepted = v->accepted + acc;
    } else if (a.kind == CTRL_ROUND || a.kind == CTRL_DRAFT1) {
        // the next candidate, for position pos + 1: the draft column that predicts the position after the
        // last emitted token, unless the host forced one for that position (a test hook that drives the
        // accept branch with known tokens; the emitted stream does not depend on the candidate)
        int cand = argmax_key_row(v->damax[a.kind == CTRL_ROUND && v->accept ? 1 : 0]);
        const int p1 = v->pos + 1;
        if (a.force != nullptr && p1 >= 0 && p1 < a.n_force) {
            const int f = a.force[p1];
            if (f >= 0) cand = f;
        }
        v->tok[1] = cand;
    }
    __threadfence();
}

// One work item of a non-GEMV op. `pos` is the op's position (trunk or draft) and `rollback` the
// GDN snapshot flag, both read from the control block when the op starts.
template <int NC>
__device__ __forceinline__ void run_item(const POp& op, Ctrl* ctrl, int item, int pos, int rollback, float* sm,
                                         float* red) {
    switch (op.kind) {
        case POP_EMBED: embed_body(op.em, ctrl, op.draft, item); break;
        case POP_GDN: gdn_quarter_body<NC>(op.gd, item >> 2, item & 3, pos, rollback != 0, sm); break;
        case POP_ATTN: attn_chunk_body<NC>(op.at, pos, item / op.at.n_kv, item % op.at.n_kv, sm); break;
        case POP_COMBINE: combine_body<NC>(op.at, pos, item / (NC * 8), (item / 8) % NC, item % 8, sm); break;
        case POP_DRAFT_PREP: draft_prep_body(op.dp, ctrl, item / kDraftParts, item % kDraftParts, sm, red); break;
        case POP_CTRL:
            if (threadIdx.x == 0) ctrl_body(op.ct, ctrl);
            break;
        default: break;
    }
}

}  // namespace rk
