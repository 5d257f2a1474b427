// engine.cu — the decode engine for the qwen35 hybrid model: the reference's Engine / load_model /
// forward_token / draft_predict / launch_token_verify (src/qwythos.cpp:152-281, :1228-1618, :1757-1824,
// :1978-2134, :2905-3251) rebuilt around op programs and a device-side control block.
//
// Every step kind is an op program (decode_ops.cuh): one token; the trunk over 2 columns; an MTP round
// (2-column verify -> accept -> 2-column draft -> next candidate); the first draft; the draft seed. Every
// op reads its tokens, positions and the rollback flag from the device Ctrl block, so no step needs a
// host round trip. Two executors (persistent.cuh) run a program: one kernel per op, replayed from a CUDA
// graph (the single-GPU default), or one persistent cooperative kernel (a whole generation in one launch);
// RK_ENGINE_MODE=graph|persistent chooses. Both write the same bits, under tensor parallelism too (the
// row-parallel exchange runs inside the GEMV op in either, xch.cuh).
//
// Ops per trunk layer:
//   GDN  : GEMV qkv||z||beta||alpha (RMSNorm+Q8_1 prologue) -> GDN (conv / L2 / delta rule / gated norm /
//          Q8_1) -> GEMV ssm_out (+residual, partials) -> GEMV up||gate (RMSNorm prologue, SwiGLU+Q8_1
//          epilogue) -> GEMV down (+residual, partials)
//   ATTN : GEMV q||k||v (RMSNorm prologue) -> attention chunks (q/k norm, RoPE and the fp16 KV store
//          folded in) -> combine (sigmoid gate + Q8_1) -> GEMV wo (+residual) -> FFN as above
// then the lm_head GEMV with the final RMSNorm prologue and a fused argmax epilogue.
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <algorithm>
#include <vector>

#include "gguf.cuh"
#include "persistent.cuh"

namespace rk {
namespace {

constexpr float kAttnScale = 0.0625f;  // 1/sqrt(256)

// ------------------------------------------------------------------------------------------------
// Synthetic weights: value(i) of tensor t = (sum of the four 16-bit fields of hash(seed_t, i) - 131070)
// * scale + mean, seed_t = hash(model seed, t). Q6_K tensors are then encoded per 256-value block.
// ------------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint64_t hash64(uint64_t seed, uint64_t idx) {
    uint64_t z = seed * 0x9E3779B97F4A7C15ull + idx + 0x632BE59BD9B4E019ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ int synth_sum(uint64_t seed, uint64_t idx) {
    const uint64_t h = hash64(seed, idx);
    return (int) (h & 0xffff) + (int) ((h >> 16) & 0xffff) + (int) ((h >> 32) & 0xffff) + (int) ((h >> 48) & 0xffff) -
           131070;
}
float synth_scale(double std) { return (float) (std * std::sqrt(3.0) / 65536.0); }

// A seeded synthetic context (rk_engine_session_fill): rows [0, n_pos) of every kv head of a cache
// [n_kv][max_ctx][256] as fp16 of synthetic N(0, 1) values; a float buffer of synthetic N(0, std) values.
__global__ void fill_kv_kernel(__half* cache, int n_kv, int max_ctx, int n_pos, uint64_t seed, float scale) {
    const long long per_head = (long long) n_pos * 256;
    const long long n = per_head * n_kv;
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x) {
        const long long h = i / per_head, r = i - h * per_head;
        cache[(size_t) h * max_ctx * 256 + (size_t) r] = __float2half_rn((float) synth_sum(seed, (uint64_t) i) * scale);
    }
}
__global__ void fill_float_kernel(float* dst, long long n, uint64_t seed, float scale) {
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long) gridDim.x * blockDim.x)
        dst[i] = (float) synth_sum(seed, (uint64_t) i) * scale;
}

// Q6_K encoder (this library's definition, restated by the CPU oracle): per 16-value sub-block amax_j,
// d = half((max_j amax_j / 31) / 127), scale_j = clamp(roundf((amax_j / 31) / d), 0, 127),
// code = clamp(roundf(x / (d * scale_j)), -32, 31) + 32. One thread per 256-value block of a slice of the
// tensor: local rows are global rows grow0 + r, local column blocks are global column blocks
// [cb_a, cb_a + ncb_a) then [cb_b, cb_b + ncb_b) (nb_full blocks per global row), written into local rows
// of row_blocks >= ncb_a + ncb_b blocks (the rest left as the caller zeroed it); block bg of the global
// tensor holds values bg*256 .. bg*256+255, so a slice holds exactly the global tensor's values.
__global__ void gen_q6k_kernel(uint64_t seed, float scale, long long rows, long long grow0, int nb_full, int ncb_a,
                               int cb_a, int ncb_b, int cb_b, int row_blocks, uint8_t* __restrict__ out) {
    const long long b = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    const int ncb = ncb_a + ncb_b;
    if (b >= rows * ncb) return;
    const long long lr = b / ncb;
    const int lcb = (int) (b - lr * ncb);
    const long long bg = (grow0 + lr) * nb_full + (lcb < ncb_a ? cb_a + lcb : cb_b + (lcb - ncb_a));
    float x[256];
    float amax[16];
    float smax = 0.0f;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
        float a = 0.0f;
        for (int i = 0; i < 16; ++i) {
            const float v = __fmul_rn((float) synth_sum(seed, (uint64_t) bg * 256 + 16 * j + i), scale);
            x[16 * j + i] = v;
            a = fmaxf(a, fabsf(v));
        }
        amax[j] = a;
        smax = fmaxf(smax, a);
    }
    const __half dh16 = __float2half_rn(__fdiv_rn(__fdiv_rn(smax, 31.0f), 127.0f));
    const float dh = __half2float(dh16);
    uint8_t ql[128], qh[64];
    for (int i = 0; i < 128; ++i) ql[i] = 0;
    for (int i = 0; i < 64; ++i) qh[i] = 0;
    uint8_t* blk = out + ((size_t) lr * row_blocks + lcb) * 210;  // local rows are row_blocks blocks wide
    for (int j = 0; j < 16; ++j) {
        int sc = 0;
        if (dh > 0.0f) {
            const float s = roundf(__fdiv_rn(__fdiv_rn(amax[j], 31.0f), dh));
            sc = (int) fminf(fmaxf(s, 0.0f), 127.0f);
        }
        blk[192 + j] = (uint8_t) sc;
        const float eff = __fmul_rn(dh, (float) sc);
        for (int i = 0; i < 16; ++i) {
            int q = 0;
            if (eff > 0.0f) q = (int) fminf(fmaxf(roundf(__fdiv_rn(x[16 * j + i], eff)), -32.0f), 31.0f);
            const int code = q + 32, v = 16 * j + i;
            const int h = v >> 7, vv = v & 127, jj = vv >> 5, l = vv & 31;
            ql[64 * h + l + 32 * (jj & 1)] |= (uint8_t) ((code & 15) << (4 * (jj >> 1)));
            qh[32 * h + l] |= (uint8_t) (((code >> 4) & 3) << (2 * jj));
        }
    }
    for (int i = 0; i < 128; ++i) blk[i] = ql[i];
    for (int i = 0; i < 64; ++i) blk[128 + i] = qh[i];
    const unsigned short dbits = __half_as_ushort(dh16);
    blk[208] = (uint8_t) (dbits & 0xff);
    blk[209] = (uint8_t) (dbits >> 8);
}

// ------------------------------------------------------------------------------------------------
// Engine
// ------------------------------------------------------------------------------------------------
struct Mat {
    uint8_t* w = nullptr;  // packed tiles
    int n_in = 0, n_out = 0;
};
struct Layer {
    bool gdn = true;
    float* attn_norm = nullptr;
    float* post_norm = nullptr;
    Mat in_proj;   // GDN: qkv||z||beta||alpha; ATTN: q||k||v
    Mat out_proj;  // GDN: ssm_out; ATTN: wo
    Mat upgate, down;
    // GDN
    float *conv_w = nullptr, *dt = nullptr, *ssm_a = nullptr, *ssm_norm = nullptr;
    float *state = nullptr, *snap = nullptr, *ring = nullptr;
    // ATTN
    float *q_norm = nullptr, *k_norm = nullptr;
    __half *kc = nullptr, *vc = nullptr;
};

// Tensor ids of the synthetic model (also used by the CPU oracle of the tests).
enum : int { T_TOK_EMBD = 1, T_OUT_NORM = 2, T_OUTPUT = 3, T_ENORM = 4, T_HNORM = 5, T_EH_PROJ = 6, T_SHNORM = 7 };
enum : int {
    L_ATTN_NORM = 0, L_POST_NORM = 1, L_FFN_UP = 2, L_FFN_GATE = 3, L_FFN_DOWN = 4,
    L_GDN_QKV = 5, L_GDN_Z = 6, L_GDN_BETA = 7, L_GDN_ALPHA = 8, L_GDN_OUT = 9, L_GDN_CONV = 10, L_GDN_A = 11,
    L_GDN_DT = 12, L_GDN_NORM = 13,
    L_ATT_Q = 5, L_ATT_K = 6, L_ATT_V = 7, L_ATT_O = 8, L_ATT_QN = 9, L_ATT_KN = 10
};
inline int layer_tid(int il, int slot) { return 100 + 32 * il + slot; }

struct TensorRec {
    int tid;
    bool q6k;
    int n_in, n_out;
    void* dev;        // f32 data, or the packed group buffer
    size_t row_off;   // first row inside a packed group
    bool raw;         // stored as GGUF rows (token embedding)
};

// A step program: its ops on the host and the device, its column count, and its graph (graph mode).
struct Program {
    std::vector<POp> ops;
    POp* dev = nullptr;
    std::vector<GemvEnt> gemvs;  // its GEMVs in order (the persistent kernel's weight cursors)
    GemvEnt* gdev = nullptr;
    int nc = 1;
    cudaGraphExec_t graph = nullptr;
    int kernels = 0;  // kernels one run launches
};
enum : int { P_SINGLE = 0, P_TRUNK2, P_ROUND, P_DRAFT1, P_SEED, P_PROBE1, P_PROBE2, P_PREFILL, P_DRAFTX, P_COUNT };
// executor slot of a column count (1, 2, 4)
inline int col_slot(int nc) { return nc >= 4 ? 2 : nc - 1; }

POp make_op(int kind) {
    POp op;
    std::memset(&op, 0, sizeof op);
    op.kind = kind;
    return op;
}

}  // namespace

struct EngineImpl {
    rk_model_config cfg;
    int dev = 0;
    cudaStream_t s = nullptr;
    // Tensor parallelism: this rank's shard of the model (tp_size 1: the whole model). H is replicated;
    // FF, hk, hv, nh, nkv and V (lm_head rows) are this rank's shares; Vg is the vocabulary.
    int tp_rank = 0, tp_size = 1;
    int H = 0, FF = 0, V = 0, Vg = 0, hk = 0, hv = 0, nh = 0, nkv = 0;
    int qkvzab_rows = 0, qkv3_rows = 0, max_in_rows = 0, max_chunks = 0, chunk_len = 32;
    int kv0 = 0;  // global index of this rank's first kv head
    std::vector<Layer> layers;
    Layer draft;
    float *enorm = nullptr, *hnorm = nullptr, *shnorm = nullptr, *out_norm = nullptr;
    Mat eh_proj, lm_head;
    uint8_t* tok_embd = nullptr;
    float* rope = nullptr;
    // activations, 2 columns
    float *x = nullptr, *xp = nullptr, *proj = nullptr, *ug = nullptr;
    uint8_t* q8 = nullptr;                        // Q8_1 input of ssm_out (the GDN output)
    float *gdn_o = nullptr, *gdn_ss = nullptr;    // GDN read-outs / per-quarter sums of squares
    unsigned* gdn_cnt = nullptr;                  // GDN last-quarter counters
    float* attn_scratch = nullptr;                // flash-decode partials
    uint8_t *q8_ff = nullptr, *q8_attn = nullptr; // Q8_1 inputs of the down and wo GEMVs
    unsigned* swiglu_cnt = nullptr;               // last-arriver counters of the up||gate epilogue
    float *hsave = nullptr, *hsave_p = nullptr, *logits = nullptr;
    float *dx = nullptr, *dxp = nullptr;
    uint8_t* eh_q8 = nullptr;
    Ctrl* ctrl = nullptr;
    int* out = nullptr;
    int max_out = 0;
    int* force = nullptr;  // test hook: forced draft candidate per position (-1: the draft's own), max_ctx + 2
    Ctrl* ctrl_stage = nullptr;  // pinned host staging, one slot per queued host write
    int stage_slots = 0, stage_next = 0;
    // session (rk_engine_session_*): the next position to write, the last emitted token not yet ingested
    // (-1: none), the GDN rollback the next pass must honour, and whether the draft slot 0 was seeded
    int s_pos = 0, s_pending = -1, s_rollback = 0;
    bool s_primed = false;
    // a run failed after it had started to change the caches and states in place: the session's bookkeeping
    // no longer describes them, so runs are refused until a reset
    bool s_poisoned = false;
    // programs and executors
    Program progs[P_COUNT];
    bool persistent = false;
    PSync* psync = nullptr;
    int p_grid = 0, p_stages[3] = {0, 0, 0}, p_region[3] = {0, 0, 0};  // per column count (1, 2, 4)
    int p_l2pf = 0;  // bytes of the next GEMV each CTA asks L2 for when an op starts
    size_t p_smem[3] = {0, 0, 0};
    bool prefill4 = false;  // the 4-column prefill program exists (single GPU, and the executor fits it)
    double probe_weight_bytes[2] = {0, 0}, probe_algo_bytes[2] = {0, 0};
    int probe_gemvs = 0;
    // tensor parallelism: this rank's exchange memory (exported by CUDA IPC), the peers' mappings, and the
    // descriptor the kernels read
    uint8_t* xmem = nullptr;
    size_t xmem_bytes = 0, xoff_flags = 0, xoff_keys = 0, xoff_ep = 0;
    XchDesc* xdesc = nullptr;
    std::vector<void*> peer_maps;
    bool tp_connected = false;
    // weights from a GGUF file instead of the synthetic generator (during build only)
    const GgufFile* gg = nullptr;
    int src_rc = RK_OK;
    std::string src_msg;
    std::vector<uint8_t> stage;
    std::vector<void*> allocs;
    std::vector<TensorRec> tensors;
    size_t bytes = 0;
    cudaError_t err = cudaSuccess;

    ~EngineImpl();
    template <typename T>
    T* alloc(size_t n) {
        void* p = nullptr;
        if (err != cudaSuccess) return nullptr;
        err = cudaMalloc(&p, n * sizeof(T));
        if (err != cudaSuccess) return nullptr;
        allocs.push_back(p);
        bytes += n * sizeof(T);
        cudaMemsetAsync(p, 0, n * sizeof(T), s);
        return static_cast<T*>(p);
    }
    int build();
    void gen_f32(int tid, float* dst, size_t n, double std, double mean, int kind,
                 const std::vector<long long>* pick = nullptr);
    void gen_q6k(int tid, Mat& group, int row_off, int n_in_full, int grow0, int rows, int cb_a, int ncb_a, int cb_b,
                 int ncb_b, uint8_t* scratch, int row_blocks = 0, int grow1 = 0, int rows1 = 0);
    void gen_q6k_into(int tid, Mat& group, int row_off, int n_in, int n_out, uint8_t* scratch) {
        gen_q6k(tid, group, row_off, n_in, 0, n_out, 0, n_in / 256, 0, 0, scratch);
    }
    std::string gguf_name(int tid) const;
    bool src_fail(int rc, const std::string& msg) {
        if (src_rc == RK_OK) {
            src_rc = rc;
            src_msg = msg;
        }
        if (err == cudaSuccess) err = cudaErrorInvalidValue;
        return false;
    }
    // the input width a row-parallel GEMV over a share of `cols` values runs at: whole 1024-value tiles
    static int tp_in(int cols) { return (cols + 1023) / 1024 * 1024; }
    int gdn_vhead(int j) const {  // global v-head of local v-head j (the v-heads paired with this rank's k-heads)
        return j < hk ? tp_rank * hk + j : cfg.ssm_h_k + tp_rank * hk + (j - hk);
    }
    // programs
    MmvqParams rms_params(const Mat& m, const float* x_, const float* w, const float* part, float* y, int y_stride);
    MmvqParams q8_params(const Mat& m, const uint8_t* xq, float* y, const float* res, float* part, int x_cols = 0);
    void add_gemv(std::vector<POp>& v, int pro, int epi, const MmvqParams& p);
    void add_rowpar(std::vector<POp>& v, MmvqParams p);
    void add_ffn(std::vector<POp>& v, const Layer& L, float* xres, float* part);
    POp attn_op(int kind, const Layer& L, int draft_flag);
    void add_trunk(std::vector<POp>& v, bool head = true);
    void add_draft(std::vector<POp>& v, bool head, float* logits_out = nullptr);
    void add_ctrl(std::vector<POp>& v, int kind);
    void add_xargmax(std::vector<POp>& v, int draft_flag);
    void add_probe(std::vector<POp>& v, int nc);
    int setup_executor();
    int finalize(Program& P, int nc);
    template <int NC>
    cudaError_t launch_op(const POp& op);
    cudaError_t run(const Program& P, int until = 0, int max_iters = 1, unsigned long long* trace = nullptr);
    void set_ctrl(const Ctrl& host_fields);
    int check_abort(const char* what);
    void set_ctrl_eos(int eos_id);
    cudaError_t ingest(const int* toks, int n, int start, int rollback0, int& launches);
};

EngineImpl::~EngineImpl() {
    if (s) cudaStreamSynchronize(s);
    for (Program& P : progs)
        if (P.graph) cudaGraphExecDestroy(P.graph);
    for (void* p : peer_maps)
        if (p) cudaIpcCloseMemHandle(p);
    for (void* p : allocs) cudaFree(p);
    if (ctrl_stage) cudaFreeHost(ctrl_stage);
    if (s) cudaStreamDestroy(s);
}

// f32 tensors are generated on the host (they are small) with the same counter-based values the device
// uses; kind 1: ssm_a = -exp(value) computed in double. pick: the global indices this rank keeps (a
// tensor-parallel slice), n of them; else the whole tensor.
// The GGUF tensor name of this library's tensor id (the reference's names, src/qwythos.cpp:2003-2124).
std::string EngineImpl::gguf_name(int tid) const {
    const std::string nx = "blk." + std::to_string(cfg.n_layer) + ".nextn.";
    switch (tid) {
        case T_TOK_EMBD: return "token_embd.weight";
        case T_OUT_NORM: return "output_norm.weight";
        case T_OUTPUT: return "output.weight";
        case T_ENORM: return nx + "enorm.weight";
        case T_HNORM: return nx + "hnorm.weight";
        case T_EH_PROJ: return nx + "eh_proj.weight";
        case T_SHNORM: return nx + "shared_head_norm.weight";
        default: break;
    }
    const int il = (tid - 100) / 32, slot = (tid - 100) % 32;
    const bool gdn = il < cfg.n_layer && (il + 1) % cfg.attn_interval != 0;
    static const char* common[] = {"attn_norm.weight", "post_attention_norm.weight", "ffn_up.weight", "ffn_gate.weight",
                                   "ffn_down.weight"};
    static const char* gdn_names[] = {"attn_qkv.weight", "attn_gate.weight", "ssm_beta.weight", "ssm_alpha.weight",
                                      "ssm_out.weight", "ssm_conv1d.weight", "ssm_a", "ssm_dt.bias", "ssm_norm.weight"};
    static const char* att_names[] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                                      "attn_q_norm.weight", "attn_k_norm.weight"};
    const std::string b = "blk." + std::to_string(il) + ".";
    if (slot < 5) return b + common[slot];
    if (gdn && slot - 5 < 9) return b + gdn_names[slot - 5];
    if (!gdn && slot - 5 < 6) return b + att_names[slot - 5];
    return b + "?";
}

void EngineImpl::gen_f32(int tid, float* dst, size_t n, double std, double mean, int kind,
                         const std::vector<long long>* pick) {
    if (gg) {  // from the file: F32 / F16 / BF16, the picked global indices or the whole tensor
        const std::string name = gguf_name(tid);
        const GgufTensor* t = gg->find(name);
        if (!t) return (void) src_fail(RK_EINVAL, "tensor " + name + " missing");
        const size_t total = (size_t) (t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]);
        if ((t->type != kGgmlF32 && t->type != kGgmlF16 && t->type != kGgmlBF16) || (!pick && total != n))
            return (void) src_fail(RK_EUNSUPPORTED, "tensor " + name + ": expected " + std::to_string(n) + " F32/F16 values");
        std::vector<float> h(n);
        for (size_t i = 0; i < n; ++i) {
            const size_t gi = pick ? (size_t) (*pick)[i] : i;
            if (gi >= total) return (void) src_fail(RK_EINVAL, "tensor " + name + " too small");
            if (t->type == kGgmlF32) {
                std::memcpy(&h[i], t->data + gi * 4, 4);
            } else {
                uint16_t b16;
                std::memcpy(&b16, t->data + gi * 2, 2);
                if (t->type == kGgmlF16) {
                    h[i] = __half2float(__ushort_as_half(b16));
                } else {
                    const uint32_t u = (uint32_t) b16 << 16;
                    std::memcpy(&h[i], &u, 4);
                }
            }
        }
        if (err == cudaSuccess) err = cudaMemcpyAsync(dst, h.data(), n * sizeof(float), cudaMemcpyHostToDevice, s);
        if (err == cudaSuccess) err = cudaStreamSynchronize(s);
        tensors.push_back({tid, false, (int) n, 1, dst, 0, false});
        return;
    }
    std::vector<float> h(n);
    const uint64_t st = hash64(cfg.seed, (uint64_t) tid);
    const float scale = synth_scale(std), m = (float) mean;
    for (size_t i = 0; i < n; ++i) {
        const uint64_t gi = pick ? (uint64_t) (*pick)[i] : (uint64_t) i;
        volatile float v = (float) synth_sum(st, gi) * scale;
        float r = v + m;
        if (kind == 1) r = (float) -std::exp((double) r);
        h[i] = r;
    }
    if (err == cudaSuccess) err = cudaMemcpyAsync(dst, h.data(), n * sizeof(float), cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    tensors.push_back({tid, false, (int) n, 1, dst, 0, false});
}

// Q6_K rows [grow0, grow0 + rows) of tensor tid (n_in_full columns), keeping the 256-column blocks
// [cb_a, cb_a + ncb_a) then [cb_b, cb_b + ncb_b) of each row: generated as GGUF rows, then repacked into
// rows [row_off, row_off + rows) of a packed group whose rows are row_blocks * 256 wide (default
// ncb_a + ncb_b; wider rows end in all-zero blocks: d = 0, so they add exactly nothing to a dot product,
// whatever the activations they meet).
void EngineImpl::gen_q6k(int tid, Mat& group, int row_off, int n_in_full, int grow0, int rows, int cb_a, int ncb_a,
                         int cb_b, int ncb_b, uint8_t* scratch, int row_blocks, int grow1, int rows1) {
    if (row_blocks < ncb_a + ncb_b) row_blocks = ncb_a + ncb_b;
    const int n_in = row_blocks * 256;
    const size_t lrb = (size_t) row_blocks * 210;
    if (row_blocks > ncb_a + ncb_b && err == cudaSuccess)
        err = cudaMemsetAsync(scratch, 0, (size_t) (rows + rows1) * lrb, s);
    // rows [grow0, grow0 + rows), then (optional) rows [grow1, grow1 + rows1), staged back to back
    const int gr[2] = {grow0, grow1}, nr[2] = {rows, rows1};
    for (int k = 0; k < 2 && nr[k] > 0; ++k) {
        uint8_t* out = scratch + (size_t) (k == 0 ? 0 : rows) * lrb;
        if (gg) {  // the GGUF rows' bytes (this slice's column blocks), then the same repack
            const std::string name = gguf_name(tid);
            const GgufTensor* t = gg->find(name);
            if (!t) return (void) src_fail(RK_EINVAL, "tensor " + name + " missing");
            if (t->type != kGgmlQ6_K)
                return (void) src_fail(RK_EUNSUPPORTED, "tensor " + name + " is ggml type " + std::to_string(t->type) +
                                                            "; the engine's GEMVs take Q6_K (14)");
            if (t->ne[0] != n_in_full || t->ne[1] < (int64_t) gr[k] + nr[k])
                return (void) src_fail(RK_EINVAL, "tensor " + name + " has an unexpected shape");
            const size_t rb = ggml_row_bytes(kGgmlQ6_K, n_in_full);
            stage.assign((size_t) nr[k] * lrb, 0);
            for (int r = 0; r < nr[k]; ++r) {
                const uint8_t* src = t->data + (size_t) (gr[k] + r) * rb;
                std::memcpy(stage.data() + (size_t) r * lrb, src + (size_t) cb_a * 210, (size_t) ncb_a * 210);
                if (ncb_b) std::memcpy(stage.data() + (size_t) r * lrb + (size_t) ncb_a * 210, src + (size_t) cb_b * 210, (size_t) ncb_b * 210);
            }
            if (err == cudaSuccess) err = cudaMemcpyAsync(out, stage.data(), stage.size(), cudaMemcpyHostToDevice, s);
            if (err == cudaSuccess) err = cudaStreamSynchronize(s);
        } else {
            const uint64_t st = hash64(cfg.seed, (uint64_t) tid);
            const long long nb = (long long) nr[k] * (ncb_a + ncb_b);
            gen_q6k_kernel<<<(unsigned) ((nb + 127) / 128), 128, 0, s>>>(st, synth_scale(0.02), nr[k], gr[k], n_in_full / 256,
                                                                         ncb_a, cb_a, ncb_b, cb_b, row_blocks, out);
            if (err == cudaSuccess) err = cudaGetLastError();
        }
    }
    if (err != cudaSuccess) return;
    uint8_t* dst = group.w + (size_t) (row_off / 4) * (n_in / 1024) * kQ6Tile;
    const int rc = rk_pack_weights(RK_TYPE_Q6_K, scratch, dst, n_in, rows + rows1, s);
    if (rc != RK_OK && err == cudaSuccess) err = cudaErrorInvalidValue;
    tensors.push_back({tid, true, n_in, rows + rows1, group.w, (size_t) row_off, false});
}

int EngineImpl::build() {
    const rk_model_config& c = cfg;
    const int N = tp_size, g = tp_rank;
    H = c.n_embd, Vg = c.n_vocab;
    FF = c.n_ff / N, V = c.n_vocab / N, hk = c.ssm_h_k / N, hv = c.ssm_h_v / N, nh = c.n_head / N, nkv = c.n_head_kv / N;
    // more ranks than kv heads (8 ranks, 4 kv heads): each rank keeps the one kv head its q heads use,
    // computed on every rank that shares it (GQA group of nh q heads per kv head on the rank)
    if (nkv == 0) nkv = 1;
    kv0 = (g * nh) / (c.n_head / c.n_head_kv);
    const int hkg = c.ssm_h_k, hvg = c.ssm_h_v, S = kSsm;
    qkvzab_rows = 2 * hk * S + 2 * hv * S + 2 * hv;
    qkv3_rows = 2 * nh * kHdA + 2 * nkv * kHdA;
    max_in_rows = qkvzab_rows > qkv3_rows ? qkvzab_rows : qkv3_rows;
    // one flash-decode chunk length for the engine (attn_chunk_len); its chunks cover the whole cache
    chunk_len = attn_chunk_len(c.max_ctx);
    max_chunks = (c.max_ctx + chunk_len - 1) / chunk_len;
    max_out = c.max_ctx;
    if ((err = cudaSetDevice(dev)) != cudaSuccess) return RK_ECUDA;
    if ((err = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess) return RK_ECUDA;
    const size_t scratch_bytes = rk_weight_bytes(RK_TYPE_Q6_K, H, Vg) > rk_weight_bytes(RK_TYPE_Q6_K, c.n_ff, H)
                                     ? rk_weight_bytes(RK_TYPE_Q6_K, H, Vg)
                                     : rk_weight_bytes(RK_TYPE_Q6_K, H, 2 * c.n_ff);
    uint8_t* scratch = nullptr;
    if ((err = cudaMalloc(&scratch, scratch_bytes)) != cudaSuccess) return RK_ENOMEM;
    auto mat = [&](int n_in, int n_out) {
        Mat m;
        m.n_in = n_in;
        m.n_out = n_out;
        m.w = alloc<uint8_t>(rk_packed_bytes(RK_TYPE_Q6_K, n_in, n_out));
        return m;
    };
    auto norm = [&](int tid, int n) {
        float* p = alloc<float>((size_t) n);
        if (p) gen_f32(tid, p, (size_t) n, 0.02, 1.0, 0);
        return p;
    };
    // rows [grow0, grow0 + rows) of a tensor, all columns
    auto rows_of = [&](int tid, Mat& m, int row_off, int n_in, int grow0, int rows) {
        gen_q6k(tid, m, row_off, n_in, grow0, rows, 0, n_in / 256, 0, 0, scratch);
    };
    // this rank's column share [col0, col0 + cols) of every row (a row-parallel weight), in rows padded with
    // zero blocks to a whole number of 1024-value tiles (tp_in)
    auto cols_of = [&](int tid, Mat& m, int n_in_full, int n_out, int col0, int cols) {
        gen_q6k(tid, m, 0, n_in_full, 0, n_out, col0 / 256, cols / 256, 0, 0, scratch, tp_in(cols) / 256);
    };
    // globals: the embedding table is replicated; the lm_head is vocabulary-sharded
    tok_embd = alloc<uint8_t>(rk_weight_bytes(RK_TYPE_Q6_K, H, Vg));
    if (tok_embd && gg) {
        const GgufTensor* t = gg->find("token_embd.weight");
        if (!t || t->type != kGgmlQ6_K || t->ne[0] != H || t->ne[1] != Vg)
            src_fail(RK_EUNSUPPORTED, "token_embd.weight must be Q6_K [n_embd x n_vocab]");
        else if (err == cudaSuccess)
            err = cudaMemcpy(tok_embd, t->data, t->bytes, cudaMemcpyHostToDevice);
        tensors.push_back({T_TOK_EMBD, true, H, Vg, tok_embd, 0, true});
    } else if (tok_embd) {
        const long long nb = (long long) Vg * (H / 256);
        gen_q6k_kernel<<<(unsigned) ((nb + 127) / 128), 128, 0, s>>>(hash64(c.seed, T_TOK_EMBD), synth_scale(0.02), Vg,
                                                                     0, H / 256, H / 256, 0, 0, 0, H / 256, tok_embd);
        tensors.push_back({T_TOK_EMBD, true, H, Vg, tok_embd, 0, true});
    }
    out_norm = norm(T_OUT_NORM, H);
    lm_head = mat(H, V);
    if (lm_head.w) rows_of(T_OUTPUT, lm_head, 0, H, g * V, V);
    const int n_blocks = c.n_layer + (c.has_mtp ? 1 : 0);
    layers.resize(c.n_layer);
    for (int il = 0; il < n_blocks && err == cudaSuccess; ++il) {
        const bool is_draft = il == c.n_layer;
        Layer& L = is_draft ? draft : layers[il];
        L.gdn = !is_draft && ((il + 1) % c.attn_interval) != 0;
        L.attn_norm = norm(layer_tid(il, L_ATTN_NORM), H);
        L.post_norm = norm(layer_tid(il, L_POST_NORM), H);
        // FFN: up||gate column-parallel (this rank's FF rows of each), down row-parallel (its FF inputs)
        L.upgate = mat(H, 2 * FF);
        if (L.upgate.w) {
            rows_of(layer_tid(il, L_FFN_UP), L.upgate, 0, H, g * FF, FF);
            rows_of(layer_tid(il, L_FFN_GATE), L.upgate, FF, H, g * FF, FF);
        }
        L.down = mat(tp_in(FF), H);
        if (L.down.w) cols_of(layer_tid(il, L_FFN_DOWN), L.down, c.n_ff, H, g * FF, FF);
        if (L.gdn) {
            // this rank's k-heads [g*hk, (g+1)*hk) and the v-heads paired with them (h and h + hkg):
            // local layout [q | k | v (pairs a, b) | z | beta | alpha], a model with hk, hv heads
            const int qa = g * hk * S, n = hk * S;  // first row / rows of this rank's q (and k) block
            const int va = g * hk * S, vb = (hkg + g * hk) * S;
            L.in_proj = mat(H, qkvzab_rows);
            if (L.in_proj.w && N == 1) {  // whole tensors (one record each for rk_engine_read_tensor)
                rows_of(layer_tid(il, L_GDN_QKV), L.in_proj, 0, H, 0, 2 * hkg * S + hvg * S);
                rows_of(layer_tid(il, L_GDN_Z), L.in_proj, 2 * hkg * S + hvg * S, H, 0, hvg * S);
                rows_of(layer_tid(il, L_GDN_BETA), L.in_proj, 2 * hkg * S + 2 * hvg * S, H, 0, hvg);
                rows_of(layer_tid(il, L_GDN_ALPHA), L.in_proj, 2 * hkg * S + 2 * hvg * S + hvg, H, 0, hvg);
            } else if (L.in_proj.w) {
                const int tq = layer_tid(il, L_GDN_QKV);
                rows_of(tq, L.in_proj, 0, H, qa, n);                        // q
                rows_of(tq, L.in_proj, n, H, hkg * S + qa, n);              // k
                rows_of(tq, L.in_proj, 2 * n, H, 2 * hkg * S + va, n);      // v, first v-heads
                rows_of(tq, L.in_proj, 3 * n, H, 2 * hkg * S + vb, n);      // v, paired v-heads
                const int z0 = 2 * hk * S + hv * S;
                rows_of(layer_tid(il, L_GDN_Z), L.in_proj, z0, H, va, n);
                rows_of(layer_tid(il, L_GDN_Z), L.in_proj, z0 + n, H, vb, n);
                const int b0 = z0 + hv * S;
                // beta / alpha rows of both v-head ranges in one repack each (hk may be 2: a 4-row tile spans both)
                gen_q6k(layer_tid(il, L_GDN_BETA), L.in_proj, b0, H, g * hk, hk, 0, H / 256, 0, 0, scratch, 0,
                        hkg + g * hk, hk);
                gen_q6k(layer_tid(il, L_GDN_ALPHA), L.in_proj, b0 + hv, H, g * hk, hk, 0, H / 256, 0, 0, scratch, 0,
                        hkg + g * hk, hk);
            }
            // ssm_out row-parallel over this rank's v-head outputs (two column ranges)
            L.out_proj = mat(tp_in(hv * S), H);
            if (L.out_proj.w)
                gen_q6k(layer_tid(il, L_GDN_OUT), L.out_proj, 0, hvg * S, 0, H, va / 256, n / 256, vb / 256, n / 256,
                        scratch, tp_in(hv * S) / 256);
            const int C = 2 * hk * S + hv * S;
            std::vector<long long> chans;  // global conv channel of each local channel
            for (int i = 0; i < n; ++i) chans.push_back(qa + i);
            for (int i = 0; i < n; ++i) chans.push_back(hkg * S + qa + i);
            for (int j = 0; j < hv; ++j)
                for (int i = 0; i < S; ++i) chans.push_back(2 * hkg * S + (long long) gdn_vhead(j) * S + i);
            std::vector<long long> taps, heads;
            for (long long ch : chans)
                for (int t = 0; t < 4; ++t) taps.push_back(ch * 4 + t);
            for (int j = 0; j < hv; ++j) heads.push_back(gdn_vhead(j));
            L.conv_w = alloc<float>((size_t) C * 4);
            if (L.conv_w) gen_f32(layer_tid(il, L_GDN_CONV), L.conv_w, (size_t) C * 4, 0.3, 0.0, 0, N > 1 ? &taps : nullptr);
            L.ssm_a = alloc<float>(hv);
            if (L.ssm_a) gen_f32(layer_tid(il, L_GDN_A), L.ssm_a, hv, 0.5, 0.0, 1, N > 1 ? &heads : nullptr);
            L.dt = alloc<float>(hv);
            if (L.dt) gen_f32(layer_tid(il, L_GDN_DT), L.dt, hv, 0.5, 0.0, 0, N > 1 ? &heads : nullptr);
            L.ssm_norm = norm(layer_tid(il, L_GDN_NORM), S);
            L.state = alloc<float>((size_t) S * hv * S);
            L.snap = alloc<float>((size_t) S * hv * S);
            L.ring = alloc<float>((size_t) C * kRingSlots);
        } else {
            // this rank's q heads [g*nh, (g+1)*nh) and kv heads [kv0, kv0 + nkv)
            L.in_proj = mat(H, qkv3_rows);
            if (L.in_proj.w) {
                rows_of(layer_tid(il, L_ATT_Q), L.in_proj, 0, H, g * nh * 2 * kHdA, nh * 2 * kHdA);
                rows_of(layer_tid(il, L_ATT_K), L.in_proj, 2 * nh * kHdA, H, kv0 * kHdA, nkv * kHdA);
                rows_of(layer_tid(il, L_ATT_V), L.in_proj, 2 * nh * kHdA + nkv * kHdA, H, kv0 * kHdA, nkv * kHdA);
            }
            L.out_proj = mat(tp_in(nh * kHdA), H);  // wo row-parallel over this rank's heads
            if (L.out_proj.w) cols_of(layer_tid(il, L_ATT_O), L.out_proj, c.n_head * kHdA, H, g * nh * kHdA, nh * kHdA);
            L.q_norm = norm(layer_tid(il, L_ATT_QN), kHdA);
            L.k_norm = norm(layer_tid(il, L_ATT_KN), kHdA);
            L.kc = alloc<__half>((size_t) nkv * c.max_ctx * kHdA);
            L.vc = alloc<__half>((size_t) nkv * c.max_ctx * kHdA);
        }
    }
    if (c.has_mtp && err == cudaSuccess) {
        enorm = norm(T_ENORM, H);
        hnorm = norm(T_HNORM, H);
        shnorm = norm(T_SHNORM, H);
        eh_proj = mat(tp_in(2 * H / N), H);  // row-parallel over this rank's share of [emb | h]
        if (eh_proj.w) cols_of(T_EH_PROJ, eh_proj, 2 * H, H, g * 2 * H / N, 2 * H / N);
    }
    cudaStreamSynchronize(s);
    cudaFree(scratch);
    // rope table (double precision on the host, stored as float; YaRN when the factor is > 1)
    {
        std::vector<float> t;
        build_rope_table(c.n_rot, c.rope_base, c.rope_yarn_factor, c.rope_orig_ctx, c.max_ctx, t);
        rope = alloc<float>(t.size());
        if (rope && err == cudaSuccess)
            err = cudaMemcpyAsync(rope, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice, s);
        if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    }
    // activations (2 columns)
    const size_t K = kMaxCols;  // activations of up to kMaxCols columns (a prefill pass)
    x = alloc<float>(K * (size_t) H);
    xp = alloc<float>(K * (size_t) H / 4);
    proj = alloc<float>(K * (size_t) max_in_rows);
    ug = alloc<float>(K * 2 * (size_t) FF);
    // Q8_1 inputs of the row-parallel GEMVs: a padded GEMV (tp_in > the share) reads past each column into
    // the next one, or for the last column into the slack after them (zeros): finite blocks that meet
    // all-zero weight blocks
    const size_t slack = rk_q8_1_bytes(2048, 1);
    q8 = alloc<uint8_t>(K * rk_q8_1_bytes(hv * S, 1) + slack);
    gdn_o = alloc<float>(K * (size_t) hv * S);
    gdn_ss = alloc<float>(K * (size_t) hv * 4);
    gdn_cnt = alloc<unsigned>((size_t) hv);
    attn_scratch = alloc<float>((size_t) nh * K * max_chunks * (kHdA + 2));
    q8_ff = alloc<uint8_t>(K * rk_q8_1_bytes(FF, 1) + slack);
    q8_attn = alloc<uint8_t>(K * rk_q8_1_bytes(nh * kHdA, 1) + slack);
    swiglu_cnt = alloc<unsigned>((size_t) FF / 32);
    hsave = alloc<float>(2 * (size_t) H);
    hsave_p = alloc<float>(2 * (size_t) H / 4);
    logits = alloc<float>(2 * (size_t) V);
    dx = alloc<float>(2 * (size_t) H);
    dxp = alloc<float>(2 * (size_t) H / 4);
    eh_q8 = alloc<uint8_t>(2 * rk_q8_1_bytes(2 * H, 1));
    ctrl = alloc<Ctrl>(1);
    out = alloc<int>((size_t) max_out);
    force = alloc<int>((size_t) c.max_ctx + 2);
    if (force && err == cudaSuccess) err = cudaMemsetAsync(force, 0xff, sizeof(int) * ((size_t) c.max_ctx + 2), s);
    psync = alloc<PSync>(1);
    xdesc = alloc<XchDesc>(1);
    stage_slots = 4096;  // plus one slot after them for the emitted-count readback
    if (err == cudaSuccess) err = cudaMallocHost(&ctrl_stage, sizeof(Ctrl) * (stage_slots + 1));
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (src_rc != RK_OK) return src_rc;
    if (err == cudaErrorMemoryAllocation) return RK_ENOMEM;
    return err == cudaSuccess ? RK_OK : RK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------
// Step programs
// ---------------------------------------------------------------------------------------------------
MmvqParams EngineImpl::rms_params(const Mat& m, const float* x_, const float* w, const float* part, float* y,
                                  int y_stride) {
    MmvqParams p = {};
    p.w = m.w;
    p.n_in = m.n_in;
    p.n_out = m.n_out;
    p.prefetch_before_wait = 1;
    p.xa = x_;
    p.xb = w;
    p.pin = part;
    p.eps = cfg.eps;
    p.y = y;
    p.y_stride = y_stride;
    p.q8out = q8_ff;
    p.cnt = swiglu_cnt;
    return p;
}

// y = W . xq (+ res) with the 4-row partials (the reference's residual epilogue; y == res in place).
// x_cols: the width of one column of xq (its producer's stride) when the matrix is wider (tp_in padding)
MmvqParams EngineImpl::q8_params(const Mat& m, const uint8_t* xq, float* y, const float* res, float* part, int x_cols) {
    MmvqParams p = {};
    p.w = m.w;
    p.n_in = m.n_in;
    p.n_out = m.n_out;
    p.prefetch_before_wait = 1;
    p.xq = xq;
    p.y = y;
    p.y_stride = m.n_out;
    p.res = res;
    p.res_stride = m.n_out;
    p.pout = part;
    p.pout_stride = m.n_out / 4;
    if (x_cols > 0) p.xq_stride = (int) rk_q8_1_bytes(x_cols, 1);
    return p;
}

void EngineImpl::add_gemv(std::vector<POp>& v, int pro, int epi, const MmvqParams& p) {
    POp op = make_op(POP_GEMV);
    op.pro = pro;
    op.epi = epi;
    op.g = p;
    v.push_back(op);
}

// A row-parallel GEMV (ssm_out, wo, down, eh_proj): y = W . xq (+ res) with the 4-row partials; under
// tensor parallelism the ranks' partial sums are added over peer memory inside the op (EPI_XRES).
void EngineImpl::add_rowpar(std::vector<POp>& v, MmvqParams p) {
    if (tp_size == 1) {
        add_gemv(v, PRO_Q8, p.res != nullptr ? EPI_RES : EPI_STORE_P, p);
        return;
    }
    p.xch = xdesc;
    add_gemv(v, PRO_Q8, EPI_XRES, p);
}

// Tensor parallelism: after an lm_head over this rank's vocabulary shard, the global argmax.
void EngineImpl::add_xargmax(std::vector<POp>& v, int draft_flag) {
    if (tp_size == 1) return;
    POp op = make_op(POP_XARGMAX);
    op.draft = draft_flag;
    op.xa.xch = xdesc;
    v.push_back(op);
}

// FFN (src/qwythos.cpp:1011-1042): RMSNorm(post_norm)+Q8_1 -> up||gate with the SwiGLU+Q8_1 epilogue ->
// down + residual.
void EngineImpl::add_ffn(std::vector<POp>& v, const Layer& L, float* xres, float* part) {
    add_gemv(v, PRO_RMS, EPI_SWIGLU, rms_params(L.upgate, xres, L.post_norm, part, ug, 2 * FF));
    add_rowpar(v, q8_params(L.down, q8_ff, xres, xres, part, FF));
}

POp EngineImpl::attn_op(int kind, const Layer& L, int draft_flag) {
    POp op = make_op(kind);
    op.draft = draft_flag;
    AttnArgs& a = op.at;
    a.proj = proj;
    a.proj_stride = L.in_proj.n_out;
    a.qn = L.q_norm;
    a.kn = L.k_norm;
    a.rope = rope;
    a.n_rot = cfg.n_rot;
    a.n_head = nh;
    a.n_kv = nkv;
    a.max_ctx = cfg.max_ctx;
    a.max_chunks = max_chunks;
    a.chunk_len = chunk_len;
    a.eps = cfg.eps;
    a.scale = kAttnScale;
    a.kc = L.kc;
    a.vc = L.vc;
    a.part_o = attn_scratch;
    a.part_ml = attn_scratch + (size_t) nh * kMaxCols * max_chunks * kHdA;
    a.o = nullptr;
    a.q8 = q8_attn;
    return op;
}

void EngineImpl::add_trunk(std::vector<POp>& v, bool head) {
    POp e = make_op(POP_EMBED);
    e.em.emb = tok_embd;
    e.em.H = H;
    e.em.V = Vg;
    e.em.x = x;
    e.em.xp = xp;
    v.push_back(e);
    for (const Layer& L : layers) {
        add_gemv(v, PRO_RMS, EPI_STORE, rms_params(L.in_proj, x, L.attn_norm, xp, proj, L.in_proj.n_out));
        if (L.gdn) {
            POp g = make_op(POP_GDN);
            GdnArgs& a = g.gd;
            a.proj = proj;
            a.proj_stride = L.in_proj.n_out;
            a.ring = L.ring;
            a.conv_w = L.conv_w;
            a.dt = L.dt;
            a.ssm_a = L.ssm_a;
            a.gamma = L.ssm_norm;
            a.state = L.state;
            a.snap = L.snap;
            a.o_scr = gdn_o;
            a.ss_scr = gdn_ss;
            a.cnt = gdn_cnt;
            a.y = nullptr;
            a.q8 = q8;
            a.hk = hk;
            a.hv = hv;
            a.eps = cfg.eps;
            v.push_back(g);
            add_rowpar(v, q8_params(L.out_proj, q8, x, x, xp, hv * kSsm));
        } else {
            v.push_back(attn_op(POP_ATTN, L, 0));
            v.push_back(attn_op(POP_COMBINE, L, 0));
            add_rowpar(v, q8_params(L.out_proj, q8_attn, x, x, xp, nh * kHdA));
        }
        add_ffn(v, L, x, xp);
    }
    if (!head) return;  // a prefill pass: no logits
    // final norm + lm_head + argmax; the normed hidden and its partials feed the draft (src/qwythos.cpp:1234-1237)
    MmvqParams p = rms_params(lm_head, x, out_norm, xp, logits, V);
    p.xn_out = hsave;
    p.xn_part = hsave_p;
    p.amax = &ctrl->amax[0];
    p.row_off = tp_rank * V;
    add_gemv(v, PRO_RMS, EPI_ARGMAX, p);
    add_xargmax(v, 0);
}

// The MTP draft (draft_predict, src/qwythos.cpp:1316-1406): [enorm(emb) | hnorm(h)] -> eh_proj -> the
// nextn attention block -> (with_head) shnorm + the shared lm_head + argmax.
void EngineImpl::add_draft(std::vector<POp>& v, bool head, float* logits_out) {
    POp d = make_op(POP_DRAFT_PREP);
    d.draft = 1;
    d.dp.emb = tok_embd;
    d.dp.H = H;
    d.dp.V = Vg;
    d.dp.enorm = enorm;
    d.dp.hnorm = hnorm;
    d.dp.hsave = hsave;
    d.dp.hsave_p = hsave_p;
    d.dp.eps = cfg.eps;
    d.dp.eh_q8 = eh_q8;
    v.push_back(d);
    {  // no residual; under tensor parallelism this rank's share of the [emb | h] input columns
        MmvqParams p = q8_params(eh_proj, eh_q8 + (size_t) tp_rank * (2 * H / tp_size / 32) * 36, dx, nullptr, dxp);
        p.xq_stride = (int) rk_q8_1_bytes(2 * H, 1);
        add_rowpar(v, p);
    }
    const Layer& D = draft;
    add_gemv(v, PRO_RMS, EPI_STORE, rms_params(D.in_proj, dx, D.attn_norm, dxp, proj, D.in_proj.n_out));
    v.push_back(attn_op(POP_ATTN, D, 1));
    v.push_back(attn_op(POP_COMBINE, D, 1));
    add_rowpar(v, q8_params(D.out_proj, q8_attn, dx, dx, dxp, nh * kHdA));
    add_ffn(v, D, dx, dxp);
    if (head) {
        MmvqParams p = rms_params(lm_head, dx, shnorm, dxp, logits_out, V);
        p.amax = &ctrl->damax[0];
        p.row_off = tp_rank * V;
        add_gemv(v, PRO_RMS, EPI_ARGMAX, p);
        add_xargmax(v, 1);
    }
}

void EngineImpl::add_ctrl(std::vector<POp>& v, int kind) {
    POp c = make_op(POP_CTRL);
    c.ct.kind = kind;
    c.ct.out = out;
    c.ct.max_out = max_out;
    c.ct.force = force;
    c.ct.n_force = cfg.max_ctx + 2;
    v.push_back(c);
}

// The GEMVs of one trunk step only (rk_engine_probe_gemv), with their byte counts.
void EngineImpl::add_probe(std::vector<POp>& v, int nc) {
    double wb = 0, ab = 0;
    int n = 0;
    auto count = [&](const Mat& m, bool fp32_in, bool res) {
        const double w = (double) rk_weight_bytes(RK_TYPE_Q6_K, m.n_in, m.n_out);
        const double in = fp32_in ? (double) m.n_in * 4 : (double) rk_q8_1_bytes(m.n_in, 1);
        wb += w;
        ab += w + nc * (in + (double) m.n_out * 4 * (res ? 2 : 1));
        ++n;
    };
    for (const Layer& L : layers) {
        add_gemv(v, PRO_RMS, EPI_STORE, rms_params(L.in_proj, x, L.attn_norm, xp, proj, L.in_proj.n_out));
        count(L.in_proj, true, false);
        add_rowpar(v, q8_params(L.out_proj, L.gdn ? q8 : q8_attn, x, x, xp, L.gdn ? hv * kSsm : nh * kHdA));
        count(L.out_proj, false, true);
        add_ffn(v, L, x, xp);
        count(L.upgate, true, false);
        count(L.down, false, true);
    }
    MmvqParams p = rms_params(lm_head, x, out_norm, xp, logits, V);
    p.xn_out = hsave;
    p.xn_part = hsave_p;
    p.amax = &ctrl->amax[0];
    add_gemv(v, PRO_RMS, EPI_ARGMAX, p);
    count(lm_head, true, false);
    probe_weight_bytes[nc - 1] = wb;
    probe_algo_bytes[nc - 1] = ab;
    probe_gemvs = n;
}

// The persistent executor (RK_ENGINE_MODE=persistent), unless the device
// cannot hold one 512-thread CTA per SM with at least two ring slots per warp. The shared-memory region (staged activations or op
// scratch) and the ring depth are set per column count. Tuning knobs (like the reference's
// QWYTHOS_Q6ROWS sweep knob, src/native_mmvq.cu:3648-3651): RK_PERSIST_STAGES caps the ring depth,
// RK_PERSIST_L2PF_KB sets the per-CTA L2 prefetch of the next GEMV (KB, 0 = off).
int EngineImpl::setup_executor() {
    // One kernel per op replayed from CUDA graphs by default (measured faster than the persistent kernel on
    // B200: on one GPU 2.45 vs 2.66 ms per token and 3.50 vs 3.66 ms per MTP round; under 2-way tensor
    // parallelism 302 vs 230 tok/s with exact MTP). RK_ENGINE_MODE=graph|persistent overrides.
    const char* mode = std::getenv("RK_ENGINE_MODE");
    persistent = mode != nullptr && std::strcmp(mode, "persistent") == 0;
    int sms = 0, optin = 0;
    if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return RK_ECUDA;
    p_grid = sms;  // also the exchange's flag slots in graph mode (one GEMV CTA per SM)
    if (!persistent) return RK_OK;
    if ((err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
        return RK_ECUDA;
    // Two slots per warp (32 tiles, 107 KB in flight per SM) keep HBM busy; deeper rings only queue more
    // bulk copies ahead of the activation loads at op boundaries, which then wait longer.
    int cap = 2;
    if (const char* st = std::getenv("RK_PERSIST_STAGES")) {
        const int v = std::atoi(st);
        if (v >= 2 && v <= kMmvqMaxStages) cap = v;
    }
    p_l2pf = 256 * 1024;
    if (const char* pf = std::getenv("RK_PERSIST_L2PF_KB")) {
        const int v = std::atoi(pf);
        if (v >= 0 && v <= 4096) p_l2pf = v * 1024;
    }
    const int max_in = FF > 2 * H ? FF : 2 * H;
    for (int nc = 1; nc <= 4; nc *= 2) {
        const void* fn = nc == 1 ? (const void*) persistent_kernel<1>
                                 : nc == 2 ? (const void*) persistent_kernel<2> : (const void*) persistent_kernel<4>;
        cudaFuncAttributes fa = {};
        if ((err = cudaFuncGetAttributes(&fa, fn)) != cudaSuccess) return RK_ECUDA;
        size_t region = (size_t) nc * (max_in / 32) * 48;
        if (op_scratch_bytes(nc, H) > region) region = op_scratch_bytes(nc, H);
        region = (region + 127) & ~(size_t) 127;
        const long long budget = (long long) optin - (long long) fa.sharedSizeBytes;
        int stages = (int) ((budget - (long long) persistent_smem_bytes((int) region, 0)) / ((long long) kPWarps * kQ6Tile));
        if (stages > cap) stages = cap;
        if (stages < 2) {
            if (nc == 4) break;  // no 4-column prefill: prompts go one token per pass
            persistent = false;
            return RK_OK;
        }
        const size_t smem = persistent_smem_bytes((int) region, stages);
        if ((err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem)) != cudaSuccess)
            return RK_ECUDA;
        int occ = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kPWarps * 32, smem);
        if (occ < 1) {
            if (nc == 4) break;
            persistent = false;
            return RK_OK;
        }
        p_stages[col_slot(nc)] = stages;
        p_region[col_slot(nc)] = (int) region;
        p_smem[col_slot(nc)] = smem;
        if (nc == 4) prefill4 = true;
    }
    p_grid = sms;
    return RK_OK;
}

template <int NC>
cudaError_t EngineImpl::launch_op(const POp& op) {
    if (op.kind == POP_GEMV) {
        const MmvqParams& p = op.g;
        // 16 warps per CTA for the 2-column GEMVs and for the single-column residual GEMVs (7 units per CTA:
        // with 16 warps they run in warp pairs, mmvq_launch_w); 8 for the rest. Measured on one box against
        // 8 warps there: the no-MTP decode +1.1 %.
        const int w = NC == 2 || (NC == 1 && op.pro == PRO_Q8) ? 16 : kMmvqWarps;
        if (op.pro == PRO_RMS) {
            if (op.epi == EPI_STORE) return mmvq_launch<RK_TYPE_Q6_K, NC, PRO_RMS, EPI_STORE>(p, s, true, w);
            if (op.epi == EPI_SWIGLU) return mmvq_launch<RK_TYPE_Q6_K, NC, PRO_RMS, EPI_SWIGLU>(p, s, true, w);
            return mmvq_launch<RK_TYPE_Q6_K, NC, PRO_RMS, EPI_ARGMAX>(p, s, true, w);
        }
        if (op.epi == EPI_RES) return mmvq_launch<RK_TYPE_Q6_K, NC, PRO_Q8, EPI_RES>(p, s, true, w);
        if constexpr (NC <= 2)  // the exchange buffers hold two columns (tensor parallelism has no prefill program)
            if (op.epi == EPI_XRES) return mmvq_launch<RK_TYPE_Q6_K, NC, PRO_Q8, EPI_XRES>(p, s, true, w);
        return mmvq_launch<RK_TYPE_Q6_K, NC, PRO_Q8, EPI_STORE_P>(p, s, true, w);
    }
    if (op.kind == POP_XARGMAX) {
        if constexpr (NC <= 2) return launch_pdl(xargmax_kernel<NC>, dim3(1), dim3(32), 0, s, true, op, ctrl);
        return cudaErrorInvalidValue;
    }
    static int sms = 0;
    if (sms == 0 && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    if (op.kind == POP_ATTN) {
        // the chunk items (their count grows with the position): every resident CTA slot takes items in turn
        const size_t smem = ((size_t) attn_scratch_floats(NC) * 4 + 127) & ~(size_t) 127;
        static int per_sm[3] = {0, 0, 0};
        int& occ = per_sm[col_slot(NC)];
        if (occ == 0) {
            const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, attn_kernel<NC>, 256, smem);
            if (e != cudaSuccess) return e;
            if (occ < 1) occ = 1;
        }
        const int grid = std::min(op.at.max_chunks * op.at.n_kv, occ * sms);
        if (op.at.n_head == 2 * op.at.n_kv)  // 2 q heads per kv head (8-way tensor parallelism)
            return launch_pdl(attn_kernel<NC, 2>, dim3((unsigned) grid), dim3(256), smem, s, true, op, ctrl);
        return launch_pdl(attn_kernel<NC>, dim3((unsigned) grid), dim3(256), smem, s, true, op, ctrl);
    }
    if (op.kind == POP_COMBINE) {  // sm: 8 x 32 + 16 floats
        return launch_pdl(combine_kernel<NC>, dim3((unsigned) pop_items<NC>(op, 0)), dim3(256), (size_t) 2048, s, true, op,
                          ctrl);
    }
    if (op.kind == POP_GDN) {
        const size_t smem = ((size_t) gdn_scratch_floats(NC) * 4 + 127) & ~(size_t) 127;
        return launch_pdl(gdn_kernel<NC>, dim3((unsigned) pop_items<NC>(op, 0)), dim3(256), smem, s, true, op, ctrl);
    }
    // grid: the op's item count, which does not depend on the position
    const int grid = pop_items<NC>(op, 0);
    const size_t smem = op_scratch_bytes(NC, H);
    static bool attr_set[3] = {false, false, false};
    if (smem > 48 * 1024 && !attr_set[col_slot(NC)]) {
        const cudaError_t e = cudaFuncSetAttribute(op_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return e;
        attr_set[col_slot(NC)] = true;
    }
    return launch_pdl(op_kernel<NC>, dim3((unsigned) grid), dim3(256), smem, s, true, op, ctrl);
}

// Upload a program; in graph mode also capture its launches.
int EngineImpl::finalize(Program& P, int nc) {
    P.nc = nc;
    for (const POp& op : P.ops) {
        if (op.kind != POP_GEMV) continue;
        if (!gemv_combo_supported(op.pro, op.epi)) return RK_EINVAL;
        P.gemvs.push_back({op.g.w, op.g.n_out / 4, op.g.n_in / 1024});
    }
    if (P.gemvs.size() > (size_t) kMaxGemvOps) return RK_EINVAL;
    // the first GEMV after each op (wrapping to the program's first for the last ones)
    {
        int gi = (int) P.gemvs.size();
        for (int j = (int) P.ops.size() - 1; j >= 0; --j) {
            P.ops[j].next_gemv = gi < (int) P.gemvs.size() ? gi : (P.gemvs.empty() ? -1 : 0);
            if (P.ops[j].kind == POP_GEMV) --gi;
        }
    }
    P.dev = alloc<POp>(P.ops.size());
    P.gdev = alloc<GemvEnt>(P.gemvs.size() ? P.gemvs.size() : 1);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(P.dev, P.ops.data(), sizeof(POp) * P.ops.size(), cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess && !P.gemvs.empty())
        err = cudaMemcpyAsync(P.gdev, P.gemvs.data(), sizeof(GemvEnt) * P.gemvs.size(), cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return RK_ECUDA;
    if (persistent) {
        P.kernels = 1;
        return RK_OK;
    }
    cudaGraph_t g = nullptr;
    if ((err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal)) != cudaSuccess) return RK_ECUDA;
    int launches = 0;
    for (const POp& op : P.ops) {
        const cudaError_t e = nc == 1 ? launch_op<1>(op) : nc == 2 ? launch_op<2>(op) : launch_op<4>(op);
        if (e != cudaSuccess && err == cudaSuccess) err = e;
        ++launches;
    }
    const cudaError_t e2 = cudaStreamEndCapture(s, &g);
    if (err == cudaSuccess) err = e2;
    if (err == cudaSuccess) err = cudaGraphInstantiate(&P.graph, g, 0ull);
    if (g) cudaGraphDestroy(g);
    P.kernels = launches;
    return err == cudaSuccess ? RK_OK : RK_ECUDA;
}

// Enqueue one run of a program. Persistent: until > 0 repeats it while ctrl->n_emitted < until, at most
// max_iters times. Graph mode runs it once (the caller loops).
cudaError_t EngineImpl::run(const Program& P, int until, int max_iters, unsigned long long* trace) {
    if (!persistent) return cudaGraphLaunch(P.graph, s);
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned) p_grid);
    c.blockDim = dim3(kPWarps * 32);
    c.dynamicSmemBytes = p_smem[col_slot(P.nc)];
    c.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    c.attrs = at;
    c.numAttrs = 1;
    const POp* prog = P.dev;
    const GemvEnt* gt = P.gdev;
    const int nops = (int) P.ops.size(), ng = (int) P.gemvs.size();
    if (P.nc == 1)
        return cudaLaunchKernelEx(&c, persistent_kernel<1>, prog, nops, gt, ng, ctrl, psync, p_stages[0], p_region[0],
                                  p_l2pf, until, max_iters, trace);
    if (P.nc == 2)
        return cudaLaunchKernelEx(&c, persistent_kernel<2>, prog, nops, gt, ng, ctrl, psync, p_stages[1], p_region[1],
                                  p_l2pf, until, max_iters, trace);
    return cudaLaunchKernelEx(&c, persistent_kernel<4>, prog, nops, gt, ng, ctrl, psync, p_stages[2], p_region[2],
                              p_l2pf, until, max_iters, trace);
}

// Host writes of the control fields go through a ring of pinned slots so that queued copies never
// read a slot the host is rewriting (one slot per queued write; the ring is drained by syncs).
void EngineImpl::set_ctrl(const Ctrl& h) {
    Ctrl* slot = ctrl_stage + stage_next;
    stage_next = (stage_next + 1) % stage_slots;
    if (stage_next == 0) cudaStreamSynchronize(s);
    std::memcpy(slot, &h, sizeof(int) * kCtrlHostFields);
    const cudaError_t e = cudaMemcpyAsync(ctrl, slot, sizeof(int) * kCtrlHostFields, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess && err == cudaSuccess) err = e;
}

// Teacher-forced ingest of toks[0..n) at positions start.. (the reference's batched ingest,
// src/qwythos.cpp:2151-2502): 4-column passes of the trunk without the lm_head while four tokens remain
// (each column bitwise the single-token pass), then single-token passes. rollback0: the GDN rollback the
// first pass honours.
cudaError_t EngineImpl::ingest(const int* toks, int n, int start, int rollback0, int& launches) {
    cudaError_t ce = cudaSuccess;
    int i = 0;
    for (; prefill4 && n - i >= 4 && ce == cudaSuccess; i += 4) {
        Ctrl h = {};
        h.pos = start + i;
        for (int c = 0; c < 4; ++c) h.tok[c] = toks[i + c];
        h.rollback = i == 0 ? rollback0 : 0;
        set_ctrl(h);
        ce = run(progs[P_PREFILL], 0);
        ++launches;
    }
    for (; i < n && ce == cudaSuccess; ++i) {
        Ctrl h = {};
        h.pos = start + i;
        h.tok[0] = toks[i];
        h.rollback = i == 0 ? rollback0 : 0;
        set_ctrl(h);
        ce = run(progs[P_SINGLE], 0);
        ++launches;
    }
    return ce;
}

// The generation counters and the end-of-sequence id (-1: none) for the next run.
void EngineImpl::set_ctrl_eos(int eos_id) {
    Ctrl* slot = ctrl_stage + stage_next;
    stage_next = (stage_next + 1) % stage_slots;
    if (stage_next == 0) cudaStreamSynchronize(s);
    *slot = Ctrl{};
    slot->eos1 = eos_id + 1;
    const size_t off = offsetof(Ctrl, n_emitted), end = offsetof(Ctrl, pad);
    const cudaError_t e = cudaMemcpyAsync(reinterpret_cast<char*>(ctrl) + off, reinterpret_cast<char*>(slot) + off,
                                          end - off, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess && err == cudaSuccess) err = e;
}

// After a synchronized run: a persistent launch that gave up on a wait, or (graph mode, tensor parallelism)
// an exchange that gave up on a peer, leaves the sticky abort word.
int EngineImpl::check_abort(const char* what) {
    if (!persistent && tp_size == 1) return RK_OK;
    PSync h = {};
    if (cudaMemcpy(&h, psync, sizeof h, cudaMemcpyDeviceToHost) != cudaSuccess)
        return set_error(RK_ECUDA, "%s: reading the executor state failed", what);
    if (h.abort) return set_error(RK_ECUDA, "%s: a device wait timed out; the step was abandoned (rk_engine_reset clears it)", what);
    return RK_OK;
}

}  // namespace rk

using namespace rk;

struct rk_engine {
    EngineImpl impl;
};

extern "C" {

void rk_model_config_9b(rk_model_config* c, int max_ctx, uint64_t seed) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->n_layer = 32;
    c->n_embd = 4096;
    c->n_ff = 12288;
    c->n_vocab = 248320;
    c->ssm_h_k = 16;
    c->ssm_h_v = 32;
    c->n_head = 16;
    c->n_head_kv = 4;
    c->n_rot = 64;
    c->attn_interval = 4;
    c->has_mtp = 1;
    c->max_ctx = max_ctx;
    c->eps = 1e-6f;
    c->rope_base = 1e7;
    c->seed = seed;
    c->rope_yarn_factor = 1.0;
    c->rope_orig_ctx = 262144.0;
}

int rk_engine_create(const rk_model_config* cfg, int device, rk_engine** out) {
    return rk_engine_create_tp(cfg, device, 0, 1, out);
}

static int create_engine(const rk_model_config* cfg, int device, int tp_rank, int tp_size, const GgufFile* gg,
                         rk_engine** out) {
    const char* what = "rk_engine_create";
    if (!cfg || !out) return set_error(RK_EINVAL, "%s: null argument", what);
    const rk_model_config& c = *cfg;
    if (tp_size < 1 || tp_size > kMaxRanks || tp_rank < 0 || tp_rank >= tp_size)
        return set_error(RK_EINVAL, "%s: bad tensor-parallel rank / size", what);
    if (tp_size > 1) {
        // k-heads and q heads split evenly; kv heads split evenly, or each rank keeps the one its q heads use
        // (2 or 4 q heads per rank); every rank's share of a row-parallel input is a whole number of 256-value
        // Q6_K blocks (padded to 1024-value tiles with zero blocks)
        const int N = tp_size;
        const bool kv_split = c.n_head_kv % N == 0;
        const bool kv_repl = N % c.n_head_kv == 0 && c.n_head % N == 0 && (c.n_head / N == 2 || c.n_head / N == 4);
        if (c.ssm_h_k % (2 * N) || c.n_head % N || !(kv_split || kv_repl) || c.n_ff % (256 * N) ||
            (c.ssm_h_v * kSsm) % (256 * N) || (2 * c.n_embd) % (256 * N) || c.n_vocab % (4 * N))
            return set_error(RK_EUNSUPPORTED,
                             "%s: tensor parallelism over %d ranks needs an even number of k-heads per rank, q heads "
                             "divisible by the ranks, 2 or 4 "
                             "q heads per kv head on a rank, and every rank's row-parallel input a multiple of 256",
                             what, N);
    }
    if (c.n_layer < 1 || c.n_embd <= 0 || c.n_embd % 1024 || c.n_ff <= 0 || c.n_ff % 1024 || c.n_vocab <= 0 ||
        c.n_vocab % 4)
        return set_error(RK_EINVAL, "%s: n_embd and n_ff must be multiples of 1024, n_vocab of 4", what);
    if (c.ssm_h_k <= 0 || c.ssm_h_v != 2 * c.ssm_h_k || c.ssm_h_v * kSsm != c.n_embd)
        return set_error(RK_EINVAL, "%s: requires ssm_h_v == 2*ssm_h_k and ssm_h_v*128 == n_embd", what);
    if (c.n_head_kv <= 0 || c.n_head != 4 * c.n_head_kv || c.n_head * kHdA != c.n_embd)
        return set_error(RK_EINVAL, "%s: requires n_head == 4*n_head_kv and n_head*256 == n_embd", what);
    if (c.n_rot <= 0 || c.n_rot > kHdA || c.n_rot % 2 || c.attn_interval < 1 || c.max_ctx < 8 || !(c.eps > 0))
        return set_error(RK_EINVAL, "%s: bad n_rot / attn_interval / max_ctx / eps", what);
    rk_engine* e = new (std::nothrow) rk_engine;
    if (!e) return set_error(RK_ENOMEM, "%s: host allocation failed", what);
    e->impl.cfg = c;
    e->impl.dev = device;
    e->impl.tp_rank = tp_rank;
    e->impl.tp_size = tp_size;
    EngineImpl& E = e->impl;
    E.gg = gg;
    int rc = E.build();
    E.gg = nullptr;
    if (rc != RK_OK && E.src_rc != RK_OK) {
        const std::string msg = E.src_msg;
        delete e;
        return set_error(rc, "%s: %s", what, msg.c_str());
    }
    if (rc == RK_OK) rc = E.setup_executor();
    if (rc == RK_OK && tp_size > 1) {
        // this rank's exchange memory: partial words [2][8][2][H] | argmax flags [grid + 1][8] | keys [2][8][2]
        // | the graph executor's epoch per slot [grid + 1] (local only; the peers write words, flags and keys)
        E.xoff_flags = (size_t) 2 * kMaxRanks * 2 * E.H * sizeof(unsigned long long);
        E.xoff_keys = E.xoff_flags + (size_t) (E.p_grid + 1) * kMaxRanks * 8;
        E.xoff_ep = E.xoff_keys + (size_t) 2 * kMaxRanks * 2 * 8;
        E.xmem_bytes = E.xoff_ep + (size_t) (E.p_grid + 1) * 8;
        void* p = nullptr;
        if ((E.err = cudaMalloc(&p, E.xmem_bytes)) != cudaSuccess) rc = RK_ENOMEM;
        if (rc == RK_OK) {
            E.xmem = static_cast<uint8_t*>(p);
            E.allocs.push_back(p);
            E.err = cudaMemset(p, 0, E.xmem_bytes);
            if (E.err != cudaSuccess) rc = RK_ECUDA;
        }
    }
    if (rc == RK_OK) {
        E.add_trunk(E.progs[P_SINGLE].ops);
        E.add_ctrl(E.progs[P_SINGLE].ops, CTRL_SINGLE);
        rc = E.finalize(E.progs[P_SINGLE], 1);
    }
    if (rc == RK_OK) {
        E.add_trunk(E.progs[P_TRUNK2].ops);
        rc = E.finalize(E.progs[P_TRUNK2], 2);
    }
    if (!E.persistent) E.prefill4 = true;  // one kernel per op takes any column count
    if (tp_size > 1) E.prefill4 = false;   // the exchange buffers hold two columns
    if (rc == RK_OK && E.prefill4) {
        E.add_trunk(E.progs[P_PREFILL].ops, false);
        rc = E.finalize(E.progs[P_PREFILL], 4);
    }
    if (rc == RK_OK && c.has_mtp) {
        std::vector<POp>& r = E.progs[P_ROUND].ops;
        E.add_trunk(r);
        E.add_ctrl(r, CTRL_ACCEPT);
        E.add_draft(r, true);
        E.add_ctrl(r, CTRL_ROUND);
        rc = E.finalize(E.progs[P_ROUND], 2);
        if (rc == RK_OK) {
            E.add_draft(E.progs[P_DRAFT1].ops, true);
            E.add_ctrl(E.progs[P_DRAFT1].ops, CTRL_DRAFT1);
            rc = E.finalize(E.progs[P_DRAFT1], 1);
        }
        if (rc == RK_OK) {
            E.add_draft(E.progs[P_SEED].ops, false);
            rc = E.finalize(E.progs[P_SEED], 1);
        }
        if (rc == RK_OK) {  // rk_engine_draft_step: the draft with its logits kept
            E.add_draft(E.progs[P_DRAFTX].ops, true, E.logits);
            rc = E.finalize(E.progs[P_DRAFTX], 1);
        }
    }
    if (rc == RK_OK) {
        E.add_probe(E.progs[P_PROBE1].ops, 1);
        rc = E.finalize(E.progs[P_PROBE1], 1);
    }
    if (rc == RK_OK) {
        E.add_probe(E.progs[P_PROBE2].ops, 2);
        rc = E.finalize(E.progs[P_PROBE2], 2);
    }
    if (rc != RK_OK) {
        const cudaError_t ce = E.err;
        delete e;
        if (rc == RK_ENOMEM || ce == cudaErrorMemoryAllocation)
            return set_error(RK_ENOMEM, "%s: out of device memory", what);
        if (rc == RK_EINVAL) return set_error(RK_EINVAL, "%s: unsupported GEMV prologue/epilogue pair", what);
        return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    }
    *out = e;
    return RK_OK;
}

int rk_engine_create_tp(const rk_model_config* cfg, int device, int tp_rank, int tp_size, rk_engine** out) {
    return create_engine(cfg, device, tp_rank, tp_size, nullptr, out);
}

int rk_engine_create_gguf(const char* path, int device, int max_ctx, int tp_rank, int tp_size, rk_engine** out) {
    rk_model_config c;
    if (int rc = rk_gguf_model_config(path, max_ctx, &c)) return rc;
    GgufFile f;
    std::string err;
    if (!f.open(path, err)) return set_error(RK_EINVAL, "rk_engine_create_gguf: %s", err.c_str());
    return create_engine(&c, device, tp_rank, tp_size, &f, out);
}

size_t rk_tp_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int rk_engine_tp_export(rk_engine* e, void* handle, size_t bytes) {
    const char* what = "rk_engine_tp_export";
    if (!e || !handle || bytes < sizeof(cudaIpcMemHandle_t)) return set_error(RK_EINVAL, "%s: bad argument", what);
    EngineImpl& E = e->impl;
    if (E.tp_size < 2) return set_error(RK_EINVAL, "%s: the engine is not tensor-parallel", what);
    cudaIpcMemHandle_t h;
    const cudaError_t ce = cudaIpcGetMemHandle(&h, E.xmem);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    std::memcpy(handle, &h, sizeof h);
    return RK_OK;
}

int rk_engine_tp_connect(rk_engine* e, const void* handles, size_t bytes_per_rank) {
    const char* what = "rk_engine_tp_connect";
    if (!e || !handles || bytes_per_rank < sizeof(cudaIpcMemHandle_t)) return set_error(RK_EINVAL, "%s: bad argument", what);
    EngineImpl& E = e->impl;
    if (E.tp_size < 2) return set_error(RK_EINVAL, "%s: the engine is not tensor-parallel", what);
    if (E.tp_connected) return set_error(RK_EINVAL, "%s: already connected", what);
    if (cudaSetDevice(E.dev) != cudaSuccess) return set_error(RK_ECUDA, "%s: cudaSetDevice failed", what);
    XchDesc d = {};
    d.rank = E.tp_rank;
    d.n = E.tp_size;
    d.rows = E.H;
    d.slots = E.p_grid + 1;
    // RK_TP_WAIT_MS bounds every cross-rank wait (default 5000 ms; a test uses a short bound)
    const char* wenv = std::getenv("RK_TP_WAIT_MS");
    const long long wms = wenv ? std::atoll(wenv) : 0;
    d.wait_ns = wms > 0 ? (unsigned long long) wms * 1000000ull : kPeerSpinNs;
    E.peer_maps.assign(E.tp_size, nullptr);
    for (int q = 0; q < E.tp_size; ++q) {
        uint8_t* base = nullptr;
        if (q == E.tp_rank) {
            base = E.xmem;
        } else {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t) q * bytes_per_rank, sizeof h);
            void* p = nullptr;
            const cudaError_t ce = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (ce != cudaSuccess)
                return set_error(RK_ECUDA, "%s: opening rank %d's exchange memory: %s", what, q, cudaGetErrorString(ce));
            E.peer_maps[q] = p;
            base = static_cast<uint8_t*>(p);
        }
        d.buf[q] = reinterpret_cast<unsigned long long*>(base);
        d.flags[q] = reinterpret_cast<unsigned long long*>(base + E.xoff_flags);
        d.keys[q] = reinterpret_cast<unsigned long long*>(base + E.xoff_keys);
    }
    d.ep = reinterpret_cast<unsigned long long*>(E.xmem + E.xoff_ep);
    d.sync = E.psync;
    const cudaError_t ce = cudaMemcpy(E.xdesc, &d, sizeof d, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    E.tp_connected = true;
    return RK_OK;
}

// After a failed step (a peer that never signalled), the ranks' exchange epochs disagree; every rank clears
// its own exchange memory (partial words, flags, keys, epoch counters: the epochs restart from zero, so no
// word from before may stay) while none of the group's kernels runs.
int rk_engine_tp_resync(rk_engine* e) {
    const char* what = "rk_engine_tp_resync";
    if (!e) return set_error(RK_EINVAL, "%s: null engine", what);
    EngineImpl& E = e->impl;
    if (E.tp_size < 2 || !E.tp_connected) return set_error(RK_EINVAL, "%s: not a connected tensor-parallel engine", what);
    cudaError_t ce = cudaSetDevice(E.dev);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
    if (ce == cudaSuccess) ce = cudaMemset(E.xmem, 0, E.xmem_bytes);  // words, flags, keys and epochs
    if (ce == cudaSuccess) ce = cudaMemset(E.psync, 0, sizeof(PSync));
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    E.s_poisoned = true;  // the caches and states may be partly advanced: a reset comes next
    return RK_OK;
}

int rk_engine_destroy(rk_engine* e) {
    delete e;
    return RK_OK;
}

int rk_engine_mode(const rk_engine* e) { return e && e->impl.persistent ? RK_ENGINE_PERSISTENT : RK_ENGINE_GRAPH; }

int rk_engine_reset(rk_engine* e) {
    if (!e) return set_error(RK_EINVAL, "rk_engine_reset: null engine");
    EngineImpl& E = e->impl;
    cudaStreamSynchronize(E.s);
    const size_t hvs = (size_t) kSsm * E.hv * kSsm;
    const int C = 2 * E.hk * kSsm + E.hv * kSsm;
    auto clear = [&](Layer& L) {
        if (L.gdn) {
            cudaMemsetAsync(L.state, 0, hvs * 4, E.s);
            cudaMemsetAsync(L.snap, 0, hvs * 4, E.s);
            cudaMemsetAsync(L.ring, 0, (size_t) C * kRingSlots * 4, E.s);
        } else if (L.kc) {
            cudaMemsetAsync(L.kc, 0, (size_t) E.nkv * E.cfg.max_ctx * kHdA * 2, E.s);
            cudaMemsetAsync(L.vc, 0, (size_t) E.nkv * E.cfg.max_ctx * kHdA * 2, E.s);
        }
    };
    for (Layer& L : E.layers) clear(L);
    if (E.cfg.has_mtp) clear(E.draft);
    cudaMemsetAsync(E.ctrl, 0, sizeof(Ctrl), E.s);
    cudaMemsetAsync(E.swiglu_cnt, 0, sizeof(unsigned) * (size_t) E.FF / 32, E.s);
    cudaMemsetAsync(E.gdn_cnt, 0, sizeof(unsigned) * (size_t) E.hv, E.s);
    cudaMemsetAsync(E.psync, 0, offsetof(PSync, xepoch), E.s);  // the exchange epoch keeps counting
    const cudaError_t ce = cudaStreamSynchronize(E.s);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "rk_engine_reset: %s", cudaGetErrorString(ce));
    E.s_pos = 0;
    E.s_pending = -1;
    E.s_rollback = 0;
    E.s_primed = false;
    E.s_poisoned = false;
    return RK_OK;
}

int rk_engine_step(rk_engine* e, const int* tokens, int ncols, int pos, float* logits, int* argmax) {
    const char* what = "rk_engine_step";
    if (!e || !tokens) return set_error(RK_EINVAL, "%s: null argument", what);
    EngineImpl& E = e->impl;
    if (E.tp_size > 1 && !E.tp_connected) return set_error(RK_EINVAL, "%s: call rk_engine_tp_connect first", what);
    if (ncols < 1 || ncols > 2) return set_error(RK_EINVAL, "%s: ncols must be 1 or 2", what);
    if (pos < 0 || pos + ncols > E.cfg.max_ctx) return set_error(RK_ERANGE, "%s: position out of range", what);
    for (int c = 0; c < ncols; ++c)
        if (tokens[c] < 0 || tokens[c] >= E.Vg) return set_error(RK_ERANGE, "%s: token out of range", what);
    Ctrl h = {};
    h.pos = pos;
    h.tok[0] = tokens[0];
    h.tok[1] = ncols > 1 ? tokens[1] : 0;
    E.set_ctrl(h);
    cudaError_t ce = E.run(E.progs[ncols == 1 ? P_SINGLE : P_TRUNK2], 0);
    if (ce == cudaSuccess && logits)
        ce = cudaMemcpyAsync(logits, E.logits, sizeof(float) * (size_t) ncols * E.V, cudaMemcpyDeviceToHost, E.s);
    Ctrl back;
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&back, E.ctrl, sizeof(Ctrl), cudaMemcpyDeviceToHost, E.s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    if (int rc = E.check_abort(what)) return rc;
    if (argmax)
        for (int c = 0; c < ncols; ++c) argmax[c] = argmax_key_row(back.amax[c]);
    return RK_OK;
}

// The MTP draft alone (draft_predict, src/qwythos.cpp:1316-1406) at draft position pos with input token tok
// and the hidden of the last trunk pass's column 0 (or h = 0, the slot-0 seed), logits kept.
int rk_engine_draft_step(rk_engine* e, int tok, int pos, int h_zero, float* logits, int* argmax) {
    const char* what = "rk_engine_draft_step";
    if (!e) return set_error(RK_EINVAL, "%s: null engine", what);
    EngineImpl& E = e->impl;
    if (!E.cfg.has_mtp) return set_error(RK_EINVAL, "%s: model built without the MTP block", what);
    if (E.tp_size > 1 && !E.tp_connected) return set_error(RK_EINVAL, "%s: call rk_engine_tp_connect first", what);
    if (pos < 0 || pos + 1 > E.cfg.max_ctx) return set_error(RK_ERANGE, "%s: position out of range", what);
    if (tok < 0 || tok >= E.Vg) return set_error(RK_ERANGE, "%s: token out of range", what);
    cudaError_t ce = cudaSuccess;
    if (h_zero) {
        ce = cudaMemsetAsync(E.hsave, 0, sizeof(float) * E.H, E.s);
        if (ce == cudaSuccess) ce = cudaMemsetAsync(E.hsave_p, 0, sizeof(float) * E.H / 4, E.s);
    }
    Ctrl h = {};
    h.dpos = pos;
    h.dtok[0] = tok;
    if (ce == cudaSuccess) E.set_ctrl(h);
    if (ce == cudaSuccess) ce = E.run(E.progs[P_DRAFTX], 0);
    if (ce == cudaSuccess && logits)
        ce = cudaMemcpyAsync(logits, E.logits, sizeof(float) * (size_t) E.V, cudaMemcpyDeviceToHost, E.s);
    Ctrl back;
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&back, E.ctrl, sizeof(Ctrl), cudaMemcpyDeviceToHost, E.s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    if (int rc = E.check_abort(what)) return rc;
    if (argmax) *argmax = argmax_key_row(back.damax[0]);
    return RK_OK;
}

int rk_engine_force_candidates(rk_engine* e, const int* tokens, int n) {
    const char* what = "rk_engine_force_candidates";
    if (!e || (n > 0 && !tokens)) return set_error(RK_EINVAL, "%s: null argument", what);
    EngineImpl& E = e->impl;
    const int cap = E.cfg.max_ctx + 2;
    if (n < 0 || n > cap) return set_error(RK_EINVAL, "%s: n must be in [0, max_ctx + 2]", what);
    for (int i = 0; i < n; ++i)
        if (tokens[i] < -1 || tokens[i] >= E.Vg) return set_error(RK_ERANGE, "%s: token out of range", what);
    cudaError_t ce = cudaStreamSynchronize(E.s);
    if (ce == cudaSuccess) ce = cudaMemset(E.force, 0xff, sizeof(int) * (size_t) cap);
    if (ce == cudaSuccess && n > 0) ce = cudaMemcpy(E.force, tokens, sizeof(int) * (size_t) n, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    return RK_OK;
}

int rk_engine_generate(rk_engine* e, const int* prompt, int n_prompt, int n_gen, int use_mtp, int* out_ids,
                       rk_gen_stats* stats) {
    const char* what = "rk_engine_generate";
    if (!e || !prompt || !out_ids) return set_error(RK_EINVAL, "%s: null argument", what);
    EngineImpl& E = e->impl;
    if (E.tp_size > 1 && !E.tp_connected) return set_error(RK_EINVAL, "%s: call rk_engine_tp_connect first", what);
    if (n_prompt < 1 || n_gen < 1) return set_error(RK_EINVAL, "%s: needs n_prompt >= 1 and n_gen >= 1", what);
    if (n_prompt + n_gen + 2 > E.cfg.max_ctx) return set_error(RK_ERANGE, "%s: prompt + generation exceed max_ctx", what);
    if (use_mtp && !E.cfg.has_mtp) return set_error(RK_EINVAL, "%s: model built without the MTP block", what);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= E.Vg) return set_error(RK_ERANGE, "%s: prompt token out of range", what);
    int rc = rk_engine_reset(e);
    if (rc) return rc;
    cudaEvent_t ev[3];
    for (auto& v : ev) cudaEventCreate(&v);
    int launches = 0;
    cudaError_t ce = cudaSuccess;
    int* pinned = reinterpret_cast<int*>(E.ctrl_stage + E.stage_slots);
    auto read_emitted = [&]() {
        if (ce == cudaSuccess) ce = cudaMemcpyAsync(pinned, &E.ctrl->n_emitted, sizeof(int), cudaMemcpyDeviceToHost, E.s);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
        return ce == cudaSuccess ? *pinned : -1;
    };
    // prefill: positions 0..P-2, teacher forced (4-column passes, then single tokens)
    cudaEventRecord(ev[0], E.s);
    ce = E.ingest(prompt, n_prompt - 1, 0, 0, launches);
    if (use_mtp && ce == cudaSuccess) {
        // seed the draft cache slot 0 with (emb(prompt[0]), h = 0) (src/qwythos.cpp:2955-2958)
        cudaMemsetAsync(E.hsave, 0, sizeof(float) * E.H, E.s);
        cudaMemsetAsync(E.hsave_p, 0, sizeof(float) * E.H / 4, E.s);
        Ctrl h = {};
        h.dpos = 0;
        h.dtok[0] = prompt[0];
        E.set_ctrl(h);
        ce = E.run(E.progs[P_SEED], 0);
        ++launches;
    }
    E.set_ctrl_eos(-1);  // n_emitted, steps, accepted, singles, bad cleared; no end-of-sequence stop
    cudaEventRecord(ev[1], E.s);
    // the seed pass at position P-1 produces the first generated token
    Ctrl h = {};
    h.pos = n_prompt - 1;
    h.tok[0] = prompt[n_prompt - 1];
    E.set_ctrl(h);
    if (!use_mtp) {
        if (E.persistent) {
            if (ce == cudaSuccess) ce = E.run(E.progs[P_SINGLE], n_gen, n_gen);  // the whole generation
            ++launches;
        } else {
            for (int i = 0; i < n_gen && ce == cudaSuccess; ++i) {
                ce = E.run(E.progs[P_SINGLE], 0);
                ++launches;
            }
        }
    } else if (ce == cudaSuccess) {
        ce = E.run(E.progs[P_SINGLE], 0);
        ++launches;
        // first candidate: draft at (emb(first token), hidden of P-1)
        if (ce == cudaSuccess) ce = E.run(E.progs[P_DRAFT1], 0);
        ++launches;
        int emitted = 1;
        if (E.persistent) {
            if (emitted < n_gen - 1 && ce == cudaSuccess) {
                ce = E.run(E.progs[P_ROUND], n_gen - 1, n_gen);  // rounds until one token is left at most
                ++launches;
                emitted = read_emitted();
            }
            if (emitted >= 0 && emitted < n_gen && ce == cudaSuccess) {
                ce = E.run(E.progs[P_SINGLE], 0);
                ++launches;
            }
        } else {
            // A round emits one or two tokens, so (n_gen - emitted) / 2 rounds can be queued without reading
            // the count back (no end-of-sequence stop here): ~log2(n_gen) host round trips per generation
            // instead of one per round.
            while (ce == cudaSuccess && emitted >= 0 && emitted < n_gen) {
                const int rounds = emitted >= n_gen - 1 ? 0 : (n_gen - emitted) / 2;
                for (int k = 0; k < rounds && ce == cudaSuccess; ++k) ce = E.run(E.progs[P_ROUND], 0);
                if (rounds == 0 && ce == cudaSuccess) ce = E.run(E.progs[P_SINGLE], 0);
                launches += rounds > 0 ? rounds : 1;
                emitted = read_emitted();
            }
        }
    }
    cudaEventRecord(ev[2], E.s);
    Ctrl back = {};
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&back, E.ctrl, sizeof(Ctrl), cudaMemcpyDeviceToHost, E.s);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(out_ids, E.out, sizeof(int) * (size_t) n_gen, cudaMemcpyDeviceToHost, E.s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
    float pre = 0.0f, gen = 0.0f;
    if (ce == cudaSuccess) {
        cudaEventElapsedTime(&pre, ev[0], ev[1]);
        cudaEventElapsedTime(&gen, ev[1], ev[2]);
    }
    for (auto& v : ev) cudaEventDestroy(v);
    E.s_poisoned = true;  // until the generation is known to be complete
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    if (int rc2 = E.check_abort(what)) return rc2;
    if (back.bad) return set_error(RK_ERANGE, "%s: a token outside the vocabulary reached the device", what);
    if (back.n_emitted < n_gen) return set_error(RK_ECUDA, "%s: generation stopped early (%d of %d)", what, back.n_emitted, n_gen);
    E.s_poisoned = false;
    E.s_pos = back.pos;  // a session may continue the generation (its last token is pending)
    E.s_pending = back.tok[0];
    E.s_rollback = back.rollback;
    E.s_primed = use_mtp != 0;
    if (stats) {
        stats->prefill_ms = pre;
        stats->gen_ms = gen;
        stats->n_gen = n_gen;
        stats->mtp_steps = back.steps;
        stats->mtp_accepted = back.accepted;
        stats->single_steps = back.singles;
        stats->graph_launches = launches;
        stats->kernels_per_single_step = E.progs[P_SINGLE].kernels;
        stats->kernels_per_round = E.progs[P_ROUND].kernels;
    }
    return RK_OK;
}

int rk_engine_session_reset(rk_engine* e) { return rk_engine_reset(e); }

// Config 5 at a long context without a long prompt: the caches of a context of n_pos tokens filled with
// seeded synthetic values (fp16 K and V ~ N(0, 1) in every attention layer and the draft layer, the
// configuration's KV distribution; GDN states ~ N(0, 0.01), conv rings 0), and the session placed after
// them, so the next run decodes at positions n_pos, n_pos + 1, ...
int rk_engine_session_fill(rk_engine* e, int n_pos, unsigned long long seed) {
    const char* what = "rk_engine_session_fill";
    if (!e) return set_error(RK_EINVAL, "%s: null engine", what);
    EngineImpl& E = e->impl;
    if (n_pos < 1 || n_pos + 8 > E.cfg.max_ctx) return set_error(RK_ERANGE, "%s: n_pos must leave room in max_ctx", what);
    if (int rc = rk_engine_reset(e)) return rc;
    const float sk = synth_scale(1.0), ss = synth_scale(0.01);
    int li = 0;
    auto fill = [&](Layer& L) {
        const uint64_t sd = hash64(seed, (uint64_t) (1000 + li++));
        if (L.kc) {
            fill_kv_kernel<<<4 * 148, 256, 0, E.s>>>(L.kc, E.nkv, E.cfg.max_ctx, n_pos, hash64(sd, 1), sk);
            fill_kv_kernel<<<4 * 148, 256, 0, E.s>>>(L.vc, E.nkv, E.cfg.max_ctx, n_pos, hash64(sd, 2), sk);
        }
        if (L.gdn && L.state)
            fill_float_kernel<<<4 * 148, 256, 0, E.s>>>(L.state, (long long) kSsm * E.hv * kSsm, hash64(sd, 3), ss);
    };
    for (Layer& L : E.layers) fill(L);
    if (E.cfg.has_mtp) fill(E.draft);
    const cudaError_t ce = cudaStreamSynchronize(E.s);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    E.s_pos = n_pos;
    E.s_pending = -1;
    E.s_rollback = 0;
    E.s_primed = true;
    return RK_OK;
}

int rk_engine_session_pos(const rk_engine* e) { return e ? e->impl.s_pos + (e->impl.s_pending >= 0 ? 1 : 0) : -1; }

// The serve loop's run (src/qwythos.cpp:2650-2812): the pending token of the previous run and then
// tokens[0..n) are ingested at the session position (every one but the last teacher-forced, the last as
// the seed pass), then up to n_gen tokens are generated greedily, stopping after eos_id. Afterwards every
// emitted token except a final eos_id is part of the context: the last one stays pending and is ingested
// first by the next run. The first run after a reset seeds the draft slot 0 when use_mtp.
int rk_engine_session_run(rk_engine* e, const int* tokens, int n_tokens, int n_gen, int use_mtp, int eos_id,
                          int* out_ids, int* n_out, float* first_logits, rk_gen_stats* stats) {
    const char* what = "rk_engine_session_run";
    if (!e || !out_ids || !n_out || (n_tokens > 0 && !tokens)) return set_error(RK_EINVAL, "%s: null argument", what);
    EngineImpl& E = e->impl;
    *n_out = 0;
    if (E.tp_size > 1 && !E.tp_connected) return set_error(RK_EINVAL, "%s: call rk_engine_tp_connect first", what);
    if (n_tokens < 0 || n_gen < 1) return set_error(RK_EINVAL, "%s: needs n_tokens >= 0 and n_gen >= 1", what);
    if (use_mtp && !E.cfg.has_mtp) return set_error(RK_EINVAL, "%s: model built without the MTP block", what);
    if (eos_id < -1 || eos_id >= E.Vg) return set_error(RK_ERANGE, "%s: eos_id out of range", what);
    if (E.s_poisoned)
        return set_error(RK_ECUDA, "%s: a previous run failed part way; call rk_engine_session_reset", what);
    std::vector<int> list;
    if (E.s_pending >= 0) list.push_back(E.s_pending);
    for (int i = 0; i < n_tokens; ++i) {
        if (tokens[i] < 0 || tokens[i] >= E.Vg) return set_error(RK_ERANGE, "%s: token out of range", what);
        list.push_back(tokens[i]);
    }
    if (list.empty()) return set_error(RK_EINVAL, "%s: nothing to ingest (no tokens and no pending token)", what);
    const int L = (int) list.size(), start = E.s_pos;
    if ((long long) start + L + n_gen + 2 > E.cfg.max_ctx)
        return set_error(RK_ERANGE, "%s: context full (position %d + %d tokens + %d generated); reset the session",
                         what, start, L, n_gen);
    cudaEvent_t ev[3];
    for (auto& v : ev) cudaEventCreate(&v);
    int launches = 0;
    cudaError_t ce = cudaSuccess;
    int* pinned = reinterpret_cast<int*>(E.ctrl_stage + E.stage_slots);
    auto read_ctrl = [&](Ctrl& h) {
        if (ce == cudaSuccess) ce = cudaMemcpyAsync(pinned, E.ctrl, sizeof(Ctrl), cudaMemcpyDeviceToHost, E.s);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
        if (ce == cudaSuccess) std::memcpy(&h, pinned, sizeof(Ctrl));
    };
    cudaEventRecord(ev[0], E.s);
    ce = E.ingest(list.data(), L - 1, start, E.s_rollback, launches);  // teacher-forced ingest
    if (use_mtp && !E.s_primed && ce == cudaSuccess) {  // draft slot 0: (emb(first token), h = 0)
        cudaMemsetAsync(E.hsave, 0, sizeof(float) * E.H, E.s);
        cudaMemsetAsync(E.hsave_p, 0, sizeof(float) * E.H / 4, E.s);
        Ctrl h = {};
        h.dpos = start;
        h.dtok[0] = list[0];
        E.set_ctrl(h);
        ce = E.run(E.progs[P_SEED], 0);
        ++launches;
    }
    if (use_mtp) E.s_primed = true;  // the draft's cache is kept only by MTP runs
    E.set_ctrl_eos(eos_id);
    cudaEventRecord(ev[1], E.s);
    {  // the seed pass: the last ingested token, the first generated one
        Ctrl h = {};
        h.pos = start + L - 1;
        h.tok[0] = list[(size_t) L - 1];
        h.rollback = L == 1 ? E.s_rollback : 0;
        E.set_ctrl(h);
        if (ce == cudaSuccess) ce = E.run(E.progs[P_SINGLE], 0);
        ++launches;
    }
    if (first_logits && ce == cudaSuccess)
        ce = cudaMemcpyAsync(first_logits, E.logits, sizeof(float) * (size_t) E.V, cudaMemcpyDeviceToHost, E.s);
    Ctrl back = {};
    read_ctrl(back);
    if (!use_mtp) {
        if (E.persistent && !back.stop && back.n_emitted < n_gen && ce == cudaSuccess) {
            ce = E.run(E.progs[P_SINGLE], n_gen, n_gen);
            ++launches;
            read_ctrl(back);
        }
        // graph mode: without an end-of-sequence id nothing stops a generation early, so the remaining
        // passes are queued at once (one host round trip); with one, the count is read after every pass
        while (!E.persistent && !back.stop && back.n_emitted < n_gen && ce == cudaSuccess) {
            const int passes = eos_id < 0 ? n_gen - back.n_emitted : 1;
            for (int k = 0; k < passes && ce == cudaSuccess; ++k) ce = E.run(E.progs[P_SINGLE], 0);
            launches += passes;
            read_ctrl(back);
        }
    } else if (!back.stop && back.n_emitted < n_gen && ce == cudaSuccess) {
        ce = E.run(E.progs[P_DRAFT1], 0);  // first candidate
        ++launches;
        if (E.persistent) {
            if (n_gen - 1 > 1 && ce == cudaSuccess) {
                ce = E.run(E.progs[P_ROUND], n_gen - 1, n_gen);
                ++launches;
            }
            read_ctrl(back);
        } else {
            // a round emits one or two tokens: without an end-of-sequence id (n_gen - emitted) / 2 rounds are
            // queued before the count is read back
            while (!back.stop && back.n_emitted < n_gen - 1 && ce == cudaSuccess) {
                const int rounds = eos_id < 0 ? (n_gen - back.n_emitted) / 2 : 1;
                for (int k = 0; k < rounds && ce == cudaSuccess; ++k) ce = E.run(E.progs[P_ROUND], 0);
                launches += rounds;
                read_ctrl(back);
            }
        }
        if (!back.stop && back.n_emitted < n_gen && ce == cudaSuccess) {
            ce = E.run(E.progs[P_SINGLE], 0);
            ++launches;
            read_ctrl(back);
        }
    }
    cudaEventRecord(ev[2], E.s);
    if (ce == cudaSuccess && back.n_emitted > 0)
        ce = cudaMemcpyAsync(out_ids, E.out, sizeof(int) * (size_t) std::min(back.n_emitted, n_gen), cudaMemcpyDeviceToHost, E.s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
    float pre = 0.0f, gen = 0.0f;
    if (ce == cudaSuccess) {
        cudaEventElapsedTime(&pre, ev[0], ev[1]);
        cudaEventElapsedTime(&gen, ev[1], ev[2]);
    }
    for (auto& v : ev) cudaEventDestroy(v);
    if (ce != cudaSuccess) {
        E.s_poisoned = true;
        return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    }
    if (int rc = E.check_abort(what)) {
        E.s_poisoned = true;
        return rc;
    }
    if (back.bad) {
        E.s_poisoned = true;
        return set_error(RK_ERANGE, "%s: a token outside the vocabulary reached the device", what);
    }
    *n_out = std::min(back.n_emitted, n_gen);
    E.s_pos = back.pos;
    E.s_pending = back.stop ? -1 : back.tok[0];
    E.s_rollback = back.rollback;
    if (stats) {
        stats->prefill_ms = pre;
        stats->gen_ms = gen;
        stats->n_gen = *n_out;
        stats->mtp_steps = back.steps;
        stats->mtp_accepted = back.accepted;
        stats->single_steps = back.singles;
        stats->graph_launches = launches;
        stats->kernels_per_single_step = E.progs[P_SINGLE].kernels;
        stats->kernels_per_round = E.progs[P_ROUND].kernels;
    }
    return RK_OK;
}

size_t rk_engine_read_tensor(rk_engine* e, int tid, void* host, size_t bytes) {
    if (!e) return 0;
    EngineImpl& E = e->impl;
    for (const TensorRec& t : E.tensors) {
        if (t.tid != tid) continue;
        if (!t.q6k) {
            const size_t need = (size_t) t.n_in * sizeof(float);
            if (!host || bytes == 0) return need;
            if (bytes < need) return 0;
            return cudaMemcpy(host, t.dev, need, cudaMemcpyDeviceToHost) == cudaSuccess ? need : 0;
        }
        const size_t need = rk_weight_bytes(RK_TYPE_Q6_K, t.n_in, t.n_out);
        if (!host || bytes == 0) return need;
        if (bytes < need) return 0;
        if (t.raw) return cudaMemcpy(host, t.dev, need, cudaMemcpyDeviceToHost) == cudaSuccess ? need : 0;
        void* tmp = nullptr;
        if (cudaMalloc(&tmp, need) != cudaSuccess) return 0;
        const uint8_t* src = static_cast<const uint8_t*>(t.dev) + (t.row_off / 4) * (size_t) (t.n_in / 1024) * kQ6Tile;
        int rc = rk_unpack_weights(RK_TYPE_Q6_K, src, tmp, t.n_in, t.n_out, E.s);
        cudaError_t ce = rc == RK_OK ? cudaStreamSynchronize(E.s) : cudaErrorInvalidValue;
        if (ce == cudaSuccess) ce = cudaMemcpy(host, tmp, need, cudaMemcpyDeviceToHost);
        cudaFree(tmp);
        return ce == cudaSuccess ? need : 0;
    }
    return 0;
}

int rk_engine_probe_gemv(rk_engine* e, int ncols, int iters, rk_probe_result* out) {
    const char* what = "rk_engine_probe_gemv";
    if (!e || !out) return set_error(RK_EINVAL, "%s: null argument", what);
    if (ncols < 1 || ncols > 2 || iters < 1) return set_error(RK_EINVAL, "%s: ncols 1..2, iters >= 1", what);
    EngineImpl& E = e->impl;
    if (E.tp_size > 1 && !E.tp_connected) return set_error(RK_EINVAL, "%s: call rk_engine_tp_connect first", what);
    const Program& P = E.progs[ncols == 1 ? P_PROBE1 : P_PROBE2];
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaError_t ce = E.run(P, 0);  // warm-up
    if (ce == cudaSuccess) ce = cudaEventRecord(a, E.s);
    for (int i = 0; i < iters && ce == cudaSuccess; ++i) ce = E.run(P, 0);
    if (ce == cudaSuccess) ce = cudaEventRecord(b, E.s);
    if (ce == cudaSuccess) ce = cudaEventSynchronize(b);
    float ms = 0.0f;
    if (ce == cudaSuccess) cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    if (int rc = E.check_abort(what)) return rc;
    out->ms = ms;
    out->launches = E.probe_gemvs;
    out->weight_bytes = E.probe_weight_bytes[ncols - 1];
    out->algo_bytes = E.probe_algo_bytes[ncols - 1];
    return RK_OK;
}

int rk_engine_trace(rk_engine* e, int program, double* stamps_us, int* kinds, int max_ops, double* cta_us,
                    int max_ctas) {
    const char* what = "rk_engine_trace";
    if (!e || !stamps_us || !kinds) return set_error(RK_EINVAL, "%s: null argument", what);
    EngineImpl& E = e->impl;
    if (!E.persistent) return set_error(RK_EUNSUPPORTED, "%s: needs the persistent executor", what);
    if (E.tp_size > 1 && !E.tp_connected) return set_error(RK_EINVAL, "%s: call rk_engine_tp_connect first", what);
    static const int ids[] = {P_SINGLE, P_ROUND, P_PROBE1, P_PROBE2, P_TRUNK2};
    if (program < 0 || program > 4) return set_error(RK_EINVAL, "%s: program must be 0..4", what);
    const Program& P = E.progs[ids[program]];
    const int nops = (int) P.ops.size();
    if (nops == 0) return set_error(RK_EINVAL, "%s: the engine has no such program (built without MTP)", what);
    if (program == 0 || program == 1 || program == 4) {
        Ctrl h = {};
        cudaMemcpy(&h, E.ctrl, sizeof h, cudaMemcpyDeviceToHost);
        if (h.pos < 0 || h.pos + 2 >= E.cfg.max_ctx) return set_error(RK_ERANGE, "%s: no room left in the cache", what);
    }
    const size_t entries = (size_t) 4 * nops + (size_t) 2 * nops * E.p_grid;
    unsigned long long* dt = nullptr;
    if (cudaMalloc(&dt, sizeof(unsigned long long) * entries) != cudaSuccess)
        return set_error(RK_ENOMEM, "%s: out of device memory", what);
    cudaError_t ce = cudaMemsetAsync(dt, 0, sizeof(unsigned long long) * entries, E.s);
    if (ce == cudaSuccess) ce = E.run(P, 0, 1, dt);
    std::vector<unsigned long long> h(entries);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(h.data(), dt, h.size() * 8, cudaMemcpyDeviceToHost, E.s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E.s);
    cudaFree(dt);
    if (ce != cudaSuccess) return set_error(RK_ECUDA, "%s: %s", what, cudaGetErrorString(ce));
    if (int rc = E.check_abort(what)) return rc;
    const int n = nops < max_ops ? nops : max_ops;
    for (int j = 0; j < n; ++j) {
        for (int k = 0; k < 4; ++k) stamps_us[4 * j + k] = (double) (h[4 * (size_t) j + k] - h[0]) * 1e-3;
        kinds[j] = P.ops[j].kind == POP_GEMV ? 100 + P.ops[j].epi : P.ops[j].kind;
        if (cta_us)
            for (int b = 0; b < max_ctas; ++b)
                for (int k = 0; k < 2; ++k) {
                    const size_t src = (size_t) 4 * nops + ((size_t) j * E.p_grid + b) * 2 + k;
                    cta_us[((size_t) j * max_ctas + b) * 2 + k] =
                        b < E.p_grid ? (double) (h[src] - h[0]) * 1e-3 : -1.0;
                }
    }
    return nops;
}

size_t rk_engine_device_bytes(const rk_engine* e) { return e ? e->impl.bytes : 0; }

}  // extern "C"
