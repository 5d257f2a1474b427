/*
 * rapier_b200.h — C-ABI of the B200-native (sm_100a) decode hot path for the qwen35 hybrid architecture.
 *
 * Operator surface: extern "C" twins of the reference engine's strata::kernels calls and of the
 * in-file kernels of src/qwythos.cpp (paths inside jollyroger1480/rapier). Conventions:
 *   - device pointers only; `stream` is a cudaStream_t passed as void* (must be non-null, as the
 *     reference's native_mmvq requires, src/native_mmvq.cu:2323-2325);
 *   - work is enqueued asynchronously, nothing synchronizes, nothing allocates, so every call can be
 *     captured into a CUDA graph;
 *   - every entry validates on the host and returns RK_OK (0) or a negative RK_E* code; the message of
 *     the last failure on the calling thread is rk_last_error(). Where the reference throws
 *     std::invalid_argument (src/native_mmvq.cu:2312-2331) or calls exit(1) (src/fused_gdn.cu:169-176),
 *     this returns RK_EINVAL;
 *   - weight type ids are ggml's: RK_TYPE_Q6_K = 14, RK_TYPE_Q5_K = 13, RK_TYPE_Q4_K = 12, RK_TYPE_Q8_0 = 8
 *     (the K-quants on GGUF rows only: rk_mmvq, rk_mmvq_res, rk_weight_bytes, rk_mmvq_isums).
 */
#ifndef RAPIER_B200_H
#define RAPIER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RK_OK 0
#define RK_EINVAL (-1)       /* bad argument: shape, null or misaligned pointer, null stream */
#define RK_ECUDA (-2)        /* a CUDA runtime call or kernel launch failed */
#define RK_ENOMEM (-3)       /* device allocation failed (engine entry points only) */
#define RK_ERANGE (-4)       /* position / token / context out of range */
#define RK_EUNSUPPORTED (-5) /* weight type or layout not handled by this entry */

#define RK_TYPE_Q8_0 8
#define RK_TYPE_Q4_K 12
#define RK_TYPE_Q5_K 13
#define RK_TYPE_Q6_K 14

/* ---------------------------------------------------------------------------------------------- */
/* diagnostics                                                                                       */
/* ---------------------------------------------------------------------------------------------- */
/* Message of the last failed rk_* call on this thread ("" when none). No reference counterpart. */
const char* rk_last_error(void);
/* ABI version: (major << 16) | minor. */
int rk_version(void);
/* OR of every kernel module's device status word (bit 0: a bulk-copy wait gave up; bit 1: a cluster
 * handshake gave up; bit 2: an index handed to a kernel was out of range); clear != 0 resets it.
 * Synchronous. A nonzero value means a kernel returned early instead of hanging. */
unsigned rk_device_status(int clear);

/* ---------------------------------------------------------------------------------------------- */
/* Q8_1 activations                                                                                 */
/* ---------------------------------------------------------------------------------------------- */
/* Replaces strata::kernels::native_q8_1_bytes (src/native_mmvq.cu:3054): bytes of ncols Q8_1 columns. */
size_t rk_q8_1_bytes(int n_in, int ncols);
/* Replaces native_quantize_q8_1 (src/native_mmvq.cu:3059-3071, kernel :158-173): fp32 -> Q8_1 blocks
 * (36 B per 32 values: half2 {d, sum}, int8[32]); columns contiguous. */
int rk_quantize_q8_1(const float* x, void* x_q8_1, int n_in, int ncols, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* Quantized GEMV, GGUF block layout (drop-in)                                                      */
/* ---------------------------------------------------------------------------------------------- */
/* Replaces native_mmvq_weight_bytes (src/native_mmvq.cu:3765-3785) for types 14, 13, 12 and 8. */
size_t rk_weight_bytes(int type, int n_in, int n_out);
/* Replaces native_mmvq (src/native_mmvq.cu:3787-3818) / native_q6_k_mmvq (:3627-3660) /
 * native_q5_k_mmvq (:3341) / native_q4_k_mmvq (:3587) / native_q8_0_mmvq (:3732-3736):
 * y[j*n_out + r] = W[r,:] . x[:, j] on GGUF Q6_K / Q5_K / Q4_K / Q8_0 rows (K-quant rows 4-byte aligned),
 * 1 <= ncols <= 16. */
int rk_mmvq(int type, const void* weights, const void* x_q8_1, float* y, int n_in, int n_out, int ncols,
            void* stream);
/* Replaces native_q6_k_mmvq_res (src/native_mmvq.cu:3187-3200) / native_q5_k_mmvq_res and
 * native_q4_k_mmvq_res (:3202-3324) / native_q8_0_mmvq_res (:3326-3339):
 * y[r] = W[r,:] . x + res[r]; partials[r/4] = sum of y^2 over rows 4(r/4)..4(r/4)+3 (y == res allowed). */
int rk_mmvq_res(int type, const void* weights, const void* x_q8_1, float* y, const float* res, float* partials,
                int n_in, int n_out, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* Quantized GEMV, packed tile layout (the fast path)                                               */
/* ---------------------------------------------------------------------------------------------- */
/* The load-time step of the reference's upload_mat (src/qwythos.cpp:908-935): a lossless repack of
 * GGUF rows into 16-byte-aligned tiles of 4 rows x 1024 values (same byte count). Requires
 * n_in % 1024 == 0 and n_out % 4 == 0; rk_packed_bytes returns 0 for other shapes. */
size_t rk_packed_bytes(int type, int n_in, int n_out);
int rk_pack_weights(int type, const void* src, void* dst, int n_in, int n_out, void* stream);
int rk_unpack_weights(int type, const void* src, void* dst, int n_in, int n_out, void* stream);
/* Same contract as rk_mmvq on packed weights, 1 <= ncols <= 16. */
int rk_mmvq_packed(int type, const void* packed, const void* x_q8_1, float* y, int n_in, int n_out, int ncols,
                   void* stream);
/* rk_mmvq_packed with launch flags. RK_FLAG_STATIC_WEIGHTS: no kernel still in flight on the stream writes
 * these weights, so the GEMV may start streaming them before the previous kernel on the stream has
 * finished (programmatic dependent launch); it still waits for that kernel before reading x_q8_1. */
#define RK_FLAG_STATIC_WEIGHTS 1u
int rk_mmvq_packed_ex(int type, const void* packed, const void* x_q8_1, float* y, int n_in, int n_out, int ncols,
                      unsigned flags, void* stream);
/* Same contract as rk_mmvq_res on packed weights, per column j: y + j*n_out, res + j*n_out,
 * partials + j*(n_out/4). 1 <= ncols <= 16. (The reference runs a 2-column GEMV plus add_partials for
 * this, src/qwythos.cpp:1489-1494.) */
int rk_mmvq_packed_res(int type, const void* packed, const void* x_q8_1, float* y, const float* res,
                       float* partials, int n_in, int n_out, int ncols, void* stream);
/* Parity probe (no reference counterpart): the exact integer sums the packed GEMV accumulates.
 * out[((j*n_out) + r)*nsub + s]; Q6_K: nsub = n_in/16, s = 16-value sub-block, value
 * sum((code-32) * x_code) * scale; Q8_0: nsub = n_in/32, value sum(w_code * x_code).
 * Q5_K / Q4_K (GGUF rows in `packed`, which they have no packed layout for): nsub = 2 * n_in/32, entries
 * 2s, 2s+1 of 32-value sub-block s = the sums of dot1 * scale and dot2 * min of the reference's block
 * threads that cover it (vec_dot_q5_K_q8_1 / _q4_K_q8_1, src/native_mmvq.cu:191-252, :543-595). */
int rk_mmvq_isums(int type, const void* packed, const void* x_q8_1, int32_t* out, int n_in, int n_out, int ncols,
                  void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* norms and elementwise (src/qwythos.cpp:602-715)                                                  */
/* ---------------------------------------------------------------------------------------------- */
/* row_sum_partials_kernel (:616-623): partials[b] = sum of x[4b..4b+3]^2. */
int rk_row_sumsq_partials(const float* x, float* partials, int n, void* stream);
/* add_partials_1024_kernel (:602-614): x += o, partials of the new x. */
int rk_add_partials(float* x, const float* o, float* partials, int n, void* stream);
/* rms_quant_apply_kernel (:627-655): Q8_1 of x * w * rsqrt(sum(partials)/cols + eps); column j reads
 * x + j*cols, partials + j*cols/4, writes y + j*rk_q8_1_bytes(cols,1). cols % 32 == 0. */
int rk_rms_quant_q8_1(const float* x, const float* w, const float* partials, void* y, int cols, int ncols, float eps,
                      void* stream);
/* rms_norm_out_kernel (:658-672): out = x * w * rsqrt(sum(partials)/cols + eps). */
int rk_rms_norm_out(const float* x, const float* w, const float* partials, float* out, int cols, int ncols, float eps,
                    void* stream);
/* swiglu_quant_kernel (:676-689): Q8_1 of silu(gate) * up. */
int rk_swiglu_q8_1(const float* up, const float* gate, void* y, int n, void* stream);
/* sig_mul_quant_kernel (:692-704): Q8_1 of o * sigmoid(g). */
int rk_sigmul_q8_1(const float* o, const float* g, void* y, int n, void* stream);
/* beta_gate_kernel (:707-715): beta = sigmoid(beta) in place; gate = softplus(alpha + dt) * ssm_a. */
int rk_beta_gate(float* beta, const float* alpha, const float* dt, const float* ssm_a, float* gate, int n,
                 void* stream);
/* Strata rms_norm_weighted (called at src/qwythos.cpp:1206-1207): per row x = x * rsqrt(mean(x^2) + eps) * w,
 * in place. */
int rk_rms_norm_rows(float* x, const float* w, int rows, int cols, float eps, void* stream);
/* Parity probe, no reference counterpart: y[i] = f(x[i]) with the exactly specified fp32 sequences every
 * kernel here uses in place of the vendor library (fn 0 exp, 1 log, 2 log1p, 3 sigmoid, 4 silu,
 * 5 1/sqrt as two correctly rounded operations; 6 the CUDA library's expf, for comparison only). */
int rk_math_probe(int fn, const float* x, float* y, int n, void* stream);
/* Greedy argmax of forward_token (src/qwythos.cpp:1803-1811) / argmax_kernel (:70-84): out[j] receives
 * the index of the largest of x[j*n .. j*n+n) (lowest index on ties). */
int rk_argmax(const float* x, int n, int ncols, int* out, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* Gated DeltaNet (src/fused_gdn.cu)                                                                 */
/* ---------------------------------------------------------------------------------------------- */
/* Replaces fused_gdn_conv_l2 (src/fused_gdn.cu:167-176, kernel :113-133). The conv history is a 4-slot
 * ring per channel, ring[c*4 + (p & 3)] = input at position p (the reference keeps [C][3] and slides);
 * *pos is read on the device. In-place h == qkv allowed. */
int rk_gdn_conv_l2(float* ring, const float* qkv, const float* conv_w, float* h, int channels, int qk_heads,
                   float eps, const int* pos, void* stream);
/* Replaces fused_gdn_step_norm_silu_q8 (src/fused_gdn.cu:221-225, kernel :39-111): the delta-rule state
 * step, RMSNorm * gamma * silu(z), and the Q8_1 blocks of y (q8 may be NULL). State fp32
 * [128][h_v][128]. */
int rk_gdn_step_norm_silu_q8(float* state, const float* q, const float* k, const float* v, const float* gate,
                             const float* beta, const float* z, const float* gamma, float eps, float* y, void* q8,
                             int h_k, int h_v, void* stream);

/* The engine's whole GDN recurrence of one layer for 1-2 tokens in one launch (it fuses
 * beta_gate_kernel, src/qwythos.cpp:707-715, fused_gdn_conv_l2 and fused_gdn_step_norm_silu_q8,
 * src/fused_gdn.cu:113-225). Column c (0 <= c < ncols) is the token at position *pos + c; its projection
 * column proj + c*proj_stride = [q h_k*128 | k h_k*128 | v h_v*128 | z h_v*128 | beta h_v | alpha h_v]
 * (the reference's qkv||z and beta||alpha GEMV outputs back to back). The state is read from `snap`
 * instead of `state` when *rollback != 0 (a rejected draft); with ncols == 2 the state after column 0 is
 * written to `snap`. Writes y + c*h_v*128 and the Q8_1 blocks q8 + c*rk_q8_1_bytes(h_v*128, 1).
 * Requires h_v == 2*h_k. */
int rk_gdn_fused(const float* proj, int proj_stride, float* ring, const float* conv_w, const float* dt_bias,
                 const float* ssm_a, const float* gamma, float* state, float* snap, const int* rollback, float* y,
                 void* q8, int h_k, int h_v, int ncols, const int* pos, float eps, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* Attention (src/qwythos.cpp:320-442)                                                               */
/* ---------------------------------------------------------------------------------------------- */
/* split_qg_kernel (:320-327): qg per head [q (hd) | gate (hd)] -> q, g. */
int rk_split_qg(const float* qg, float* q, float* g, int heads, int hd, void* stream);
/* Strata native_rope_apply (called at :1210-1211): NEOX rotate-half over the first n_rot dims of each
 * head, in place, cos/sin from `table` (table[(p*(n_rot/2) + i)*2 + {0,1}] for p < max_pos, built on the
 * host), at position *pos (device; a position outside the table sets status bit 2 and changes nothing). */
int rk_rope(float* x, int heads, int hd, int n_rot, const float* table, int max_pos, const int* pos, void* stream);
/* store_kv2_kernel (:340-345) with fp16 head-major caches [n_kv][max_ctx][hd]:
 * kcache/vcache[(h*max_ctx + *pos)*hd + d] = k/v[h*hd + d]. */
int rk_store_kv_f16(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v, const int* pos, int n_kv,
                    int hd, int max_ctx, void* stream);
/* gqa_head_kernel (:380-442) with fp16 K/V caches [n_kv][max_ctx][hd], split over token chunks: column c
 * (0 <= c < ncols) of q [ncols][n_head][hd] attends tokens 0..*pos + c (device) and writes
 * o [ncols][n_head][hd] = softmax(q . K^T * scale) V. The chunk partials go to `scratch` (caller-owned,
 * like the reference's `scores` buffer), at least rk_gqa_scratch_bytes(n_head, ncols, max_ctx) bytes,
 * max_ctx > *pos + ncols - 1. hd == 256, n_head == 4 * n_kv, 1 <= ncols <= 2. */
size_t rk_gqa_scratch_bytes(int n_head, int ncols, int max_ctx);
int rk_gqa_decode_f16(const float* q, const uint16_t* kcache, const uint16_t* vcache, float* o, int n_head,
                      int n_kv, int hd, int ncols, const int* pos, int max_ctx, float scale, void* scratch,
                      size_t scratch_bytes, void* stream);
/* No counterpart in the reference. rk_gqa_decode_f16 for callers that cannot allocate device memory (an
 * application that owns all device memory through its own pool, a loop that cannot afford cudaMalloc's
 * device synchronization): the chunk partials go to an array built into the library (16 MiB per device,
 * held until exit) and nothing is allocated. Same arguments minus the scratch buffer; rejects shapes
 * whose partials exceed 16 MiB (rk_gqa_scratch_bytes > 16 MiB; e.g. n_head 16, 2 columns fits up to
 * max_ctx 126976) with RK_EINVAL. The first call on each device looks up the array's address; make it
 * before any stream capture. All calls on a device share the array: calls that overlap on the GPU race. */
int rk_gqa_decode_f16_noalloc(const float* q, const uint16_t* kcache, const uint16_t* vcache, float* o, int n_head,
                              int n_kv, int hd, int ncols, const int* pos, int max_ctx, float scale, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* Decode engine (the reference's Engine / load_model / forward_token / draft_predict /              */
/* launch_token_verify, src/qwythos.cpp:152-281, :1228-1618, :1757-1824, :1978-2134, :2905-3251)      */
/* ---------------------------------------------------------------------------------------------- */
/* Model geometry (the reference's compile-time constants, src/qwythos.cpp:33-44, as a runtime struct).
 * Layer il is full attention when (il + 1) % attn_interval == 0 (src/qwythos.cpp:2016), else Gated
 * DeltaNet. The weights are synthetic: every tensor is drawn from `seed` by the counter-based generator
 * and quantized to Q6_K by this library's encoder (no model file is read). */
typedef struct rk_model_config {
    int n_layer;       /* trunk layers (32) */
    int n_embd;        /* hidden (4096) */
    int n_ff;          /* SwiGLU width (12288) */
    int n_vocab;       /* 248320 */
    int ssm_h_k;       /* GDN key heads (16), head size 128 */
    int ssm_h_v;       /* GDN value heads (32) == 2 * ssm_h_k */
    int n_head;        /* attention query heads (16), head_dim 256 */
    int n_head_kv;     /* attention kv heads (4) == n_head / 4 */
    int n_rot;         /* rotary dims (64) */
    int attn_interval; /* 4 */
    int has_mtp;       /* build the nextn draft block (block n_layer) */
    int max_ctx;       /* KV capacity in positions */
    float eps;         /* RMSNorm epsilon (1e-6) */
    double rope_base;  /* 1e7 */
    uint64_t seed;
    double rope_yarn_factor; /* YaRN context scaling (src/qwythos.cpp:1990-1999); <= 1: plain RoPE */
    double rope_orig_ctx;    /* YaRN original context length */
} rk_model_config;

/* Fills `cfg` with the 9B (Qwythos / Qwen3.5-9B) geometry and the given context and seed. */
void rk_model_config_9b(rk_model_config* cfg, int max_ctx, uint64_t seed);


typedef struct rk_engine rk_engine;

/* The model geometry of a qwen35 GGUF file (the reference's load_model, src/qwythos.cpp:1978-2016):
 * layer count from qwen35.block_count minus qwen35.nextn_predict_layers, widths and head counts from the
 * tensor shapes, eps / rope base / YaRN factor and original context from the metadata. Reads the file
 * only (no GPU). RK_EUNSUPPORTED for another architecture. */
int rk_gguf_model_config(const char* path, int max_ctx, rk_model_config* cfg);
/* An engine whose weights come from a qwen35 GGUF file (Q6_K matrices, F32/F16 vectors) instead of the
 * synthetic generator; otherwise as rk_engine_create_tp (tp_size 1: a single GPU). Matrices of other
 * quantization types are refused with RK_EUNSUPPORTED (this engine's GEMVs are Q6_K). */
int rk_engine_create_gguf(const char* path, int device, int max_ctx, int tp_rank, int tp_size, rk_engine** out);
/* The engine's RoPE table [n_pos][n_rot/2][cos, sin] (YaRN when factor > 1). No reference counterpart
 * (a test hook for the table the engine builds). */
int rk_rope_table(int n_rot, double base, double factor, double orig_ctx, int n_pos, float* out);

typedef struct rk_gen_stats {
    double prefill_ms; /* prompt positions 0..P-2 */
    double gen_ms;     /* from the seed pass (position P-1) to the last generated token, device time */
    int n_gen;
    int mtp_steps;     /* verify rounds */
    int mtp_accepted;  /* accepted drafts */
    int single_steps;  /* 1-token trunk passes inside the generation */
    int graph_launches;          /* step-program runs enqueued (graph replays or persistent launches) */
    int kernels_per_single_step; /* kernels one single-token program run launches (1 when persistent) */
    int kernels_per_round;       /* kernels one MTP-round program run launches (1 when persistent) */
} rk_gen_stats;

/* Allocates the engine on `device`, generates the synthetic model and builds the step programs.
 * Returns RK_ENOMEM when the device cannot hold it. */
int rk_engine_create(const rk_model_config* cfg, int device, rk_engine** out);
/* Tensor parallelism (the reference's optional row split, src/qwythos.cpp:908-935, generalized to 2/4/8
 * ranks; one process and one GPU per rank). Rank tp_rank of tp_size holds: its k-heads and the v-heads
 * paired with them (GDN), its q and kv heads (attention), its FF rows of up||gate, its vocabulary shard of
 * the lm_head; the row-parallel GEMVs (ssm_out, wo, down, eh_proj) take its share of their inputs and
 * sum the ranks' partials over NVLink peer memory inside the decode kernel, so every rank keeps the same
 * residual stream; the argmax is global. k-heads and q heads split evenly over the ranks; kv heads too, or,
 * with more ranks than kv heads, each rank keeps the kv head its 2 or 4 q heads use (the 9B geometry at 8
 * ranks); every rank's share of a row-parallel input must be a multiple of 256 (it is padded with zero
 * weight blocks to whole 1024-value tiles) else RK_EUNSUPPORTED. The 9B geometry runs at 2, 4 and 8 ranks.
 * Either executor: the exchange runs inside the row-parallel GEMV kernels (graph) or inside the persistent
 * kernel. After all ranks have created their engines: rk_engine_tp_export on each, an exchange of the handles between the
 * processes, rk_engine_tp_connect on each with all handles (rank-major, rk_tp_handle_bytes each). All
 * ranks then call generate / step / probe in lockstep; logits hold the rank's vocabulary shard. No
 * reference counterpart for the API shape. */
int rk_engine_create_tp(const rk_model_config* cfg, int device, int tp_rank, int tp_size, rk_engine** out);
size_t rk_tp_handle_bytes(void);
int rk_engine_tp_export(rk_engine* e, void* handle, size_t bytes);
int rk_engine_tp_connect(rk_engine* e, const void* handles, size_t bytes_per_rank);
/* Recovery after a failed tensor-parallel call (a rank that did not take part in a step leaves the others'
 * cross-rank waits to give up after RK_TP_WAIT_MS, default 5000, with RK_ECUDA and status bit 3): every rank
 * calls this while none of the group's kernels runs, the ranks meet on the host, then every rank calls
 * rk_engine_reset before the next step. It clears this rank's exchange epochs and flags. No reference
 * counterpart (the reference's row split has no failure path). */
int rk_engine_tp_resync(rk_engine* e);
int rk_engine_destroy(rk_engine* e);
/* Clears KV caches, GDN states, conv rings and the draft cache (the reference's op:reset,
 * src/qwythos.cpp:2533-2549). */
int rk_engine_reset(rk_engine* e);
/* Greedy generation (the reference's CLI loop, src/qwythos.cpp:2905-3251): feeds prompt[0..n_prompt-1]
 * (positions 0..n_prompt-2 as prefill, the last one as the seed pass), then generates n_gen tokens into
 * out_ids. use_mtp != 0: exact MTP (draft 1 token, 2-column verify, greedy acceptance, rollback); the
 * token stream is identical to use_mtp == 0. stats may be NULL. */
int rk_engine_generate(rk_engine* e, const int* prompt, int n_prompt, int n_gen, int use_mtp, int* out_ids,
                       rk_gen_stats* stats);
/* One teacher-forced trunk pass (forward_token, src/qwythos.cpp:1773-1824) of ncols (1 or 2) tokens at
 * positions pos, pos+1: updates the caches and states like a decode step and copies the logits
 * (ncols x n_vocab floats) and argmax ids to the host (either may be NULL). */
int rk_engine_step(rk_engine* e, const int* tokens, int ncols, int pos, float* logits, int* argmax);
/* The MTP draft alone (draft_predict, src/qwythos.cpp:1316-1406): the nextn block at draft position pos
 * (it writes the draft KV slot pos) on [enorm(emb(tok)) | hnorm(h)], h = the final-normed hidden of the
 * last trunk pass's column 0, or h = 0 when h_zero != 0 (the slot-0 seed, src/qwythos.cpp:2955-2958; this
 * also zeroes the saved hidden), then the shared head norm, the lm_head and argmax. Copies the draft
 * logits (n_vocab floats, may be NULL) and the argmax id (may be NULL). A parity hook for the draft. */
int rk_engine_draft_step(rk_engine* e, int tok, int pos, int h_zero, float* logits, int* argmax);
/* Test hook, no reference counterpart: forced MTP draft candidates by position. tokens[p] (p < n), when
 * >= 0, replaces the draft's own prediction as the candidate verified at position p; -1 keeps the draft's.
 * n == 0 clears every entry. The emitted stream does not depend on the candidate (acceptance is exact),
 * so this drives the accept branch with known tokens (e.g. a previous greedy stream) to test it, the way
 * the reference's QWYTHOS_NOACCEPT knob (src/qwythos.cpp:3210) drives the reject branch. Synchronous. */
int rk_engine_force_candidates(rk_engine* e, const int* tokens, int n);
/* Serving session (the reference's --serve loop, src/qwythos.cpp:2593-2812): the engine keeps a context
 * across runs. rk_engine_session_reset clears it (op "reset"; same as rk_engine_reset). A run (op "run")
 * ingests the previous run's last emitted token (still pending) and then tokens[0..n_tokens), all but the
 * last teacher-forced, and generates up to n_gen tokens greedily into out_ids (*n_out of them), stopping
 * after eos_id (-1: never). use_mtp != 0: exact MTP rounds (the stream is the same as use_mtp == 0); the
 * first run after a reset seeds the draft's slot 0. Every emitted token except a final eos_id belongs to the
 * context afterwards. first_logits (n_vocab floats, may be NULL) receives the logits of the first generated
 * token. RK_ERANGE when the context cannot hold the run ("context full; send op reset"). rk_engine_generate
 * leaves a session positioned after its generation. The draft's own cache is filled only by MTP runs: an
 * MTP run after non-MTP runs drafts from an empty cache for the earlier positions, which lowers its
 * acceptance (never its tokens). A run that fails after it has started (a CUDA error, a device-side wait
 * that gave up) leaves the caches and states partly advanced, so every later run returns RK_ECUDA until
 * rk_engine_session_reset (or rk_engine_reset). */
int rk_engine_session_reset(rk_engine* e);
int rk_engine_session_run(rk_engine* e, const int* tokens, int n_tokens, int n_gen, int use_mtp, int eos_id,
                          int* out_ids, int* n_out, float* first_logits, rk_gen_stats* stats);
/* Benchmark helper (no reference counterpart): resets the engine, fills the caches of a context of n_pos
 * tokens with seeded synthetic values (fp16 K and V ~ N(0, 1) in every attention layer and the draft
 * layer; GDN states ~ N(0, 0.01)) and places the session after them, so the next rk_engine_session_run
 * decodes at positions n_pos, n_pos + 1, ... (config 5 at a 65536-token context without a 65536-token
 * prompt). */
int rk_engine_session_fill(rk_engine* e, int n_pos, unsigned long long seed);
/* The session's next position (tokens in the context plus the pending one), -1 for a NULL engine. */
int rk_engine_session_pos(const rk_engine* e);
/* Copies tensor `tid` (this library's synthetic tensor id) to the host: GGUF Q6_K bytes for quantized
 * matrices, fp32 values otherwise. bytes == 0 returns the size. Test hook, no reference counterpart. */
size_t rk_engine_read_tensor(rk_engine* e, int tid, void* host, size_t bytes);
typedef struct rk_probe_result {
    double ms;           /* device time of `iters` replays */
    int launches;        /* GEMV launches per replay */
    double weight_bytes; /* Q6_K weight bytes streamed per replay */
    double algo_bytes;   /* weights + activation inputs + outputs (+ residual reads) per replay */
} rk_probe_result;
/* The reference's probe_gemv (src/qwythos.cpp:1621-1755): runs the GEMVs of one trunk step (every
 * layer's four projection groups and the lm_head, ncols columns) back to back through the engine's
 * executor (one persistent launch, or one graph of GEMV launches), `iters` times, timed with CUDA events.
 * It overwrites the engine's activation buffers (not the caches or states); call rk_engine_reset or
 * generate afterwards. */
int rk_engine_probe_gemv(rk_engine* e, int ncols, int iters, rk_probe_result* out);
/* Device bytes the engine holds. */
size_t rk_engine_device_bytes(const rk_engine* e);
/* The executor the engine runs its step programs with: RK_ENGINE_GRAPH (one kernel per op, replayed from
 * CUDA graphs; the default) or RK_ENGINE_PERSISTENT (one cooperative kernel per program, a whole greedy
 * generation in one launch). The environment variable RK_ENGINE_MODE=graph|persistent, read at
 * rk_engine_create, chooses. Both produce the same bits, with or without tensor parallelism. No reference
 * counterpart (the reference replays a CUDA graph). */
#define RK_ENGINE_GRAPH 0
#define RK_ENGINE_PERSISTENT 1
int rk_engine_mode(const rk_engine* e);
/* Profiling hook (persistent executor only; no reference counterpart): runs one pass of a step program
 * (0 single token, 1 MTP round, 2 / 3 GEMV probe with 1 / 2 columns, 4 the 2-column trunk) with CTA 0
 * recording four stamps per op: op start, prologue done, its own work done, grid barrier passed, in
 * microseconds from the first op's start (stamps_us[4*j .. 4*j+3]). kinds[j]: the op kind (a GEMV is
 * reported as 100 + its epilogue). cta_us (may be NULL): per op and CTA b < max_ctas the CTA's op start
 * and work-done stamps (cta_us[(j*max_ctas + b)*2 + 0/1]; -1 past the grid). Programs 0, 1 and 4 advance
 * the decode state like a step. Returns the program's op count (at most max_ops are written) or a
 * negative RK_E* code. */
int rk_engine_trace(rk_engine* e, int program, double* stamps_us, int* kinds, int max_ops, double* cta_us,
                    int max_ctas);

#ifdef __cplusplus
}
#endif
#endif /* RAPIER_B200_H */
