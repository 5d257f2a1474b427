/*
 * oracle.h — CPU restatement of the reference decode path (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the checker for the CUDA kernels in rapier_b200/csrc. Only tests/, the
 * smoke() of __graft_entry__.py and the cpu_baseline leg of bench.py may load it. The product path
 * never calls it.
 *
 * Parity status (see the pin list at the top of oracle.c):
 *   - Q6_K / Q8_0 block layouts and dequantization: pinned against gguf-py 0.19.0 (an independent
 *     implementation of the ggml formats) by tests/golden fixtures.
 *   - Q8_0 encoding: pinned against gguf-py's quantizer (bit-exact).
 *   - Q6_K x Q8_1 / Q8_0 x Q8_1 integer sub-block sums: pinned by an integer identity against the
 *     gguf-decoded codes (tests/golden).
 *   - q8_1_finite / q8_1_quant / rms_norm_weighted / native_rope_apply live in the out-of-tree Strata
 *     fork and are not in the reference tree: their rules here are a written definition ("parity
 *     unpinned" for those three rules).
 *   - fp32 reductions follow the reference kernels' order as written in its source.
 */
#ifndef RAPIER_ORACLE_H
#define RAPIER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 ---- */
uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);
void or_f32_to_f16_n(const float* x, uint16_t* y, size_t n);
void or_f16_to_f32_n(const uint16_t* x, float* y, size_t n);

/* ---- seeded synthetic values (identical stream to the device generator) ---- */
uint64_t or_hash64(uint64_t seed, uint64_t idx);
void or_synth_normal(uint64_t seed, uint64_t offset, float scale, float mean, float* out, size_t n);

/* ---- Q8_1 activations ---- */
size_t or_q8_1_bytes(int n_in, int ncols);
void or_quantize_q8_1(const float* x, void* y, int n_in, int ncols);
void or_dequantize_q8_1(const void* y, float* x, int n);

/* ---- weights: GGUF layouts (type 14 = Q6_K, type 8 = Q8_0) ---- */
size_t or_weight_bytes(int type, int n_in, int n_out);
/* Q5_K (13) / Q4_K (12) blocks to fp32 (ggml's dequantize_row_q5_K / _q4_K). */
void or_dequant_kq(int type, const void* w, float* y, int n_values);
size_t or_packed_bytes(int type, int n_in, int n_out);
void or_quantize_weights(int type, const float* w, void* dst, int n_in, int n_out);
void or_dequantize_weights(int type, const void* w, float* dst, int n_in, int n_out);
int or_pack_weights(int type, const void* src, void* dst, int n_in, int n_out);
int or_unpack_weights(int type, const void* src, void* dst, int n_in, int n_out);

/* ---- GEMV ---- */
void or_mmvq(int type, const void* w, const void* xq, float* y, int n_in, int n_out, int ncols);
void or_mmvq_res(int type, const void* w, const void* xq, float* y, const float* res, float* partials,
                 int n_in, int n_out, int ncols);
/* The GEMV in the packed-tile kernel's order (y = W x (+ res), optional 4-row partials; res and partials
 * may be NULL). */
void or_mmvq_packed(int type, const void* w, const void* xq, float* y, const float* res, float* partials, int n_in,
                    int n_out, int ncols);
void or_mmvq_isums(int type, const void* w, const void* xq, int32_t* out, int n_in, int n_out, int ncols);

/* ---- norms / elementwise ---- */
void or_row_sumsq_partials(const float* x, float* partials, int n);
void or_add_partials(float* x, const float* o, float* partials, int n);
float or_partials_sumsq(const float* partials, int nslots);
void or_rms_quant_q8_1(const float* x, const float* w, const float* partials, void* y, int cols, float eps);
void or_rms_norm_out(const float* x, const float* w, const float* partials, float* out, int cols, float eps);
void or_swiglu_q8_1(const float* up, const float* gate, void* y, int n);
void or_sigmul_q8_1(const float* o, const float* g, void* y, int n);
void or_beta_gate(float* beta, const float* alpha, const float* dt, const float* ssm_a, float* gate, int n);
void or_rms_norm_rows(float* x, const float* w, int rows, int cols, float eps);

/* ---- Gated DeltaNet ---- */
void or_gdn_conv_l2(float* ring, const float* qkv, const float* conv_w, float* h, int channels, int qk_heads,
                    float eps, int pos);
void or_gdn_step_norm_silu_q8(float* state, const float* q, const float* k, const float* v, const float* gate,
                              const float* beta, const float* z, const float* gamma, float eps, float* y,
                              void* q8, int h_k, int h_v);

/* ---- attention ---- */
void or_rope_table(float* table, int max_pos, int n_rot, double freq_base);
void or_rope_apply(float* x, int heads, int hd, int n_rot, const float* table, int pos);
void or_split_qg(const float* qg, float* q, float* g, int heads, int hd);
void or_store_kv_f16(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v, int pos, int n);
void or_gqa_decode_f16(const float* q, const uint16_t* kc, const uint16_t* vc, float* o, int n_head, int n_kv,
                       int hd, int n_tok, float scale);

/* ---- greedy ---- */
void or_attn_flash_f16(const float* proj, int ncols, int proj_stride, const float* qn, const float* kn,
                       const float* rope, int n_rot, int n_head, int n_kv, uint16_t* kc, uint16_t* vc, int pos,
                       int chunk_len, float eps, float scale, float* o, void* q8);
int or_argmax(const float* x, int n);

/* ---- timing helper for the CPU baseline ---- */
/* The exactly specified transcendentals (fn 0 exp, 1 log, 2 log1p, 3 sigmoid, 4 silu, 5 1/sqrt). */
float or_expf(float x);
float or_logf(float x);
float or_log1pf(float t);
void or_math_n(int fn, const float* x, float* y, size_t n);
int or_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
