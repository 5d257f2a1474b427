// Interface of the reference's fused Gated-DeltaNet launchers, for compiling its src/fused_gdn.cu into the
// test-only oracle/_ref library (the header itself is not part of the reference tree). The signatures must
// be those the reference defines, or the objects would not link.
#pragma once

#include <cstdint>

namespace strata::kernels {

void fused_gdn_conv_l2(float* history, const float* qkv, const float* conv_w, float* h, int channels, int qk_heads,
                       float eps, void* stream);
void fused_gdn_ab(const float* x, const uint16_t* w_alpha, const uint16_t* w_beta, const float* dt, const float* ssm_a,
                  float* gate, float* beta, int n_embd, int h_v, void* stream);
void fused_gdn_step_norm(float* state, const float* q, const float* k, const float* v, const float* gate,
                         const float* beta, const float* z, const float* gamma, float eps, float* y, int h_k, int h_v,
                         void* stream);
void fused_gdn_step_norm_silu(float* state, const float* q, const float* k, const float* v, const float* gate,
                              const float* beta, const float* z, const float* gamma, float eps, float* y, int h_k,
                              int h_v, void* stream);
void fused_gdn_step_norm_silu_q8(float* state, const float* q, const float* k, const float* v, const float* gate,
                                 const float* beta, const float* z, const float* gamma, float eps, float* y,
                                 uint8_t* q8, int h_k, int h_v, void* stream);

}  // namespace strata::kernels
