// Test infrastructure, not product code: C entry points over the reference's own fused Gated-DeltaNet
// launchers (src/fused_gdn.cu of the reference, compiled from the reference tree by `make -C oracle ref`
// into oracle/_ref/libref_gdn.so). tests/test_ref_pin_gpu.py runs them on the GPU box to pin the CPU
// oracle's GDN restatement (or_gdn_conv_l2, or_beta_gate, or_gdn_step_norm_silu_q8) to the reference's
// kernels. The reference's launchers exit the process on invalid arguments, so callers pass valid ones.
#include <cstdint>

#include "strata/kernels/fused_gdn.hpp"

extern "C" {

void ref_gdn_conv_l2(float* history, const float* qkv, const float* conv_w, float* h, int channels, int qk_heads,
                     float eps, void* stream) {
    strata::kernels::fused_gdn_conv_l2(history, qkv, conv_w, h, channels, qk_heads, eps, stream);
}

void ref_gdn_ab(const float* x, const uint16_t* w_alpha, const uint16_t* w_beta, const float* dt, const float* ssm_a,
                float* gate, float* beta, int n_embd, int h_v, void* stream) {
    strata::kernels::fused_gdn_ab(x, w_alpha, w_beta, dt, ssm_a, gate, beta, n_embd, h_v, stream);
}

void ref_gdn_step_norm_silu_q8(float* state, const float* q, const float* k, const float* v, const float* gate,
                               const float* beta, const float* z, const float* gamma, float eps, float* y, uint8_t* q8,
                               int h_k, int h_v, void* stream) {
    strata::kernels::fused_gdn_step_norm_silu_q8(state, q, k, v, gate, beta, z, gamma, eps, y, q8, h_k, h_v, stream);
}

}  // extern "C"
