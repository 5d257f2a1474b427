// The one geometry constant the reference's src/fused_gdn.cu checks at compile time (the GDN state size of
// the qwen35 models), for building that file into the test-only oracle/_ref library.
#pragma once

namespace strata::core {

struct CompiledGeometry {
    int ssm_state_size;
};
inline constexpr CompiledGeometry kCompiledGeometry{128};

}  // namespace strata::core
