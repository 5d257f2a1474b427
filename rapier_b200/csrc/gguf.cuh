// gguf.cuh — a read-only GGUF (versions 2 and 3) reader for the decode engine's model files: the header,
// the key/value metadata (numbers and strings; arrays are skipped), and the tensor directory, over a
// memory-mapped file. Every offset and length is checked against the file size.
//
// The format is the public GGUF layout: magic "GGUF", version, tensor count, metadata count; metadata
// entries (key string, value type, value); tensor infos (name, dims ne[0..n), ggml type, offset); tensor
// data from the first multiple of general.alignment (default 32) after the infos.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace rk {

constexpr int kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ8_0 = 8, kGgmlQ6_K = 14, kGgmlBF16 = 30;

struct GgufTensor {
    std::string name;
    int type = -1;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    const uint8_t* data = nullptr;  // inside the mapping
    size_t bytes = 0;
};

class GgufFile {
public:
    ~GgufFile();
    // Maps and parses `path`; on failure returns false with a message in `err`.
    bool open(const char* path, std::string& err);
    const GgufTensor* find(const std::string& name) const;
    bool num(const std::string& key, double& out) const;
    bool str(const std::string& key, std::string& out) const;
    const std::vector<GgufTensor>& tensors() const { return tensors_; }

private:
    uint8_t* map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, double> nums_;
    std::map<std::string, std::string> strs_;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> index_;
};

// Bytes of one row of ne0 values of a ggml type this reader knows (0: unknown type or ragged row).
size_t ggml_row_bytes(int type, int64_t ne0);

// The RoPE cos / sin table [n_pos][n_rot/2][2] (YaRN scaling when factor > 1), in gguf.cu.
void build_rope_table(int n_rot, double base, double factor, double orig_ctx, int n_pos, std::vector<float>& t);

}  // namespace rk
