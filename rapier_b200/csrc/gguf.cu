// gguf.cu — the GGUF reader (gguf.cuh), the model geometry of a qwen35 GGUF file (rk_gguf_model_config,
// the reference's load_model checks, src/qwythos.cpp:1978-2016), and the RoPE cos / sin table with YaRN
// scaling (rk_rope_table).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "gguf.cuh"

namespace rk {

size_t ggml_row_bytes(int type, int64_t ne0) {
    if (ne0 <= 0) return 0;
    switch (type) {
        case kGgmlF32: return (size_t) ne0 * 4;
        case kGgmlF16:
        case kGgmlBF16: return (size_t) ne0 * 2;
        case kGgmlQ8_0: return ne0 % 32 ? 0 : (size_t) ne0 / 32 * 34;
        case kGgmlQ6_K: return ne0 % 256 ? 0 : (size_t) ne0 / 256 * 210;
        default: return 0;
    }
}

namespace {
// Bounds-checked little-endian cursor over the mapping.
struct Reader {
    const uint8_t* p;
    size_t n, at = 0;
    bool ok = true;
    bool need(size_t k) {
        if (!ok || k > n - at) ok = false;
        return ok;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            std::memcpy(&v, p + at, sizeof(T));
            at += sizeof(T);
        }
        return v;
    }
    std::string string() {
        const uint64_t len = get<uint64_t>();
        if (!need((size_t) len) || len > (1ull << 30)) return ok = false, std::string();
        std::string s(reinterpret_cast<const char*>(p + at), (size_t) len);
        at += (size_t) len;
        return s;
    }
};

enum : uint32_t { GU8, GI8, GU16, GI16, GU32, GI32, GF32, GBOOL, GSTR, GARR, GU64, GI64, GF64 };

bool scalar_size(uint32_t t, size_t& sz) {
    switch (t) {
        case GU8: case GI8: case GBOOL: sz = 1; return true;
        case GU16: case GI16: sz = 2; return true;
        case GU32: case GI32: case GF32: sz = 4; return true;
        case GU64: case GI64: case GF64: sz = 8; return true;
        default: return false;
    }
}

double scalar_value(Reader& r, uint32_t t) {
    switch (t) {
        case GU8: return r.get<uint8_t>();
        case GI8: return r.get<int8_t>();
        case GBOOL: return r.get<uint8_t>();
        case GU16: return r.get<uint16_t>();
        case GI16: return r.get<int16_t>();
        case GU32: return r.get<uint32_t>();
        case GI32: return r.get<int32_t>();
        case GF32: return r.get<float>();
        case GU64: return (double) r.get<uint64_t>();
        case GI64: return (double) r.get<int64_t>();
        case GF64: return r.get<double>();
        default: r.ok = false; return 0.0;
    }
}
}  // namespace

GgufFile::~GgufFile() {
    if (map_) munmap(map_, size_);
}

bool GgufFile::open(const char* path, std::string& err) {
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return err = std::string("cannot open ") + path, false;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        return err = "not a GGUF file (too short)", false;
    }
    size_ = (size_t) st.st_size;
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) return err = "mmap failed", false;
    map_ = static_cast<uint8_t*>(m);
    Reader r{map_, size_};
    const uint32_t magic = r.get<uint32_t>();
    const uint32_t version = r.get<uint32_t>();
    if (magic != 0x46554747u) return err = "not a GGUF file (bad magic)", false;
    if (version != 2 && version != 3) return err = "unsupported GGUF version " + std::to_string(version), false;
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return err = "corrupt GGUF header", false;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.string();
        const uint32_t t = r.get<uint32_t>();
        size_t sz = 0;
        if (t == GSTR) {
            strs_[key] = r.string();
        } else if (t == GARR) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t cnt = r.get<uint64_t>();
            if (et == GSTR) {
                for (uint64_t k = 0; k < cnt && r.ok; ++k) r.string();
            } else if (scalar_size(et, sz) && cnt <= (uint64_t) (size_ / (sz ? sz : 1))) {
                if (r.need((size_t) (cnt * sz))) r.at += (size_t) (cnt * sz);
            } else {
                r.ok = false;
            }
        } else if (scalar_size(t, sz)) {
            nums_[key] = scalar_value(r, t);
        } else {
            r.ok = false;
        }
    }
    if (!r.ok) return err = "corrupt GGUF metadata", false;
    tensors_.resize((size_t) n_tensors);
    std::vector<uint64_t> offs((size_t) n_tensors);
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        GgufTensor& t = tensors_[(size_t) i];
        t.name = r.string();
        t.n_dims = (int) r.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) r.ok = false;
        for (int d = 0; d < t.n_dims && r.ok; ++d) {
            const uint64_t ne = r.get<uint64_t>();
            if (ne < 1 || ne > (1ull << 40)) r.ok = false;  // also keeps every product below 2^128
            t.ne[d] = (int64_t) ne;
        }
        t.type = (int) r.get<uint32_t>();
        offs[(size_t) i] = r.get<uint64_t>();
    }
    if (!r.ok) return err = "corrupt GGUF tensor directory", false;
    double align = 32;
    num("general.alignment", align);
    const size_t a = align >= 1 ? (size_t) align : 32;
    const size_t data0 = (r.at + a - 1) / a * a;
    for (size_t i = 0; i < tensors_.size(); ++i) {
        GgufTensor& t = tensors_[i];
        const size_t row = ggml_row_bytes(t.type, t.ne[0]);
        // bytes = row * ne1 * ne2 * ne3 in exact integer arithmetic (each factor < 2^41 here)
        unsigned __int128 bytes = row;
        bool big = false;
        for (int d = 1; d < 4; ++d) {
            bytes *= (unsigned __int128) (uint64_t) t.ne[d];
            if (bytes > (unsigned __int128) size_) big = true;  // larger than the file: refused below
            if (big) break;
        }
        t.bytes = big ? size_ + 1 : (size_t) bytes;
        if (row && (big || offs[i] > size_ || data0 + offs[i] > size_ || t.bytes > size_ - data0 - offs[i]))
            return err = "tensor " + t.name + " extends past the end of the file", false;
        t.data = row ? map_ + data0 + offs[i] : nullptr;
        index_[t.name] = i;
    }
    return true;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
    const auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}
bool GgufFile::num(const std::string& key, double& out) const {
    const auto it = nums_.find(key);
    if (it == nums_.end()) return false;
    out = it->second;
    return true;
}
bool GgufFile::str(const std::string& key, std::string& out) const {
    const auto it = strs_.find(key);
    if (it == strs_.end()) return false;
    out = it->second;
    return true;
}

// The cos / sin table [pos][n_rot/2][2] of NEOX RoPE. factor <= 1: theta = pos * base^(-2i/n_rot). factor
// > 1: YaRN (Peng et al. 2023, "YaRN: Efficient Context Window Extension of Large Language Models"), as
// the reference configures it (src/qwythos.cpp:1990-1999: ext_factor 1, attn_factor 1, beta_fast 32,
// beta_slow 1): per dimension pair the interpolated angle pos * theta_i / factor and the extrapolated
// pos * theta_i are mixed by a ramp over the pair index between the correction dims of beta_fast and
// beta_slow, and cos / sin are scaled by 1 + 0.1 ln(factor).
void build_rope_table(int n_rot, double base, double factor, double orig_ctx, int n_pos, std::vector<float>& t) {
    const int half = n_rot / 2;
    t.assign((size_t) n_pos * half * 2, 0.0f);
    const bool yarn = factor > 1.0;
    double lo = 0, hi = 0, mscale = 1.0;
    if (yarn) {
        auto corr_dim = [&](double beta) {
            return n_rot * std::log(orig_ctx / (beta * 2.0 * M_PI)) / (2.0 * std::log(base));
        };
        lo = std::max(0.0, std::floor(corr_dim(32.0)));
        hi = std::min((double) (n_rot - 1), std::ceil(corr_dim(1.0)));
        mscale = 1.0 + 0.1 * std::log(factor);
    }
    for (int p = 0; p < n_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const double ext = (double) p * std::pow(base, -2.0 * i / (double) n_rot);
            double a = ext, m = 1.0;
            if (yarn) {
                const double y = ((double) i - lo) / std::max(0.001, hi - lo);
                const double ramp = 1.0 - std::min(1.0, std::max(0.0, y));  // 1: extrapolate, 0: interpolate
                a = ext / factor * (1.0 - ramp) + ext * ramp;
                m = mscale;
            }
            t[((size_t) p * half + i) * 2 + 0] = (float) (std::cos(a) * m);
            t[((size_t) p * half + i) * 2 + 1] = (float) (std::sin(a) * m);
        }
}

}  // namespace rk

using namespace rk;

extern "C" {

int rk_gguf_model_config(const char* path, int max_ctx, rk_model_config* cfg) {
    const char* what = "rk_gguf_model_config";
    if (!path || !cfg) return set_error(RK_EINVAL, "%s: null argument", what);
    if (max_ctx < 8) return set_error(RK_EINVAL, "%s: max_ctx must be >= 8", what);
    GgufFile f;
    std::string err;
    if (!f.open(path, err)) return set_error(RK_EINVAL, "%s: %s", what, err.c_str());
    std::string arch;
    if (!f.str("general.architecture", arch) || arch != "qwen35")
        return set_error(RK_EUNSUPPORTED, "%s: not a qwen35 GGUF (general.architecture '%s')", what, arch.c_str());
    double blocks = 0, nextn = 0;
    if (!f.num("qwen35.block_count", blocks)) return set_error(RK_EINVAL, "%s: qwen35.block_count missing", what);
    f.num("qwen35.nextn_predict_layers", nextn);
    const int n_layer = (int) blocks - (int) nextn;
    auto tensor = [&](const std::string& name) { return f.find(name); };
    const GgufTensor* emb = tensor("token_embd.weight");
    const GgufTensor* up = tensor("blk.0.ffn_up.weight");
    if (n_layer < 1 || !emb || !up || emb->n_dims != 2 || up->n_dims != 2)
        return set_error(RK_EINVAL, "%s: token_embd.weight / blk.0.ffn_up.weight missing", what);
    std::memset(cfg, 0, sizeof *cfg);
    cfg->n_layer = n_layer;
    cfg->n_embd = (int) emb->ne[0];
    cfg->n_vocab = (int) emb->ne[1];
    cfg->n_ff = (int) up->ne[1];
    // layer kinds: full attention every `interval` layers (the first layer holding attn_q)
    int interval = 0;
    double iv = 0;
    if (f.num("qwen35.full_attention_interval", iv)) interval = (int) iv;
    for (int il = 0; il < n_layer && interval == 0; ++il)
        if (tensor("blk." + std::to_string(il) + ".attn_q.weight")) interval = il + 1;
    if (interval < 1) return set_error(RK_EINVAL, "%s: no attention layer found", what);
    cfg->attn_interval = interval;
    int gdn = -1, att = interval - 1;
    for (int il = 0; il < n_layer && gdn < 0; ++il)
        if ((il + 1) % interval != 0) gdn = il;
    if (gdn >= 0) {
        const std::string b = "blk." + std::to_string(gdn) + ".";
        const GgufTensor *beta = tensor(b + "ssm_beta.weight"), *qkv = tensor(b + "attn_qkv.weight"),
                         *sn = tensor(b + "ssm_norm.weight");
        if (!beta || !qkv || !sn) return set_error(RK_EINVAL, "%s: GDN tensors of layer %d missing", what, gdn);
        if (sn->ne[0] != 128) return set_error(RK_EUNSUPPORTED, "%s: GDN head size %lld (128 expected)", what, (long long) sn->ne[0]);
        cfg->ssm_h_v = (int) beta->ne[1];
        cfg->ssm_h_k = (int) ((qkv->ne[1] - (int64_t) cfg->ssm_h_v * 128) / 256);
    }
    {
        const std::string b = "blk." + std::to_string(att) + ".";
        const GgufTensor *q = tensor(b + "attn_q.weight"), *k = tensor(b + "attn_k.weight");
        if (!q || !k) return set_error(RK_EINVAL, "%s: attention tensors of layer %d missing", what, att);
        cfg->n_head = (int) (q->ne[1] / 512);
        cfg->n_head_kv = (int) (k->ne[1] / 256);
    }
    cfg->has_mtp = nextn > 0 && tensor("blk." + std::to_string(n_layer) + ".nextn.eh_proj.weight") != nullptr;
    cfg->max_ctx = max_ctx;
    double v = 64;
    f.num("qwen35.rope.dimension_count", v);
    cfg->n_rot = (int) v;
    v = 1e-6;
    f.num("qwen35.attention.layer_norm_rms_epsilon", v);
    cfg->eps = (float) v;
    cfg->rope_base = 1e7;
    f.num("qwen35.rope.freq_base", cfg->rope_base);
    cfg->rope_yarn_factor = 1.0;
    f.num("qwen35.rope.scaling.factor", cfg->rope_yarn_factor);
    cfg->rope_orig_ctx = 262144;
    f.num("qwen35.rope.scaling.original_context_length", cfg->rope_orig_ctx);
    cfg->seed = 0;
    return RK_OK;
}

int rk_rope_table(int n_rot, double base, double factor, double orig_ctx, int n_pos, float* out) {
    if (n_rot <= 0 || n_rot % 2 || n_pos <= 0 || !out || !(base > 1.0))
        return set_error(RK_EINVAL, "rk_rope_table: bad arguments");
    std::vector<float> t;
    build_rope_table(n_rot, base, factor, orig_ctx, n_pos, t);
    std::memcpy(out, t.data(), t.size() * sizeof(float));
    return RK_OK;
}

}  // extern "C"
