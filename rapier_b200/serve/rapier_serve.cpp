// rapier_serve: the engine process behind the reference's server (server/rapier_server.py starts
// `ENGINE --model FILE --serve` and speaks JSON lines on stdin / stdout), over librapier_b200's C-ABI.
//
//   rapier_serve --model FILE.gguf --serve            a qwen35 GGUF (Q6_K matrices)
//   rapier_serve --synthetic 9b|tiny [--seed N] --serve   the synthetic model (no file)
//   rapier_serve ... --prompt 1,2,3 --gen N [--mtp]    one greedy generation, a JSON summary on stdout
//
// Options: --max-ctx N (else $QWYTHOS_MAXCTX, else 4096), --device N, --eos ID (default 248046; -1 none).
//
// The protocol (src/qwythos.cpp:2139-2147, :2593-2812), one JSON object per line:
//   {"op":"reset"}                                   -> {"ok":true,"op":"reset"}
//   {"op":"run","tokens":[..],"gen":N,"mtp":B,"topk":K}
//        -> one {"id":I,"top":[[id,logit],..]} per generated token, then {"done":true,"pos":P}
// tokens are appended to the context kept across runs; generation stops after the end-of-sequence id.
// Without MTP every token carries the top-K logits (K = "topk", default 40); with MTP the first token
// does and the rest carry an empty list (the reference skips the logits copy on its MTP path). Errors:
// {"error":"need tokens and gen"}, {"error":"context full; send op reset"}, {"error":"<message>"}.
// P counts the context's tokens, the last emitted one included.
#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <string>
#include <utility>
#include <vector>

#include "rapier_b200.h"

namespace {

struct Args {
    std::string model, synthetic;
    bool serve = false, mtp = false;
    int max_ctx = 0, device = 0, eos = 248046, gen = 32;
    unsigned long long seed = 1;
    std::vector<int> prompt;
};

[[noreturn]] void usage(const char* msg) {
    std::fprintf(stderr, "rapier_serve: %s\nusage: rapier_serve (--model FILE.gguf | --synthetic 9b|tiny [--seed N]) "
                         "(--serve | --prompt IDS --gen N [--mtp]) [--max-ctx N] [--device N] [--eos ID]\n", msg);
    std::exit(2);
}

std::vector<int> parse_ids(const char* s) {
    std::vector<int> v;
    const char* p = s;
    while (*p) {
        char* end = nullptr;
        const long x = std::strtol(p, &end, 10);
        if (end == p) usage("bad id list");
        v.push_back((int) x);
        p = end;
        while (*p == ',' || *p == ' ') ++p;
    }
    return v;
}

Args parse_args(int argc, char** argv) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        const std::string k = argv[i];
        auto val = [&]() -> const char* {
            if (i + 1 >= argc) usage(("missing value for " + k).c_str());
            return argv[++i];
        };
        if (k == "--model") a.model = val();
        else if (k == "--synthetic") a.synthetic = val();
        else if (k == "--seed") a.seed = std::strtoull(val(), nullptr, 10);
        else if (k == "--serve") a.serve = true;
        else if (k == "--mtp") a.mtp = true;
        else if (k == "--prompt") a.prompt = parse_ids(val());
        else if (k == "--gen") a.gen = std::atoi(val());
        else if (k == "--max-ctx") a.max_ctx = std::atoi(val());
        else if (k == "--device") a.device = std::atoi(val());
        else if (k == "--eos") a.eos = std::atoi(val());
        else usage(("unknown option " + k).c_str());
    }
    if (a.model.empty() == a.synthetic.empty()) usage("give exactly one of --model and --synthetic");
    if (!a.serve && a.prompt.empty()) usage("give --serve or --prompt");
    if (a.max_ctx <= 0) {
        const char* env = std::getenv("QWYTHOS_MAXCTX");
        a.max_ctx = env ? std::atoi(env) : 4096;
    }
    return a;
}

// ---- the few JSON shapes of the protocol (keys of one flat object; numbers, booleans, one int array) ----
size_t find_key(const std::string& line, const char* key) {
    const std::string pat = std::string("\"") + key + "\"";
    size_t at = line.find(pat);
    if (at == std::string::npos) return std::string::npos;
    at += pat.size();
    while (at < line.size() && std::isspace((unsigned char) line[at])) ++at;
    if (at >= line.size() || line[at] != ':') return std::string::npos;
    ++at;
    while (at < line.size() && std::isspace((unsigned char) line[at])) ++at;
    return at;
}
long long num_field(const std::string& line, const char* key, long long dflt) {
    const size_t at = find_key(line, key);
    if (at == std::string::npos) return dflt;
    char* end = nullptr;
    const long long v = std::strtoll(line.c_str() + at, &end, 10);
    return end == line.c_str() + at ? dflt : v;
}
bool bool_field(const std::string& line, const char* key) {
    const size_t at = find_key(line, key);
    return at != std::string::npos && line.compare(at, 4, "true") == 0;
}
bool str_field_is(const std::string& line, const char* key, const char* value) {
    const size_t at = find_key(line, key);
    return at != std::string::npos && line.compare(at, std::strlen(value) + 2, std::string("\"") + value + "\"") == 0;
}
std::vector<int> ids_field(const std::string& line, const char* key) {
    std::vector<int> v;
    size_t at = find_key(line, key);
    if (at == std::string::npos || line[at] != '[') return v;
    const char* p = line.c_str() + at + 1;
    while (*p && *p != ']') {
        char* end = nullptr;
        const long x = std::strtol(p, &end, 10);
        if (end == p) {
            ++p;
            continue;
        }
        v.push_back((int) x);
        p = end;
    }
    return v;
}

// The reference's topk_out order (src/qwythos.cpp:2511-2531): larger logit first, the lower id among equals.
std::vector<std::pair<int, float>> top_k(const std::vector<float>& logits, int k) {
    std::vector<std::pair<int, float>> top;
    if (k <= 0) return top;
    auto better = [](const std::pair<int, float>& a, const std::pair<int, float>& b) {
        return a.second > b.second || (a.second == b.second && a.first < b.first);
    };
    top.reserve((size_t) k + 1);
    for (int i = 0; i < (int) logits.size(); ++i) {
        const std::pair<int, float> c(i, logits[(size_t) i]);
        if ((int) top.size() < k) {
            top.push_back(c);
            std::push_heap(top.begin(), top.end(), better);  // the heap's front: the worst kept
        } else if (better(c, top.front())) {
            std::pop_heap(top.begin(), top.end(), better);
            top.back() = c;
            std::push_heap(top.begin(), top.end(), better);
        }
    }
    std::sort(top.begin(), top.end(), better);
    return top;
}

void emit(int id, const std::vector<std::pair<int, float>>& top) {
    std::printf("{\"id\":%d,\"top\":[", id);
    for (size_t i = 0; i < top.size(); ++i) std::printf("%s[%d,%.5f]", i ? "," : "", top[i].first, top[i].second);
    std::printf("]}\n");
    std::fflush(stdout);
}

void reply(const char* json) {
    std::printf("%s\n", json);
    std::fflush(stdout);
}

int serve_loop(rk_engine* e, const rk_model_config& cfg, int eos) {
    std::fprintf(stderr, "rapier serve: ready\n");
    std::string line;
    std::vector<float> logits((size_t) cfg.n_vocab);
    while (std::getline(std::cin, line)) {
        if (line.find_first_not_of(" \t\r") == std::string::npos) continue;
        if (str_field_is(line, "op", "reset")) {
            if (rk_engine_session_reset(e) != RK_OK) {
                std::printf("{\"error\":\"reset failed: %s\"}\n", rk_last_error());
                std::fflush(stdout);
                continue;
            }
            reply("{\"ok\":true,\"op\":\"reset\"}");
            continue;
        }
        const long long gen = num_field(line, "gen", -1);
        const bool mtp = bool_field(line, "mtp") && cfg.has_mtp;
        const int topk = (int) std::min<long long>(std::max<long long>(num_field(line, "topk", 40), 0), 1000);
        const std::vector<int> toks = ids_field(line, "tokens");
        if (toks.empty() || gen <= 0) {
            reply("{\"error\":\"need tokens and gen\"}");
            continue;
        }
        bool bad = false;
        for (int t : toks) bad |= t < 0 || t >= cfg.n_vocab;
        if (bad) {
            reply("{\"error\":\"token id outside the vocabulary\"}");
            continue;
        }
        if ((long long) rk_engine_session_pos(e) + (long long) toks.size() + gen + 8 >= cfg.max_ctx) {
            reply("{\"error\":\"context full; send op reset\"}");
            continue;
        }
        std::vector<int> out((size_t) gen);
        int n_out = 0, rc = RK_OK;
        if (mtp) {  // one exact-MTP run; the first token carries its top-k
            rc = rk_engine_session_run(e, toks.data(), (int) toks.size(), (int) gen, 1, eos, out.data(), &n_out,
                                       logits.data(), nullptr);
            for (int i = 0; rc == RK_OK && i < n_out; ++i)
                emit(out[(size_t) i], i == 0 ? top_k(logits, topk) : std::vector<std::pair<int, float>>());
        } else {  // token by token, each with the top-k of its logits
            const int* in = toks.data();
            int n_in = (int) toks.size();
            for (long long i = 0; rc == RK_OK && i < gen; ++i) {
                int id = -1, n1 = 0;
                rc = rk_engine_session_run(e, in, n_in, 1, 0, eos, &id, &n1, logits.data(), nullptr);
                if (rc != RK_OK || n1 < 1) break;
                emit(id, top_k(logits, topk));
                ++n_out;
                in = nullptr;  // later steps ingest only the pending token
                n_in = 0;
                if (id == eos) break;
            }
        }
        if (rc != RK_OK) {
            std::string msg = rk_last_error();
            for (char& c : msg)
                if (c == '"' || c == '\\') c = '\'';
            std::printf("{\"error\":\"%s\"}\n", msg.c_str());
            std::fflush(stdout);
            continue;
        }
        std::printf("{\"done\":true,\"pos\":%d}\n", rk_engine_session_pos(e));
        std::fflush(stdout);
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    const Args a = parse_args(argc, argv);
    rk_model_config cfg;
    rk_engine* e = nullptr;
    int rc = RK_OK;
    if (!a.model.empty()) {
        rc = rk_gguf_model_config(a.model.c_str(), a.max_ctx, &cfg);
        if (rc == RK_OK) rc = rk_engine_create_gguf(a.model.c_str(), a.device, a.max_ctx, 0, 1, &e);
    } else {
        rk_model_config_9b(&cfg, a.max_ctx, a.seed);
        if (a.synthetic == "tiny") {  // the test geometry: 4 layers, 1024 wide, 4096 tokens
            cfg.n_layer = 4;
            cfg.n_embd = 1024;
            cfg.n_ff = 2048;
            cfg.n_vocab = 4096;
            cfg.ssm_h_k = 4;
            cfg.ssm_h_v = 8;
            cfg.n_head = 4;
            cfg.n_head_kv = 1;
        } else if (a.synthetic != "9b") {
            usage("--synthetic takes 9b or tiny");
        }
        rc = rk_engine_create(&cfg, a.device, &e);
    }
    if (rc != RK_OK) {
        std::fprintf(stderr, "rapier_serve: %s\n", rk_last_error());
        return 1;
    }
    const int eos = a.eos >= 0 && a.eos < cfg.n_vocab ? a.eos : -1;
    int status = 0;
    if (a.serve) {
        status = serve_loop(e, cfg, eos);
    } else {
        std::vector<int> out((size_t) a.gen);
        rk_gen_stats st;
        rc = rk_engine_generate(e, a.prompt.data(), (int) a.prompt.size(), a.gen, a.mtp && cfg.has_mtp ? 1 : 0,
                                out.data(), &st);
        if (rc != RK_OK) {
            std::fprintf(stderr, "rapier_serve: %s\n", rk_last_error());
            status = 1;
        } else {
            std::printf("{\"ids\":[");
            for (size_t i = 0; i < out.size(); ++i) std::printf("%s%d", i ? "," : "", out[i]);
            std::printf("],\"tok_per_s\":%.2f,\"gen_ms\":%.3f,\"mtp_steps\":%d,\"mtp_accepted\":%d}\n",
                        st.gen_ms > 0 ? a.gen / (st.gen_ms / 1e3) : 0.0, st.gen_ms, st.mtp_steps, st.mtp_accepted);
        }
    }
    rk_engine_destroy(e);
    return status;
}
