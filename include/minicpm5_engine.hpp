// Header-only C++ facade with the reference engine's interface (class MiniCPM5Engine,
// include/model.h:37-70 of astrowar/MiniCPM5.cpp): init_kv_cache, load_model and forward
// with the same arguments and meaning, so a token loop written against the reference
// (src/chat_session.cpp:154-186, src/main.cpp:107-114) compiles unchanged against this
// header and runs on the GPU.  Link with libmcpm.so.
//
// Differences a caller can observe:
//  * forward() returns the logits of the step in a host vector, as the reference does; the
//    greedy token of that step is also available from last_argmax() (computed on the device,
//    lowest index on ties), which saves the host scan over 130,560 logits.
//  * Errors that the reference reports as a console warning (pos >= max_seq_len, a token id
//    out of range) print the status string and leave the previous logits in place.
#pragma once

#include <cstdio>
#include <string>
#include <vector>

#include "mcpm.h"

class MiniCPM5Engine {
public:
    explicit MiniCPM5Engine(int device = 0, int n_ctas = 0) : device_(device), n_ctas_(n_ctas) {}
    ~MiniCPM5Engine() {
        if (eng_) mcpm_engine_destroy(eng_);
    }
    MiniCPM5Engine(const MiniCPM5Engine&) = delete;
    MiniCPM5Engine& operator=(const MiniCPM5Engine&) = delete;

    // Reference model.cpp:17-24: (re)allocates the fp32 KV cache for max_seq_len positions.
    // May be called before or after load_model.
    void init_kv_cache(int max_seq_len) {
        max_seq_ = max_seq_len;
        if (eng_ && loaded_) report(mcpm_init_kv(eng_, max_seq_len), "init_kv_cache");
    }

    // Reference model.cpp:33-133: reads the GGUF file and uploads every tensor's bytes
    // unchanged into device memory.  Returns false (and prints why) on any failure.
    bool load_model(const std::string& gguf_path, bool verbose = false) {
        if (!eng_) {
            mcpm_config cfg{};
            cfg.device = device_;
            cfg.max_seq = max_seq_;
            cfg.n_ctas = n_ctas_;
            if (!report(mcpm_engine_create(&cfg, &eng_), "engine_create")) return false;
        }
        if (!report(mcpm_load_gguf(eng_, gguf_path.c_str()), "load_model")) return false;
        int dims[6] = {0, 0, 0, 0, 0, 0};
        if (!report(mcpm_model_dims(eng_, dims), "model_dims")) return false;
        logits_.assign(static_cast<size_t>(dims[5]), 0.0f);
        loaded_ = true;
        if (verbose)
            std::printf("[mcpm] loaded %s: %d layers, n_embd %d, n_ff %d, heads %d/%d, vocab %d\n", gguf_path.c_str(),
                        dims[0], dims[1], dims[2], dims[3], dims[4], dims[5]);
        return true;
    }

    // Reference model.cpp:142-242: one decode step for `token_id` at position `pos`.  The
    // returned reference stays valid until the next call.  max_seq_len is checked against
    // pos as the reference's attention does (ops.cpp:550-553).
    const std::vector<float>& forward(int token_id, int pos, int max_seq_len) {
        if (!eng_ || !loaded_) {
            std::fprintf(stderr, "[mcpm] forward before load_model\n");
            return logits_;
        }
        if (pos >= max_seq_len) {
            std::fprintf(stderr, "[mcpm] position %d exceeds max_seq_len %d\n", pos, max_seq_len);
            return logits_;
        }
        int tok = -1;
        if (report(mcpm_forward(eng_, token_id, pos, logits_.data(), &tok), "forward")) argmax_ = tok;
        return logits_;
    }

    // Greedy token of the last successful forward (device argmax; not in the reference).
    int last_argmax() const { return argmax_; }

private:
    bool report(mcpm_status s, const char* what) const {
        if (s == MCPM_OK) return true;
        std::fprintf(stderr, "[mcpm] %s: %s\n", what, mcpm_status_string(s));
        return false;
    }

    int device_ = 0, n_ctas_ = 0, max_seq_ = 4096;
    mcpm_engine* eng_ = nullptr;
    bool loaded_ = false;
    int argmax_ = -1;
    std::vector<float> logits_;
};
