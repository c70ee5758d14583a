// Header-only C++ facades with the reference's interfaces, so a token loop written against
// the reference (src/chat_session.cpp:154-186, src/main.cpp:107-114) compiles unchanged
// against this header and runs on the GPU.  Link with libmcpm.so.
//   class MiniCPM5Engine   include/model.h:37-70: init_kv_cache, load_model, forward
//   class Sampler          include/sampler.h:14-25: Sampler(temperature, top_p), sample(logits)
//
// Differences a caller can observe:
//  * forward() returns the logits of the step in a host vector, as the reference does; the
//    greedy token of that step is also available from last_argmax() (computed on the device,
//    lowest index on ties), which saves the host scan over 130,560 logits.
//  * set_host_logits(false) skips that 522 KB device-to-host copy per step: forward() then
//    returns the engine's vector unchanged, and Sampler::sample given that vector samples the
//    step's logits where they are, on the device.  The reference's loop
//    `logits = engine_.forward(...); next = sampler_.sample(logits);` runs unchanged.
//  * Sampler draws r from its own std::mt19937 (seeded from std::random_device, as the
//    reference's, or from a seed given to the third constructor argument) and samples on the
//    device in a fixed canonical order (ties by index); for the same r it returns the token of
//    the reference's algorithm up to float rounding of the cumulative sums.
//  * The KV cache holds at most 16,384 positions (the reference allocates any size):
//    init_kv_cache reports a larger max_seq_len at once and load_model then fails.
//  * Errors that the reference reports as a console warning (pos >= max_seq_len, a token id
//    out of range) print the status string and leave the previous logits in place.
#pragma once

#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <random>
#include <string>
#include <vector>

#include "mcpm.h"

namespace mcpm_facade {
// Logits vectors of live MiniCPM5Engine facades -> their engines, so Sampler::sample can find
// the device copy of a vector that forward() returned.
inline std::mutex& registry_mutex() {
    static std::mutex m;
    return m;
}
inline std::map<const std::vector<float>*, mcpm_engine*>& registry() {
    static std::map<const std::vector<float>*, mcpm_engine*> r;
    return r;
}
inline mcpm_engine* engine_of(const std::vector<float>* v) {
    std::lock_guard<std::mutex> lock(registry_mutex());
    auto it = registry().find(v);
    return it == registry().end() ? nullptr : it->second;
}
constexpr int MAX_SEQ = 16384;
}  // namespace mcpm_facade

class MiniCPM5Engine {
public:
    explicit MiniCPM5Engine(int device = 0, int n_ctas = 0) : device_(device), n_ctas_(n_ctas) {}
    ~MiniCPM5Engine() {
        {
            std::lock_guard<std::mutex> lock(mcpm_facade::registry_mutex());
            mcpm_facade::registry().erase(&logits_);
        }
        if (eng_) mcpm_engine_destroy(eng_);
    }
    MiniCPM5Engine(const MiniCPM5Engine&) = delete;
    MiniCPM5Engine& operator=(const MiniCPM5Engine&) = delete;

    // Reference model.cpp:17-24: (re)allocates the fp32 KV cache for max_seq_len positions.
    // May be called before or after load_model.
    void init_kv_cache(int max_seq_len) {
        max_seq_ = max_seq_len;
        if (max_seq_len <= 0 || max_seq_len > mcpm_facade::MAX_SEQ) {
            std::fprintf(stderr, "[mcpm] init_kv_cache: max_seq_len %d outside 1..%d positions\n", max_seq_len,
                         mcpm_facade::MAX_SEQ);
            return;
        }
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
        {
            std::lock_guard<std::mutex> lock(mcpm_facade::registry_mutex());
            mcpm_facade::registry()[&logits_] = eng_;
        }
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
        if (host_logits_) {
            if (report(mcpm_forward(eng_, token_id, pos, logits_.data(), &tok), "forward")) argmax_ = tok;
        } else if (report(mcpm_forward_async(eng_, token_id, pos, 1), "forward") && report(mcpm_sync(eng_), "forward")) {
            argmax_ = -1;   // on the device (mcpm_argmax_device); the host vector is not refreshed
        }
        return logits_;
    }

    // true (default): forward() copies the step's logits into the returned vector.  false:
    // the logits stay on the device; pass the returned vector to Sampler::sample, which samples
    // them there (not in the reference).
    void set_host_logits(bool on) { host_logits_ = on; }

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
    bool loaded_ = false, host_logits_ = true;
    int argmax_ = -1;
    std::vector<float> logits_;
};

// Reference include/sampler.h:14-25 / src/sampler.cpp:8-72: softmax with temperature,
// top-p truncation, one uniform draw r in [0, 1).  The draw comes from this object's
// std::mt19937; the sampling itself runs on the device: on the engine's device logits when
// `logits` is the vector a MiniCPM5Engine facade returned, otherwise on a device copy of
// `logits`.  Returns -1 (and prints why) if the device call fails.
class Sampler {
public:
    Sampler(float temperature = 1.0f, float top_p = 0.95f)
        : temperature_(temperature), top_p_(top_p), rng_(std::random_device{}()) {}
    Sampler(float temperature, float top_p, uint32_t seed) : temperature_(temperature), top_p_(top_p), rng_(seed) {}

    int sample(const std::vector<float>& logits) {
        std::uniform_real_distribution<float> dist(0.0f, 1.0f);
        const float r = dist(rng_);
        int tok = -1;
        mcpm_engine* e = mcpm_facade::engine_of(&logits);
        const mcpm_status st = e ? mcpm_sample(e, temperature_, top_p_, r, &tok)
                                 : mcpm_sample_top_p_host(logits.data(), static_cast<int>(logits.size()), temperature_,
                                                          top_p_, r, &tok);
        if (st != MCPM_OK) {
            std::fprintf(stderr, "[mcpm] Sampler::sample: %s\n", mcpm_status_string(st));
            return -1;
        }
        return tok;
    }

private:
    float temperature_;
    float top_p_;
    std::mt19937 rng_;
};
