// The reference's sampling loop (src/chat_session.cpp:154-186: logits = engine.forward(...);
// next = sampler.sample(logits)) written against include/minicpm5_engine.hpp.
//   sampler_driver <model.gguf> <mode> <n_generate> <temperature> <top_p> <seed> <prompt ids...>
// mode "host":   forward() copies the logits to the host vector, which Sampler::sample is given
// mode "device": set_host_logits(false): the logits stay on the device and are sampled there
// mode "copy":   the host logits are copied into a vector of the caller's, which the sampler
//                uploads (mcpm_sample_top_p_host)
// Prints, per sampled token, "token r" where r is the sampler's draw (the same std::mt19937
// stream the Sampler consumes, replayed from the seed).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "minicpm5_engine.hpp"

int main(int argc, char** argv) {
    if (argc < 8) {
        std::fprintf(stderr, "usage: %s model.gguf host|device|copy n_generate temperature top_p seed id...\n", argv[0]);
        return 2;
    }
    const std::string path = argv[1], mode = argv[2];
    const int n_gen = std::atoi(argv[3]);
    const float temp = static_cast<float>(std::atof(argv[4])), top_p = static_cast<float>(std::atof(argv[5]));
    const uint32_t seed = static_cast<uint32_t>(std::strtoul(argv[6], nullptr, 10));
    std::vector<int> prompt;
    for (int i = 7; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
    const int max_seq = static_cast<int>(prompt.size()) + n_gen + 1;
    MiniCPM5Engine engine;
    engine.init_kv_cache(max_seq);
    if (!engine.load_model(path)) return 1;
    if (mode == "device") engine.set_host_logits(false);
    Sampler sampler(temp, top_p, seed);
    std::mt19937 replay(seed);   // the draws Sampler makes, for the caller's check
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    int next = -1;
    for (size_t pos = 0; pos < prompt.size(); ++pos) {
        const std::vector<float>& logits = engine.forward(prompt[pos], static_cast<int>(pos), max_seq);
        if (pos == prompt.size() - 1) {
            if (mode == "copy") {
                std::vector<float> mine(logits);
                next = sampler.sample(mine);
            } else {
                next = sampler.sample(logits);
            }
            std::printf("%d %.9g\n", next, static_cast<double>(dist(replay)));
        }
    }
    int cur = static_cast<int>(prompt.size());
    for (int step = 0; step < n_gen; ++step, ++cur) {
        if (next < 0) return 3;
        const std::vector<float>& logits = engine.forward(next, cur, max_seq);
        if (mode == "copy") {
            std::vector<float> mine(logits);
            next = sampler.sample(mine);
        } else {
            next = sampler.sample(logits);
        }
        std::printf("%d %.9g\n", next, static_cast<double>(dist(replay)));
    }
    return next < 0 ? 3 : 0;
}
