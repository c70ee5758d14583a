// Token loop written against the reference's engine interface (MiniCPM5Engine with
// init_kv_cache / load_model / forward), built on include/minicpm5_engine.hpp.
//   facade_driver <model.gguf> <n_generate> <prompt ids...>
// Prints one greedy token per line (host argmax of the returned logits, lowest index on
// ties) and exits non-zero if it disagrees with the engine's device argmax.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "minicpm5_engine.hpp"

int main(int argc, char** argv) {
    if (argc < 4) {
        std::fprintf(stderr, "usage: %s model.gguf n_generate id...\n", argv[0]);
        return 2;
    }
    const std::string path = argv[1];
    const int n_gen = std::atoi(argv[2]);
    std::vector<int> prompt;
    for (int i = 3; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
    const int max_seq = static_cast<int>(prompt.size()) + n_gen + 1;
    MiniCPM5Engine engine;
    engine.init_kv_cache(max_seq);
    if (!engine.load_model(path)) return 1;
    int tok = prompt[0];
    for (int pos = 0; pos < static_cast<int>(prompt.size()) + n_gen; ++pos) {
        if (pos < static_cast<int>(prompt.size())) tok = prompt[pos];
        const std::vector<float>& logits = engine.forward(tok, pos, max_seq);
        int best = 0;
        for (size_t i = 1; i < logits.size(); ++i)
            if (logits[i] > logits[best]) best = static_cast<int>(i);
        if (best != engine.last_argmax()) {
            std::fprintf(stderr, "pos %d: host argmax %d != device argmax %d\n", pos, best, engine.last_argmax());
            return 3;
        }
        std::printf("%d\n", best);
        tok = best;
    }
    return 0;
}
