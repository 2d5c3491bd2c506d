// shim_demo.cpp -- drives moss::gpu::LlmModel (dsh-moss-tts_b200/csrc/llm_gpu.h) the way the
// reference's moss_llm CLI drives moss::LlmModel (reference main.cpp:98-167): load, prefill
// a prompt, optionally save/restore the prefix cache, generate greedy frames, print codes.
//   shim_demo <weights.moss> <prompt_rows.bin [n][17] int32> <frames> [prefix.mosskv]
// Exit codes: 0 ok, 2 load failed (message on stderr), 3 other error.
#include <cstdio>
#include <fstream>
#include <vector>

#include "llm_gpu.h"

int main(int argc, char **argv) {
    if (argc < 4) return 3;
    std::vector<moss::gpu::Row> rows;
    {
        std::ifstream in(argv[2], std::ios::binary);
        moss::gpu::Row r{};
        while (in.read(reinterpret_cast<char *>(r.data()), sizeof(int32_t) * r.size())) rows.push_back(r);
    }
    const int frames = std::atoi(argv[3]);
    moss::gpu::LlmModel model(4, 0, 1024);
    std::string err;
    if (!model.load(argv[1], &err)) {
        std::fprintf(stderr, "load failed: %s\n", err.c_str());
        return 2;
    }
    try {
        model.prefill(rows);
        if (argc > 4) {
            if (!model.save_prefix(argv[4], rows, &err)) throw std::runtime_error(err);
            model.reset();
            if (!model.load_prefix(argv[4], rows, &err)) throw std::runtime_error(err);
            model.restore_prefix();
        }
        moss::gpu::SampleParams p;
        p.greedy = true;
        p.repetition_penalty = 1.2f;
        p.min_frames = 1 << 20;
        const auto out = model.generate(frames, p, 0);
        std::printf("{\"position\": %d, \"codes\": [", model.position());
        for (size_t i = 0; i < out.size(); ++i) {
            std::printf("%s[", i ? ", " : "");
            for (int ch = 0; ch < 16; ++ch) std::printf("%s%d", ch ? ", " : "", out[i][ch + 1]);
            std::printf("]");
        }
        std::printf("]}\n");
    } catch (const std::exception &e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 3;
    }
    return 0;
}
