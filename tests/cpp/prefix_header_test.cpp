// The .mosskv header as moss::gpu::LlmModel (llm_gpu.h) writes it: the struct layout and the
// two fingerprints (rows: FNV-1a over the prompt rows, llm.cpp:410-423; weights: FNV-1a over
// the file size and first 4 KB, llm.cpp:426-439), printed for comparison with a header the
// reference's save_prefix wrote.  Host-only: no engine call is made, so no GPU is needed.
//   prefix_header_test <weights.moss> <rows.bin [n][17] int32>
// Prints "size <bytes> offsets <magic> <version> <layers> <n_pos> <hidden> <rows_fp> <weights_fp>",
// "fp <rows_fp> <weights_fp>" and "magic <prefix-file magic bytes> <state-file magic bytes>".
#include <array>
#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

// the header struct and fingerprint helpers are private members of the shim class
#define private public
#include "llm_gpu.h"
#undef private

int main(int argc, char **argv) {
    if (argc != 3) return 2;
    std::vector<moss::gpu::Row> rows;
    std::ifstream in(argv[2], std::ios::binary);
    moss::gpu::Row r{};
    while (in.read(reinterpret_cast<char *>(r.data()), sizeof(int32_t) * r.size())) rows.push_back(r);
    using H = moss::gpu::LlmModel::KvHeader;
    std::printf("size %zu offsets %zu %zu %zu %zu %zu %zu %zu\n", sizeof(H), offsetof(H, magic), offsetof(H, version),
                offsetof(H, layers), offsetof(H, n_pos), offsetof(H, hidden), offsetof(H, rows_fp),
                offsetof(H, weights_fp));
    std::printf("fp %llu %llu\n", static_cast<unsigned long long>(moss::gpu::LlmModel::fp_rows(rows)),
                static_cast<unsigned long long>(moss::gpu::LlmModel::fp_weights(argv[1])));
    std::printf("magic");
    for (const char *m : {moss::gpu::LlmModel::kKvMagic, moss::gpu::LlmModel::kStateMagic})
        for (int i = 0; i < 8; ++i) std::printf(" %d", static_cast<int>(static_cast<unsigned char>(m[i])));
    std::printf("\n");
    return 0;
}
