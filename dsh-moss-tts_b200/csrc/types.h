// types.h -- constants and plain structs shared by host code and kernels (no device code).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace mossgpu {

constexpr int kHidden = 768;
constexpr int kHeads = 12;
constexpr int kHeadDim = 64;
constexpr int kFF = 3072;
constexpr int kQKV = 3 * kHidden;
constexpr int kVocab = 16384;
constexpr int kNVq = 16;
constexpr int kCodebook = 1024;
constexpr int kAudioPad = 1024;
constexpr int kSlotToken = 9;
constexpr int kEndToken = 7;
constexpr int kLocalLen = 17;
constexpr int kLayers = 12;
constexpr int kPage = 16;                                  // positions per KV page
constexpr int kPageHalfs = 2 * kHeads * kPage * kHeadDim;  // one page of one layer (k and v)
constexpr int kNumSMs = 148;                                // B200: persistent grids (one CTA per SM)
constexpr int kPlanThreads = 1024;                          // threads of the split-K plan kernel
constexpr int kAttnChunk = 16;                             // minimum split-K chunk (positions, one page)
constexpr int kPartStride = 68;  // floats per split-K partial: m, l, 2 pad, o[64] (16-byte rows)

struct QMat {
    const int8_t *qs;   // [rows/4][nb][4][32]
    const __half *sc;   // [rows/4][nb][4]
    int rows, cols;
};

struct EmbedTables {
    QMat wte;
    QMat aemb[kNVq];
};

// Per-frame sampling/stop controls in device memory (moss::SampleParams, sampler.h:8-22).
struct FrameCtl {
    int min_frames;
    int greedy_frames;
    float rep_penalty;
    int end_greedy;
    int has_forced;
    int greedy;         // sampler.h:8-22
    float temperature;
    int top_k;
    float top_p;
};
constexpr int kFrameCtlInts = 12;  // control-block ints reserved for FrameCtl
static_assert(sizeof(FrameCtl) <= kFrameCtlInts * sizeof(int), "FrameCtl outgrew its control-block slot");

}  // namespace mossgpu
