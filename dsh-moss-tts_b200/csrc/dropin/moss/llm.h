// dropin/moss/llm.h -- the GPU engine as the reference's moss::LlmModel, for building the
// reference's own C++ layers (TtsEngine engine.cpp, Runtime runtime.cpp, the C ABI capi.cpp,
// the moss_llm CLI main.cpp) on the B200 engine with no source change.
//
// Integration: put this directory ahead of the reference's csrc/include on the include path,
// leave llm.cpp out of the build, and link libmossgpu.so.  Every reference file that includes
// "moss/llm.h" then gets:
//   - the model constants, Row and FrameTiming that the reference's llm.h:18-37 declares (the
//     interface the callers use: prompt rows [text id, code0..15], per-frame timings);
//   - moss::SampleParams from the reference's own sampler.h (included from its directory);
//   - moss::LlmModel = moss::gpu::LlmModel (llm_gpu.h): the same constructor (threads),
//     load / reset / prefill / snapshot_prefix / restore_prefix / save_prefix / load_prefix /
//     save_state / load_state / generate / set_logits_dump / set_gate_dump /
//     set_cancel_flag / hidden / position / info, backed by one stream of a device engine.
// The reference's llm.h also pulls in common.h, gemv.h, parallel.h and weights.h; they are
// included here too, so that files relying on them through llm.h still compile.
#pragma once

#include <array>
#include <cstdint>

#include "moss/common.h"
#include "moss/gemv.h"
#include "moss/parallel.h"
#include "moss/sampler.h"
#include "moss/weights.h"

namespace moss {

// model shape (llm.h:18-29); kMaxCtx is the GPU engine's default context (mossgpu_create)
constexpr int kHidden = 768;
constexpr int kHeads = 12;
constexpr int kHeadDim = 64;
constexpr int kFF = 3072;
constexpr int kVocab = 16384;
constexpr int kNVq = 16;
constexpr int kCodebook = 1024;
constexpr int kAudioPad = 1024;
constexpr int kSlotToken = 9;
constexpr int kEndToken = 7;
constexpr int kMaxCtx = 4608;
constexpr int kLocalLen = 17;

using Row = std::array<int32_t, kNVq + 1>;

struct FrameTiming {
    double global_ms = 0.0;
    double local_ms = 0.0;
};

}  // namespace moss

#include "../../llm_gpu.h"

namespace moss {
using LlmModel = gpu::LlmModel;
}  // namespace moss
