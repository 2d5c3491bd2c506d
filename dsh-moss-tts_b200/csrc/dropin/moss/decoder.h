// dropin/moss/decoder.h -- the GPU codec decoder as the reference's moss::AudioDecoder, for
// building the reference's own C++ layers (TtsEngine engine.cpp, the moss_decoder CLI
// decoder_main.cpp) on the B200 codec with no source change.
//
// Integration: this directory ahead of the reference's csrc/include on the include path,
// decoder.cpp left out of the build, libmossgpu.so linked.  Every reference file that includes
// "moss/decoder.h" then gets moss::AudioDecoder = moss::gpu::AudioDecoder (codec_gpu.h): the
// reference class's constructor (threads) and load / decode / reset_stream / decode_chunk /
// last_ms / stage_ms / info, backed by one codec stream on the GPU.  The reference's header
// also pulls in audio_layer.h, common.h, gemv.h, parallel.h and weights.h; they are included
// here too, so that files relying on them through decoder.h still compile.
#pragma once

#include <string>
#include <vector>

#include "moss/audio_layer.h"
#include "moss/common.h"
#include "moss/gemv.h"
#include "moss/parallel.h"
#include "moss/weights.h"

#include "../../codec_gpu.h"

namespace moss {
using AudioDecoder = gpu::AudioDecoder;
}  // namespace moss
