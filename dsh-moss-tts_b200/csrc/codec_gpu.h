// codec_gpu.h -- the GPU codec decoder (mossgpu_codec_*, codec.cu) for C++ callers:
// CodecStreams, the job runtime's codec (one codec stream per job, below), and AudioDecoder, the
// reference's single-utterance class moss::AudioDecoder (csrc/include/moss/decoder.h:16-33): the same
// constructor (threads, accepted and unused: the work runs on the GPU) and methods load /
// decode / reset_stream / decode_chunk / last_ms / stage_ms / info, backed by one codec stream.
//
// Differences a caller can see: load() reads only .moss decoder files whose matrices are f16
// (decoder_f16.moss, the shipped form), and a decode call that the codec rejects (a code
// outside [0, 1024), an activation beyond fp16 range) throws std::runtime_error where the
// reference has no error path.  stage_ms() stays empty (the stages run as one stream of
// kernels); last_ms() is decode()'s wall time, as in the reference.
#pragma once

#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/mossgpu.h"

namespace moss {
namespace gpu {

class AudioDecoder {
public:
    // max_chunk_frames sizes the codec's buffers; longer decode_chunk / decode calls are split
    // into pieces of that many frames, which the streaming state joins exactly
    explicit AudioDecoder(int threads = 1, int device = 0, int max_chunk_frames = 64)
        : device_(device), max_chunk_(max_chunk_frames > 0 ? max_chunk_frames : 64) {
        (void)threads;
    }
    ~AudioDecoder() {
        if (c_) mossgpu_codec_destroy(c_);
    }
    AudioDecoder(const AudioDecoder &) = delete;
    AudioDecoder &operator=(const AudioDecoder &) = delete;

    // decoder.cpp:28-71
    bool load(const std::string &path, std::string *err) {
        if (c_) {
            mossgpu_codec_destroy(c_);
            c_ = nullptr;
        }
        char buf[512] = {0};
        c_ = mossgpu_codec_create(path.c_str(), device_, 1, max_chunk_, buf, int(sizeof(buf)));
        if (!c_) {
            if (err) *err = buf;
            return false;
        }
        if (mossgpu_codec_open(c_, &sid_) != 0) {
            if (err) *err = mossgpu_codec_last_error(c_);
            mossgpu_codec_destroy(c_);
            c_ = nullptr;
            return false;
        }
        spf_ = mossgpu_codec_samples_per_frame(c_);
        info_ = "decoder weights=" + path + " device=" + std::to_string(device_) + " (GPU)";
        return true;
    }

    // decoder.cpp:254-280: the whole utterance, codes [16][frames], interleaved stereo out
    std::vector<float> decode(const int32_t *codes, int frames) {
        const auto t0 = std::chrono::steady_clock::now();
        std::vector<float> out(size_t(frames > 0 ? frames : 0) * size_t(spf_));
        int n = 0;
        check(mossgpu_codec_decode(c_, codes, frames, out.data(), out.size(), &n));
        out.resize(size_t(n));
        last_ms_ = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        return out;
    }

    // decoder.cpp:105-114
    void reset_stream() { check(mossgpu_codec_reset(c_, sid_)); }

    // decoder.cpp:211-225: one chunk of the stream, codes [16][frames]
    std::vector<float> decode_chunk(const int32_t *codes, int frames) {
        std::vector<float> out(size_t(frames > 0 ? frames : 0) * size_t(spf_));
        std::vector<int32_t> piece;
        size_t at = 0;
        for (int f0 = 0; f0 < frames; f0 += max_chunk_) {
            const int k = frames - f0 < max_chunk_ ? frames - f0 : max_chunk_;
            const int32_t *src = codes;
            if (k != frames) {  // [16][frames] -> the [16][k] block of frames f0..f0+k-1
                piece.resize(size_t(16) * size_t(k));
                for (int i = 0; i < 16; ++i)
                    std::memcpy(piece.data() + size_t(i) * k, codes + size_t(i) * frames + f0, sizeof(int32_t) * k);
                src = piece.data();
            }
            int n = 0;
            check(mossgpu_codec_decode_chunk(c_, sid_, src, k, out.data() + at, out.size() - at, &n));
            at += size_t(n);
        }
        out.resize(at);
        return out;
    }

    double last_ms() const { return last_ms_; }
    const std::vector<double> &stage_ms() const { return stage_ms_; }
    const std::string &info() const { return info_; }

private:
    void check(int rc) const {
        if (!c_) throw std::runtime_error("AudioDecoder: load() has not succeeded");
        if (rc != 0) throw std::runtime_error(std::string("AudioDecoder: ") + mossgpu_codec_last_error(c_));
    }

    mossgpu_codec *c_ = nullptr;
    int device_ = 0, max_chunk_ = 64, sid_ = -1, spf_ = 0;
    double last_ms_ = 0.0;
    std::vector<double> stage_ms_;
    std::string info_;
};

// The Codec of TextJobRuntime (job_runtime.h) on one GPU codec: open() gives each job its own
// codec stream (the reference's decoder_->reset_stream() at the start of synthesize,
// engine.cpp:434), and Stream::decode turns one nq-major block codes[16][n] into interleaved
// stereo samples (decode_chunk, engine.cpp:495).  Every call on the shared codec holds one
// mutex: submit() opens streams on the caller's thread while the runtime's worker decodes.
class CodecStreams {
public:
    class Stream {
    public:
        Stream(CodecStreams *owner, int sid) : owner_(owner), sid_(sid) {}
        ~Stream() { owner_->close(sid_); }
        Stream(const Stream &) = delete;
        Stream &operator=(const Stream &) = delete;
        // segment: the text segment; the stream carries on across segments as one utterance
        bool decode(int segment, const int32_t *codes, int n, std::vector<float> *audio, std::string *err) {
            (void)segment;
            return owner_->decode(sid_, codes, n, audio, err);
        }
        int id() const { return sid_; }

    private:
        CodecStreams *owner_;
        int sid_;
    };

    CodecStreams(const std::string &decoder_path, int device, int max_streams, int max_chunk_frames = 64)
        : max_chunk_(max_chunk_frames > 0 ? max_chunk_frames : 64) {
        char buf[512] = {0};
        c_ = mossgpu_codec_create(decoder_path.c_str(), device, max_streams, max_chunk_, buf, int(sizeof(buf)));
        if (!c_) throw std::runtime_error(std::string("codec: ") + buf);
        spf_ = mossgpu_codec_samples_per_frame(c_);
    }
    ~CodecStreams() { mossgpu_codec_destroy(c_); }
    CodecStreams(const CodecStreams &) = delete;
    CodecStreams &operator=(const CodecStreams &) = delete;

    // nullptr when every codec stream is taken
    std::unique_ptr<Stream> open() {
        std::lock_guard<std::mutex> lock(mu_);
        int sid = -1;
        if (mossgpu_codec_open(c_, &sid) != 0) return nullptr;
        return std::unique_ptr<Stream>(new Stream(this, sid));
    }

private:
    void close(int sid) {
        std::lock_guard<std::mutex> lock(mu_);
        mossgpu_codec_close(c_, sid);
    }
    bool decode(int sid, const int32_t *codes, int n, std::vector<float> *audio, std::string *err) {
        std::lock_guard<std::mutex> lock(mu_);
        audio->assign(size_t(n > 0 ? n : 0) * size_t(spf_), 0.0f);
        std::vector<int32_t> piece;
        size_t at = 0;
        for (int f0 = 0; f0 < n; f0 += max_chunk_) {
            const int k = n - f0 < max_chunk_ ? n - f0 : max_chunk_;
            const int32_t *src = codes;
            if (k != n) {
                piece.resize(size_t(16) * size_t(k));
                for (int i = 0; i < 16; ++i)
                    std::memcpy(piece.data() + size_t(i) * k, codes + size_t(i) * n + f0, sizeof(int32_t) * k);
                src = piece.data();
            }
            int got = 0;
            if (mossgpu_codec_decode_chunk(c_, sid, src, k, audio->data() + at, audio->size() - at, &got) != 0) {
                if (err) *err = mossgpu_codec_last_error(c_);
                return false;
            }
            at += size_t(got);
        }
        audio->resize(at);
        return true;
    }

    mossgpu_codec *c_ = nullptr;
    int max_chunk_ = 64, spf_ = 0;
    std::mutex mu_;
};

}  // namespace gpu
}  // namespace moss
