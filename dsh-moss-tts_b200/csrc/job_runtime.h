// job_runtime.h -- moss::gpu::TextJobRuntime: the reference Runtime's text-level job API,
// submit(request, PcmSink, job_id, err) / wait / job / cancel / queue_depth (reference
// csrc/include/moss/runtime.h:45-113, runtime.cpp:282-432), over BatchRuntime, so that every
// admitted utterance advances in the same batched engine calls instead of one synthesize() at
// a time.  Header-only C++17, host side.
//
// The text front end and the audio codec are the reference's and stay outside the engine; they
// plug in as template parameters:
//   Frontend  bool prepare(const std::string &text, const std::string &voice,
//                          const std::string &profile, TextJob *out, std::string *err)
//             -- TtsEngine's set_voice + split_text + text_to_ids + build_text_suffix and its
//             prefix cache (engine.cpp:201-243,305-463): the suffix rows of every text segment
//             and the engine stream that holds the voice prefix.  Prefix streams must be
//             prefilled before the runtime's worker starts (the engine is the worker's then).
//             Called on the submitting thread.
//   Codec     std::unique_ptr<Stream> open()  -- one streaming decoder per job, where Stream
//             has bool decode(int segment, const int32_t *codes, int n,
//                             std::vector<float> *audio, std::string *err)
//             turning one nq-major block codes[16][n] into interleaved stereo float samples at
//             48 kHz (AudioDecoder::decode_chunk + the on_audio hand-off, engine.cpp:480-502).
//             Called on the worker thread.  A decode failure ends the job the way a failing
//             sink does (Cancelled), with the codec's message as the job's error.
// The runtime converts the audio to int16 as the reference's to_pcm16 does (runtime.cpp,
// capi.cpp:29-32: clamp to [-1, 1], lrintf(v * 32767)) and hands it to the job's PcmSink with
// the count of sample frames (runtime.h:83); a sink returning false cancels the job.
//
// Request: the reference's moss::JobRequest, or any struct with its members (id, text, voice,
// profile, seed, greedy, max_frames, chunk_frames, min_frames, temperature, top_k, top_p,
// repetition_penalty).  Zero sampling fields take the engine defaults, as run_job does
// (runtime.cpp:346-357).  The request's `pace` (sleeping between audio blocks to stay a fixed
// time ahead of playback) is not applied: one job sleeping would hold back every job in its
// batch; a paced client is served from the sink side instead.
#pragma once

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "batch_runtime.h"

namespace moss {
namespace gpu {

// What a front end produces for one request.
struct TextJob {
    std::vector<std::vector<FrameRow>> segments;  // suffix rows [m][17] per text segment
    int prefix_stream = -1;                       // engine stream of the voice prefix, or -1
    int prefix_len = 0;                           // its positions (fork length)
    int text_tokens = 0;                          // SentencePiece tokens of the text
    bool cache_hit = false;                       // the voice prefix came from the prefix cache
};

using PcmSink = std::function<bool(const int16_t *pcm, int frames)>;  // runtime.h:83

struct TextJobInfo {  // runtime.h:64-77
    std::string id;
    GenJobState state = GenJobState::Queued;
    int frames = 0;             // LLM frames decoded to audio
    double audio_ms = 0.0;
    double compute_ms = 0.0;    // wall time minus the time spent inside the sink
    double wall_ms = 0.0;       // submit to end
    double first_pcm_ms = -1.0; // submit() call to the first audio handed to the sink
    double rtf = 0.0;           // compute_ms / audio_ms
    int text_tokens = 0;
    bool cache_hit = false;
    std::string error;
};

inline int16_t to_pcm16(float v) {  // runtime.cpp / capi.cpp:29-32
    const float c = v < -1.0f ? -1.0f : (v > 1.0f ? 1.0f : v);
    return static_cast<int16_t>(std::lrintf(c * 32767.0f));
}

template <class Ops, class Frontend, class Codec>
class TextJobRuntime {
    using Clock = std::chrono::steady_clock;
    using Stream = typename decltype(std::declval<Codec &>().open())::element_type;

public:
    static constexpr int kSampleRate = 48000;

    TextJobRuntime(Ops &ops, Frontend &frontend, Codec &codec, BatchRuntimeOptions opt)
        : frontend_(frontend), codec_(codec), rt_(ops, opt) {}
    ~TextJobRuntime() { shutdown(); }

    void start() { rt_.start(); }
    void shutdown() { rt_.shutdown(); }
    bool run_once() { return rt_.run_once(); }

    template <class Request>
    bool submit(const Request &req, PcmSink sink, std::string *job_id, std::string *err) {
        TextJob tj;
        std::string why;
        if (!frontend_.prepare(req.text, req.voice, req.profile, &tj, &why)) {
            if (err) *err = why.empty() ? "front end failed" : why;
            return false;
        }
        GenJobRequest g;
        g.id = req.id;
        g.segments = std::move(tj.segments);
        g.prefix_stream = tj.prefix_stream;
        g.prefix_len = tj.prefix_len;
        g.seed = req.seed;
        g.greedy = req.greedy;
        g.max_frames = req.max_frames;
        g.chunk_frames = req.chunk_frames;
        g.min_frames = req.min_frames;
        g.temperature = req.temperature;
        g.top_k = req.top_k;
        g.top_p = req.top_p;
        g.repetition_penalty = req.repetition_penalty;
        auto a = std::make_shared<Audio>();
        a->decoder = codec_.open();
        a->sink = std::move(sink);
        a->text_tokens = tj.text_tokens;
        a->cache_hit = tj.cache_hit;
        a->submitted = Clock::now();
        if (!a->decoder) {
            if (err) *err = "codec failed to open a stream";
            return false;
        }
        // the worker hands each code block to the job's decoder, then its PCM to the sink
        CodeSink code_sink = [a](int segment, const int32_t *codes, int n) { return a->deliver(segment, codes, n); };
        std::string id;
        if (!rt_.submit(g, std::move(code_sink), &id, err)) return false;
        {
            std::lock_guard<std::mutex> lock(mutex_);
            audio_[id] = a;
            prune_locked();
        }
        if (job_id) *job_id = id;
        return true;
    }

    bool wait(const std::string &id, int timeout_ms, TextJobInfo *out) {
        GenJobInfo g;
        const bool ended = rt_.wait(id, timeout_ms, &g);
        if (!ended && g.id.empty()) return false;  // unknown job
        if (out) fill(g, out);
        return ended;
    }
    bool job(const std::string &id, TextJobInfo *out) const {
        GenJobInfo g;
        if (!rt_.job(id, &g)) return false;
        if (out) fill(g, out);
        return true;
    }
    bool cancel(const std::string &id) { return rt_.cancel(id); }
    int queue_depth() const { return rt_.queue_depth(); }
    int max_queue() const { return rt_.max_queue(); }

private:
    struct Audio {
        std::unique_ptr<Stream> decoder;
        PcmSink sink;
        int text_tokens = 0;
        bool cache_hit = false;
        Clock::time_point submitted;
        mutable std::mutex mu;  // the worker writes the counters, wait()/job() read them
        int frames = 0;
        int64_t samples = 0;
        double sink_ms = 0.0, first_pcm_ms = -1.0;
        std::string error;
        std::vector<float> buf;
        std::vector<int16_t> pcm;

        bool deliver(int segment, const int32_t *codes, int n) {
            buf.clear();
            std::string why;
            if (!decoder->decode(segment, codes, n, &buf, &why)) {
                std::lock_guard<std::mutex> lock(mu);
                error = why.empty() ? "codec failed" : why;
                return false;
            }
            const int sframes = static_cast<int>(buf.size() / 2);
            pcm.resize(buf.size());
            for (size_t i = 0; i < buf.size(); ++i) pcm[i] = to_pcm16(buf[i]);
            const auto t0 = Clock::now();
            {
                std::lock_guard<std::mutex> lock(mu);
                frames += n;
                samples += sframes;
                if (first_pcm_ms < 0.0 && sframes > 0)
                    first_pcm_ms = std::chrono::duration<double, std::milli>(t0 - submitted).count();
            }
            const bool ok = sframes <= 0 || !sink || sink(pcm.data(), sframes);
            std::lock_guard<std::mutex> lock(mu);
            sink_ms += std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
            return ok;
        }
    };

    void fill(const GenJobInfo &g, TextJobInfo *out) const {
        out->id = g.id;
        out->state = g.state;
        out->wall_ms = g.wall_ms;
        out->error = g.error;
        std::shared_ptr<Audio> a;
        {
            std::lock_guard<std::mutex> lock(mutex_);
            auto it = audio_.find(g.id);
            if (it != audio_.end()) a = it->second;
        }
        if (!a) return;
        std::lock_guard<std::mutex> lock(a->mu);
        out->frames = a->frames;
        out->audio_ms = 1000.0 * static_cast<double>(a->samples) / kSampleRate;
        out->first_pcm_ms = a->first_pcm_ms;
        out->text_tokens = a->text_tokens;
        out->cache_hit = a->cache_hit;
        if (g.wall_ms > 0.0) out->compute_ms = std::max(0.0, g.wall_ms - a->sink_ms);
        out->rtf = out->audio_ms > 0.0 ? out->compute_ms / out->audio_ms : 0.0;
        if (!a->error.empty()) out->error = a->error;  // the codec's reason, not just "cancelled"
    }

    // keep the audio state of about as many jobs as the batch runtime keeps records of
    void prune_locked() {
        while (static_cast<int>(audio_.size()) > 4 * BatchRuntime<Ops>::kKeepJobs) {
            auto oldest = audio_.begin();
            for (auto it = audio_.begin(); it != audio_.end(); ++it)
                if (it->second->submitted < oldest->second->submitted) oldest = it;
            audio_.erase(oldest);
        }
    }

    Frontend &frontend_;
    Codec &codec_;
    BatchRuntime<Ops> rt_;
    mutable std::mutex mutex_;
    std::map<std::string, std::shared_ptr<Audio>> audio_;
};

}  // namespace gpu
}  // namespace moss
