// TextJobRuntime::submit takes the reference's own request type: this file includes the
// reference's runtime.h (through dsh-moss-tts_b200/csrc/dropin, so its engine.h sees the GPU
// LlmModel), fills a moss::JobRequest and a moss::PcmSink as the reference's transports do,
// and runs the job over the engine double.  Exit 0 = the job completed with audio.
#include "moss/runtime.h"

#include <cstdio>

#include "fake_engine.h"
#include "job_runtime.h"

namespace {

struct Frontend {
    bool prepare(const std::string &text, const std::string &, const std::string &, moss::gpu::TextJob *out,
                 std::string *) {
        out->segments.push_back(fake::rows_of(4 + static_cast<int>(text.size() % 7), 5));
        out->text_tokens = 1;
        return true;
    }
};

struct Codec {
    struct Stream {
        bool decode(int, const int32_t *codes, int n, std::vector<float> *audio, std::string *) {
            for (int j = 0; j < 2 * n; ++j) audio->push_back(static_cast<float>(codes[j % n] % 100) / 100.0f);
            return true;
        }
    };
    std::unique_ptr<Stream> open() { return std::make_unique<Stream>(); }
};

}  // namespace

int main() {
    fake::FakeOps eng(4, 4096);
    Frontend fe;
    Codec codec;
    moss::gpu::TextJobRuntime<fake::FakeOps, Frontend, Codec> rt(eng, fe, codec, moss::gpu::BatchRuntimeOptions{});
    moss::JobRequest req;  // runtime.h:45-62, defaults as a transport leaves them
    req.text = "hello";
    req.greedy = true;
    req.min_frames = 3;
    int got = 0;
    moss::PcmSink sink = [&](const int16_t *, int frames) {
        got += frames;
        return true;
    };
    std::string id, err;
    if (!rt.submit(req, sink, &id, &err)) {
        std::printf("submit failed: %s\n", err.c_str());
        return 1;
    }
    while (rt.run_once()) {
    }
    moss::gpu::TextJobInfo info;
    if (!rt.job(id, &info) || info.state != moss::gpu::GenJobState::Completed || got <= 0 || info.frames < 3) {
        std::printf("job %s: %s frames %d audio frames %d\n", id.c_str(), moss::gpu::gen_job_state_name(info.state),
                    info.frames, got);
        return 1;
    }
    std::printf("ok frames=%d pcm_frames=%d\n", info.frames, got);
    return 0;
}
