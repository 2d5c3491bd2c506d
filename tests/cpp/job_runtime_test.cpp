// TextJobRuntime (job_runtime.h): the reference Runtime's text-level submit / wait / job /
// cancel (runtime.h:92-113) over BatchRuntime, on the host-only engine double with a test
// front end (text -> suffix rows per segment, voice -> prefix stream) and a test codec (code
// blocks -> stereo float audio).  Expected PCM: the same requests turned into token jobs by
// the same front end, run through the sequential restatement of synthesize's loop, each block
// decoded by a fresh codec stream and converted as the reference's to_pcm16.
// Exit 0 = all checks passed; failures print and exit 1.
#include "job_runtime.h"

#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "fake_engine.h"

using namespace moss::gpu;
using namespace fake;

namespace {

int g_failures = 0;
#define CHECK(cond, ...)                                     \
    do {                                                     \
        if (!(cond)) {                                       \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                        \
            std::printf("\n");                               \
            ++g_failures;                                    \
        }                                                    \
    } while (0)

// The members of the reference's moss::JobRequest (runtime.h:45-62).
struct Req {
    std::string id, text, voice, profile;
    uint64_t seed = 0;
    bool greedy = false;
    int max_frames = 375, chunk_frames = 8, min_frames = 0;
    float temperature = 0.0f;
    int top_k = 0;
    float top_p = 0.0f, repetition_penalty = 0.0f;
    double pace = 0.0;
};

uint64_t hash_text(const std::string &t) {
    uint64_t h = 1469598103934665603ull;
    for (unsigned char c : t) h = mix(h, c);
    return h;
}

// Segments are separated by '|'; a segment's rows follow from its text; words count as tokens.
struct Frontend {
    std::map<std::string, std::pair<int, int>> voices;  // name -> (prefix stream, positions)
    bool prepare(const std::string &text, const std::string &voice, const std::string &profile, TextJob *out,
                 std::string *err) {
        const std::string v = profile.empty() ? voice : profile;
        if (!v.empty()) {
            auto it = voices.find(v);
            if (it == voices.end()) {
                *err = "unknown voice " + v;
                return false;
            }
            out->prefix_stream = it->second.first;
            out->prefix_len = it->second.second;
            out->cache_hit = true;
        }
        size_t a = 0;
        for (;;) {
            const size_t b = text.find('|', a);
            const std::string seg = text.substr(a, b == std::string::npos ? std::string::npos : b - a);
            out->segments.push_back(seg.empty() ? std::vector<FrameRow>{}
                                                : rows_of(3 + static_cast<int>(seg.size() % 13), hash_text(seg)));
            for (size_t i = 0; i < seg.size(); ++i)
                if (seg[i] != ' ' && (i == 0 || seg[i - 1] == ' ')) ++out->text_tokens;
            if (b == std::string::npos) break;
            a = b + 1;
        }
        return true;
    }
};

// Four stereo sample frames per LLM frame; values beyond [-1, 1] exercise the clamp.
struct Codec {
    struct Stream {
        bool fail = false;
        bool decode(int segment, const int32_t *codes, int n, std::vector<float> *audio, std::string *err) {
            if (fail) {
                *err = "codec: bad block";
                return false;
            }
            for (int j = 0; j < n; ++j)
                for (int k = 0; k < 4; ++k) {
                    const float v = static_cast<float>((codes[j] + codes[15 * n + j] + 7 * k + segment) % 300 - 150) / 100.0f;
                    audio->push_back(v);
                    audio->push_back(-0.5f * v);
                }
            return true;
        }
    };
    bool fail_next = false;
    std::unique_ptr<Stream> open() {
        auto s = std::make_unique<Stream>();
        s->fail = fail_next;
        fail_next = false;
        return s;
    }
};

GenJobRequest token_job(Frontend &fe, const Req &r) {
    TextJob tj;
    std::string err;
    fe.prepare(r.text, r.voice, r.profile, &tj, &err);
    GenJobRequest g;
    g.segments = tj.segments;
    g.prefix_stream = tj.prefix_stream;
    g.prefix_len = tj.prefix_len;
    g.seed = r.seed;
    g.greedy = r.greedy;
    g.max_frames = r.max_frames;
    g.chunk_frames = r.chunk_frames;
    g.min_frames = r.min_frames;
    g.temperature = r.temperature;
    g.top_k = r.top_k;
    g.top_p = r.top_p;
    g.repetition_penalty = r.repetition_penalty;
    return g;
}

std::vector<int16_t> expected_pcm(FakeOps &ref, Frontend &fe, const Req &r, int *frames) {
    std::vector<int16_t> pcm;
    Codec codec;
    auto dec = codec.open();
    *frames = 0;
    for (const Block &b : expected_blocks(ref, token_job(fe, r))) {
        const int n = static_cast<int>(b.codes.size() / 16);
        std::vector<float> audio;
        std::string err;
        dec->decode(b.segment, b.codes.data(), n, &audio, &err);
        for (float v : audio) pcm.push_back(to_pcm16(v));
        *frames += n;
    }
    return pcm;
}

struct Sinks {
    std::mutex mu;
    std::map<std::string, std::vector<int16_t>> pcm;
    std::map<std::string, int> calls;
    PcmSink make(const std::string &key, int fail_after = -1) {
        return [this, key, fail_after](const int16_t *p, int frames) {
            std::lock_guard<std::mutex> lock(mu);
            auto &v = pcm[key];
            v.insert(v.end(), p, p + 2 * frames);
            return fail_after < 0 || ++calls[key] <= fail_after;
        };
    }
};

void test_text_jobs_match_sequential_synthesis() {
    FakeOps eng(24, 4096), ref(24, 4096);
    const int psid = setup_prefix(eng, 20), rsid = setup_prefix(ref, 20);
    CHECK(psid == rsid, "prefix stream ids differ");
    Frontend fe, fe_ref;
    fe.voices["alice"] = fe_ref.voices["alice"] = {psid, 20};
    fe.voices["p/bob.mossclone"] = fe_ref.voices["p/bob.mossclone"] = {psid, 17};
    Codec codec;
    TextJobRuntime<FakeOps, Frontend, Codec> rt(eng, fe, codec, BatchRuntimeOptions{8, 64, 4});
    std::vector<Req> reqs;
    for (int i = 0; i < 10; ++i) {
        Req r;
        r.text = "segment one " + std::to_string(i) + (i % 3 ? "|second part here" : "") + (i == 5 ? "||tail" : "");
        r.voice = i % 2 ? "alice" : "";
        if (i == 7) r.profile = "p/bob.mossclone";
        r.seed = 40 + static_cast<uint64_t>(i);
        r.greedy = i % 2 == 0;
        r.max_frames = i % 3 == 0 ? 6 : 30;
        r.chunk_frames = i % 4 == 0 ? 0 : 1 + i % 5;
        r.repetition_penalty = i % 4 == 1 ? 1.1f : 0.0f;
        r.min_frames = i % 5 == 0 ? 2 : 0;
        r.pace = i == 3 ? 0.5 : 0.0;
        reqs.push_back(r);
    }
    Sinks sinks;
    std::vector<std::string> ids;
    for (size_t i = 0; i < reqs.size(); ++i) {
        std::string id, err;
        CHECK(rt.submit(reqs[i], sinks.make("j" + std::to_string(i)), &id, &err), "submit %zu: %s", i, err.c_str());
        ids.push_back(id);
    }
    rt.start();
    for (size_t i = 0; i < reqs.size(); ++i) {
        TextJobInfo info;
        CHECK(rt.wait(ids[i], 20000, &info), "job %zu did not end", i);
        CHECK(info.state == GenJobState::Completed, "job %zu: %s %s", i, gen_job_state_name(info.state),
              info.error.c_str());
        int frames = 0;
        const auto want = expected_pcm(ref, fe_ref, reqs[i], &frames);
        std::lock_guard<std::mutex> lock(sinks.mu);
        CHECK(sinks.pcm["j" + std::to_string(i)] == want, "job %zu: %zu samples, expected %zu", i,
              sinks.pcm["j" + std::to_string(i)].size(), want.size());
        CHECK(info.frames == frames, "job %zu frames %d vs %d", i, info.frames, frames);
        CHECK(std::abs(info.audio_ms - 1000.0 * static_cast<double>(want.size() / 2) / 48000.0) < 1e-6,
              "job %zu audio_ms %f", i, info.audio_ms);
        // a job whose gate ends it before any frame has no first audio (-1), as the reference
        CHECK(info.text_tokens > 0 && (frames == 0 ? info.first_pcm_ms < 0.0 : info.first_pcm_ms >= 0.0) &&
                  info.wall_ms + 1.0 >= info.first_pcm_ms,
              "job %zu stats: tokens %d first_pcm %f wall %f frames %d", i, info.text_tokens, info.first_pcm_ms,
              info.wall_ms, info.frames);
        CHECK(info.cache_hit == (!reqs[i].voice.empty() || !reqs[i].profile.empty()), "job %zu cache_hit", i);
    }
    rt.shutdown();
    CHECK(eng.open_streams() == 1, "streams left open: %d", eng.open_streams() - 1);
    std::printf("A jobs=%zu\n", reqs.size());
}

void test_errors_cancel_and_failures() {
    FakeOps eng(8, 4096);
    Frontend fe;
    Codec codec;
    TextJobRuntime<FakeOps, Frontend, Codec> rt(eng, fe, codec, BatchRuntimeOptions{4, 2, 4});
    std::string id, err;
    Req r;
    r.text = "hello there";
    r.voice = "nobody";
    CHECK(!rt.submit(r, nullptr, &id, &err) && err == "unknown voice nobody", "unknown voice: %s", err.c_str());
    r.voice = "";
    r.max_frames = 200;
    r.min_frames = 200;  // the double's gate cannot end it early
    Sinks sinks;
    std::string sink_fail, codec_fail, queued;
    CHECK(rt.submit(r, sinks.make("s", 2), &sink_fail, &err), "submit: %s", err.c_str());
    codec.fail_next = true;
    CHECK(rt.submit(r, sinks.make("c"), &codec_fail, &err), "submit: %s", err.c_str());
    CHECK(!rt.submit(r, sinks.make("q"), &queued, &err) && err == "busy", "queue limit: %s", err.c_str());
    for (int it = 0; it < 10000 && rt.run_once(); ++it) {
    }
    TextJobInfo a, b;
    CHECK(rt.job(sink_fail, &a) && a.state == GenJobState::Cancelled, "failing sink: %s", gen_job_state_name(a.state));
    CHECK(rt.job(codec_fail, &b) && b.state == GenJobState::Cancelled && b.error == "codec: bad block",
          "failing codec: %s %s", gen_job_state_name(b.state), b.error.c_str());
    {
        std::lock_guard<std::mutex> lock(sinks.mu);
        CHECK(sinks.calls["s"] == 3, "the sink saw %d blocks", sinks.calls["s"]);
        CHECK(sinks.pcm["c"].empty(), "a failing codec produced audio");
    }
    CHECK(rt.submit(r, sinks.make("x"), &id, &err), "submit after: %s", err.c_str());
    CHECK(rt.cancel(id), "cancel");
    for (int it = 0; it < 10000 && rt.run_once(); ++it) {
    }
    TextJobInfo c;
    CHECK(rt.job(id, &c) && c.state == GenJobState::Cancelled, "cancelled job: %s", gen_job_state_name(c.state));
    CHECK(!rt.job("no-such-job", &c) && !rt.wait("no-such-job", 0, &c), "unknown job id");
    CHECK(eng.open_streams() == 0, "streams left open: %d", eng.open_streams());
    std::printf("B ok\n");
}

}  // namespace

int main() {
    test_text_jobs_match_sequential_synthesis();
    test_errors_cancel_and_failures();
    if (g_failures) {
        std::printf("%d failure(s)\n", g_failures);
        return 1;
    }
    return 0;
}
