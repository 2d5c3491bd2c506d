// fake_engine.h -- a host-only double of the engine's C ABI (the Ops interface of
// batch_runtime.h) and a sequential restatement of TtsEngine::synthesize's token loop over it,
// shared by the runtime tests.  The double's codes and end gate depend only on a stream's own
// contents, the frame index, the sampling parameters and the seed, so a job produces the same
// blocks however a runtime batches it.
#pragma once

#include <algorithm>
#include <array>
#include <cstdint>
#include <string>
#include <vector>

#include "batch_runtime.h"

namespace fake {

using namespace moss::gpu;

inline uint64_t mix(uint64_t h, uint64_t v) {
    h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    return h * 0x100000001B3ull;
}

struct FakeOps {
    struct Stream {
        bool open = false;
        std::vector<uint64_t> toks;  // one entry per position
        uint64_t seed = 0;
        int frame = 0;
    };
    explicit FakeOps(int streams, int ctx) : s(static_cast<size_t>(streams)), ctx_(ctx) {}
    std::vector<Stream> s;
    int ctx_;
    std::string err;
    std::vector<int> prefill_n, step_n, step_frames_n;

    bool bad(int sid) const { return sid < 0 || sid >= static_cast<int>(s.size()) || !s[static_cast<size_t>(sid)].open; }
    int fail(const char *why) {
        err = why;
        return 1;
    }
    int open(int *sid) {
        for (size_t i = 0; i < s.size(); ++i)
            if (!s[i].open) {
                s[i] = Stream{};
                s[i].open = true;
                *sid = static_cast<int>(i);
                return 0;
            }
        return fail("no free stream slot");
    }
    int fork(int src, int n_pos, int *sid) {
        if (bad(src) || n_pos > static_cast<int>(s[static_cast<size_t>(src)].toks.size())) return fail("bad fork");
        if (open(sid)) return 1;
        auto &t = s[static_cast<size_t>(src)].toks;
        s[static_cast<size_t>(*sid)].toks.assign(t.begin(), t.begin() + n_pos);
        return 0;
    }
    int close(int sid) {
        if (bad(sid)) return fail("stream not open");
        s[static_cast<size_t>(sid)] = Stream{};
        return 0;
    }
    int position(int sid, int *pos) {
        if (bad(sid)) return fail("stream not open");
        *pos = static_cast<int>(s[static_cast<size_t>(sid)].toks.size());
        return 0;
    }
    int prefill_batch(int n, const int32_t *sids, const int32_t *m, const int32_t *start, const int32_t *rows) {
        size_t k = 0;
        for (int i = 0; i < n; ++i) {  // validate everything first: nothing changes on failure
            if (bad(sids[i])) return fail("stream not open");
            if (start[i] != static_cast<int>(s[static_cast<size_t>(sids[i])].toks.size())) return fail("bad start");
            if (start[i] + m[i] > ctx_) return fail("context full");
            for (int r = 0; r < m[i]; ++r, ++k)
                if (rows[k * 17] < 0 || rows[k * 17] >= 16384) return fail("text id out of range");
        }
        k = 0;
        for (int i = 0; i < n; ++i)
            for (int r = 0; r < m[i]; ++r, ++k) {
                uint64_t h = 1469598103934665603ull;
                for (int c = 0; c < 17; ++c) h = mix(h, static_cast<uint64_t>(rows[k * 17 + c]) + 1);
                s[static_cast<size_t>(sids[i])].toks.push_back(h);
            }
        prefill_n.push_back(n);
        return 0;
    }
    int generate_begin(int sid, uint64_t seed) {
        if (bad(sid)) return fail("stream not open");
        s[static_cast<size_t>(sid)].seed = seed;
        s[static_cast<size_t>(sid)].frame = 0;
        return 0;
    }
    int step_frames(const int32_t *sids, int n, const mossgpu_sample_params &p, int frames, int32_t *codes,
                    int32_t *done) {
        if (frames < 1 || frames > 1024) return fail("bad frame count");
        for (int i = 0; i < n; ++i) {
            if (bad(sids[i])) return fail("stream not open");
            if (static_cast<int>(s[static_cast<size_t>(sids[i])].toks.size()) + frames > ctx_) return fail("context full");
        }
        const uint64_t pk = static_cast<uint64_t>(p.greedy) * 5 + static_cast<uint64_t>(p.repetition_penalty * 1000.0f) * 7 +
                            static_cast<uint64_t>(p.min_frames) * 11 + static_cast<uint64_t>(p.top_k) * 13;
        for (int i = 0; i < n; ++i) {
            Stream &st = s[static_cast<size_t>(sids[i])];
            int f = 0;
            for (; f < frames; ++f) {
                uint64_t h = 1469598103934665603ull;
                for (uint64_t t : st.toks) h = mix(h, t);
                h = mix(mix(h, st.seed), pk);
                if (st.frame >= p.min_frames && (h >> 11) % 9 == 0) break;  // the end gate
                uint64_t row = h;
                for (int ch = 0; ch < 16; ++ch) {
                    const int32_t c = static_cast<int32_t>(mix(h, static_cast<uint64_t>(ch) * 131 + static_cast<uint64_t>(st.frame)) % 1024);
                    codes[(static_cast<size_t>(f) * n + i) * 16 + ch] = c;
                    row = mix(row, static_cast<uint64_t>(c));
                }
                st.toks.push_back(row);
                ++st.frame;
            }
            for (int g = f; g < frames; ++g)
                for (int ch = 0; ch < 16; ++ch) codes[(static_cast<size_t>(g) * n + i) * 16 + ch] = -1;
            done[i] = f;
        }
        step_n.push_back(n);
        step_frames_n.push_back(frames);
        return 0;
    }
    const char *last_error() { return err.c_str(); }
    int max_ctx() const { return ctx_; }
    int open_streams() const {
        int c = 0;
        for (auto &x : s) c += x.open ? 1 : 0;
        return c;
    }
};

struct Block {
    int segment;
    std::vector<int32_t> codes;  // [16][n]
    bool operator==(const Block &o) const { return segment == o.segment && codes == o.codes; }
};

inline std::vector<FrameRow> rows_of(int m, uint64_t seed, int bad_row = -1) {
    std::vector<FrameRow> out(static_cast<size_t>(m));
    uint64_t h = seed * 7919 + 1;
    for (int r = 0; r < m; ++r) {
        h = mix(h, static_cast<uint64_t>(r));
        out[static_cast<size_t>(r)][0] = r == bad_row ? 16384 : static_cast<int32_t>(h % 16384);
        for (int c = 1; c < 17; ++c) out[static_cast<size_t>(r)][static_cast<size_t>(c)] = static_cast<int32_t>(mix(h, static_cast<uint64_t>(c)) % 1025);
    }
    return out;
}

inline mossgpu_sample_params params_of(const GenJobRequest &r) {
    mossgpu_sample_params p{};
    p.greedy = r.greedy;
    p.temperature = r.temperature > 0 ? r.temperature : 0.8f;
    p.top_k = r.top_k > 0 ? r.top_k : 25;
    p.top_p = r.top_p > 0 ? r.top_p : 0.95f;
    p.repetition_penalty = r.repetition_penalty > 0 ? r.repetition_penalty : 1.2f;
    p.end_greedy = 1;
    p.min_frames = r.min_frames;
    p.greedy_frames = r.greedy_frames;
    return p;
}

// synthesize's loop, one frame per call, on its own engine double
inline std::vector<Block> expected_blocks(FakeOps &eng, const GenJobRequest &r) {
    std::vector<Block> out;
    const int chunk = r.chunk_frames > 0 ? r.chunk_frames : 8;
    const int max_frames = r.max_frames > 0 ? r.max_frames : 375;
    const mossgpu_sample_params p = params_of(r);
    int frames_total = 0;
    for (size_t si = 0; si < r.segments.size(); ++si) {
        const auto &seg = r.segments[si];
        if (seg.empty()) continue;
        int sid = -1;
        if (r.prefix_stream >= 0)
            eng.fork(r.prefix_stream, r.prefix_len, &sid);
        else
            eng.open(&sid);
        const int32_t m = static_cast<int32_t>(seg.size()), st = r.prefix_stream >= 0 ? r.prefix_len : 0;
        std::vector<int32_t> flat;
        for (auto &row : seg) flat.insert(flat.end(), row.begin(), row.end());
        if (eng.prefill_batch(1, &sid, &m, &st, flat.data()) != 0) {
            eng.close(sid);
            return {};
        }
        eng.generate_begin(sid, r.seed);
        std::vector<std::array<int32_t, 16>> pending;
        auto decode_pending = [&](bool force) {
            const size_t want = frames_total == 0 ? std::min<size_t>(4, static_cast<size_t>(chunk)) : static_cast<size_t>(chunk);
            const size_t n = pending.size();
            if (n == 0 || (!force && n < want)) return;
            Block b{static_cast<int>(si), std::vector<int32_t>(16 * n)};
            for (size_t ch = 0; ch < 16; ++ch)
                for (size_t j = 0; j < n; ++j) b.codes[ch * n + j] = pending[j][ch];
            out.push_back(b);
            frames_total += static_cast<int>(n);
            pending.clear();
        };
        for (int f = 0; f < max_frames; ++f) {
            int pos = 0;
            eng.position(sid, &pos);
            if (pos >= eng.max_ctx()) break;
            int32_t codes[16], done = 0;
            eng.step_frames(&sid, 1, p, 1, codes, &done);
            if (done == 0) break;
            std::array<int32_t, 16> c{};
            std::copy(codes, codes + 16, c.begin());
            pending.push_back(c);
            decode_pending(false);
        }
        decode_pending(true);
        eng.close(sid);
    }
    return out;
}

inline int setup_prefix(FakeOps &eng, int m) {
    int sid = -1;
    eng.open(&sid);
    auto rows = rows_of(m, 999);
    std::vector<int32_t> flat;
    for (auto &row : rows) flat.insert(flat.end(), row.begin(), row.end());
    const int32_t mm = m, st = 0;
    eng.prefill_batch(1, &sid, &mm, &st, flat.data());
    eng.prefill_n.clear();
    return sid;
}

}  // namespace fake
