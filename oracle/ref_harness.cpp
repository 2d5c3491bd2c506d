// ref_harness.cpp -- C entry points over the reference's own moss::LlmModel.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with the
// reference's sources (read in place from the reference checkout, never copied) into
// oracle/_ref/libmossref.so.  It is used to pin the C restatement (moss_oracle.c) and as
// the "reference" CPU baseline in bench.py.  It drives LlmModel through its public API
// (prefill, generate, set_logits_dump, position, hidden) and, to inject a KV state or an
// embedding directly (the reference CLI only takes token rows), through its private
// members -- llm.h is included with `private` mapped to `public` in this translation unit
// only; the class layout is unchanged.
#include <algorithm>
#include <array>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>
#include <barrier>
#include <condition_variable>
#include <mutex>
#include <thread>

#define private public
#include "moss/llm.h"
#undef private
#include "moss/quant.h"
#include "moss/gemv.h"
#include "moss/sampler.h"
#include "moss/fp16.h"
#include "moss/decoder.h"

using namespace moss;

extern "C" {

int ref_max_ctx() { return kMaxCtx; }

// MOSS_A16 is read once per process (gemv.cpp:26-35); set it before the first model call.
void ref_set_a16_env(const char *mode) { setenv("MOSS_A16", mode, 1); }

void *ref_create(const char *path, int threads) {
    auto *m = new LlmModel(threads);
    std::string err;
    if (!m->load(path, &err)) {
        std::fprintf(stderr, "ref_create: %s\n", err.c_str());
        delete m;
        return nullptr;
    }
    return m;
}

void ref_destroy(void *h) { delete static_cast<LlmModel *>(h); }

int ref_position(void *h) { return static_cast<LlmModel *>(h)->position(); }

void ref_hidden(void *h, float *out) { std::memcpy(out, static_cast<LlmModel *>(h)->hidden(), sizeof(float) * kHidden); }

void ref_prefill_rows(void *h, const int32_t *rows, int n, int start) {
    std::vector<Row> r(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < kNVq + 1; ++j) r[i][j] = rows[static_cast<size_t>(i) * 17 + j];
    static_cast<LlmModel *>(h)->prefill(r, start);
}

// LlmModel::save_prefix (llm.cpp:485-509): the reference's own .mosskv writer, for the
// prefix-file interchange fixture.  Returns 1 on success.
int ref_save_prefix(void *h, const char *path, const int32_t *rows, int n) {
    std::vector<Row> r(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < kNVq + 1; ++j) r[i][j] = rows[static_cast<size_t>(i) * 17 + j];
    std::string err;
    return static_cast<LlmModel *>(h)->save_prefix(path, r, &err) ? 1 : 0;
}

// LlmModel::save_state (llm.cpp:561-587): the reference's state-file writer.  Returns 1 on success.
int ref_save_state(void *h, const char *path, const int32_t *rows, int n) {
    std::vector<Row> r(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < kNVq + 1; ++j) r[i][j] = rows[static_cast<size_t>(i) * 17 + j];
    std::string err;
    return static_cast<LlmModel *>(h)->save_state(path, r, &err) ? 1 : 0;
}

// llm.cpp:588-632 semantics (state injection) without the file round trip
int ref_set_state(void *h, const float *k, const float *v, int n_pos, const float *hidden) {
    auto *m = static_cast<LlmModel *>(h);
    if (n_pos <= 0 || n_pos > kMaxCtx) return 0;
    for (int l = 0; l < 12; ++l) {
        const size_t dst = static_cast<size_t>(l) * kMaxCtx * kHidden;
        const size_t src = static_cast<size_t>(l) * n_pos * kHidden;
        std::memcpy(m->g_k_.data() + dst, k + src, sizeof(float) * n_pos * kHidden);
        std::memcpy(m->g_v_.data() + dst, v + src, sizeof(float) * n_pos * kHidden);
    }
    if (hidden) std::memcpy(m->hidden_.data(), hidden, sizeof(float) * kHidden);
    m->pos_ = n_pos;
    return 1;
}

void ref_get_kv(void *h, int layer, int p0, int n, float *k, float *v) {
    auto *m = static_cast<LlmModel *>(h);
    const size_t base = (static_cast<size_t>(layer) * kMaxCtx + p0) * kHidden;
    if (k) std::memcpy(k, m->g_k_.data() + base, sizeof(float) * n * kHidden);
    if (v) std::memcpy(v, m->g_v_.data() + base, sizeof(float) * n * kHidden);
}

// global_step (llm.cpp:248-255) with x_ given directly
void ref_global_step_embed(void *h, const float *x, float *hidden_out) {
    auto *m = static_cast<LlmModel *>(h);
    std::memcpy(m->x_.data(), x, sizeof(float) * kHidden);
    for (int i = 0; i < 12; ++i)
        m->block_forward(m->global_layers_[i], false, i, m->pos_, m->x_.data(), m->qkv_.data(), m->attn_buf_.data(),
                         m->mlp_buf_.data());
    m->normalize(m->x_.data(), m->lnf_w_, m->lnf_b_, m->hidden_.data());
    ++m->pos_;
    if (hidden_out) std::memcpy(hidden_out, m->hidden_.data(), sizeof(float) * kHidden);
}

void ref_global_step_row(void *h, const int32_t *row17, float *hidden_out) {
    auto *m = static_cast<LlmModel *>(h);
    Row r{};
    for (int j = 0; j < 17; ++j) r[j] = row17[j];
    m->global_step(r, m->hidden_.data());
    if (hidden_out) std::memcpy(hidden_out, m->hidden_.data(), sizeof(float) * kHidden);
}

void ref_embed_row(void *h, const int32_t *row17, float *out) {
    Row r{};
    for (int j = 0; j < 17; ++j) r[j] = row17[j];
    static_cast<LlmModel *>(h)->embed_row(r, out);
}

// One local step at an explicit local position (llm.cpp:257-264)
void ref_local_step(void *h, int lpos, const float *input, float *out) {
    auto *m = static_cast<LlmModel *>(h);
    m->lpos_ = lpos;
    m->local_step(input, out);
}

void ref_audio_logits(void *h, int ch, const float *hidden, float *logits) {
    static_cast<LlmModel *>(h)->audio_logits(ch, hidden, logits);
}

void ref_assistant_logits(void *h, const float *hidden, float *pair) {
    static_cast<LlmModel *>(h)->assistant_logits(hidden, pair);
}

// generate (llm.cpp:634-733).  forced [max_frames][16] or NULL; codes [max_frames][16];
// logits [max_frames][16][1024] or NULL (read from the model's own dump buffer).
int ref_generate(void *h, int max_frames, int greedy, float temperature, int top_k, float top_p, float rep,
                 int end_greedy, int min_frames, int greedy_frames, uint64_t seed, const int32_t *forced,
                 int32_t *codes, float *logits, const char *logits_tmp_path) {
    auto *m = static_cast<LlmModel *>(h);
    SampleParams p;
    p.greedy = greedy != 0;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repetition_penalty = rep;
    p.end_greedy = end_greedy != 0;
    p.min_frames = min_frames;
    p.greedy_frames = greedy_frames;
    std::vector<Row> f;
    if (forced) {
        f.resize(static_cast<size_t>(max_frames));
        for (int i = 0; i < max_frames; ++i) {
            f[i][0] = kSlotToken;
            for (int ch = 0; ch < kNVq; ++ch) f[i][ch + 1] = forced[static_cast<size_t>(i) * kNVq + ch];
        }
    }
    m->logits_dump_.clear();
    if (logits && logits_tmp_path) m->set_logits_dump(logits_tmp_path);
    const std::vector<Row> out = m->generate(max_frames, p, seed, nullptr, forced ? &f : nullptr);
    for (size_t i = 0; i < out.size(); ++i)
        for (int ch = 0; ch < kNVq; ++ch) codes[i * kNVq + ch] = out[i][ch + 1];
    if (logits && logits_tmp_path)
        std::memcpy(logits, m->logits_dump_.data(), sizeof(float) * m->logits_dump_.size());
    m->logits_dump_path_.clear();
    return static_cast<int>(out.size());
}

// n_frames whole frames, each = the body of generate()'s loop (llm.cpp:647-708) with the
// global step always taken: local decoder from hidden_, the end gate (not acted on), 16
// greedy codes with the repetition penalty, then global_step([9, codes]).  Used to time the
// reference per frame.  codes [n_frames][16].
void ref_frames(void *h, int n_frames, float rep, int32_t *codes) {
    auto *m = static_cast<LlmModel *>(h);
    SampleParams p;
    p.greedy = true;
    p.repetition_penalty = rep;
    Rng rng;
    rng.seed(0);
    std::array<std::vector<int>, kNVq> history;
    for (int f = 0; f < n_frames && m->pos_ < kMaxCtx; ++f) {
        m->local_reset();
        m->local_step(m->hidden_.data(), m->lx_.data());
        float pair[2];
        m->assistant_logits(m->lx_.data(), pair);
        Row frame{};
        std::array<float, kHidden> input{};
        m->lookup_row(m->wte_, kSlotToken, input.data());
        for (int ch = 0; ch < kNVq; ++ch) {
            m->local_step(input.data(), m->lx_.data());
            m->audio_logits(ch, m->lx_.data(), m->logits_.data());
            const int pred = sample_token(m->logits_.data(), kCodebook, p, history[ch].data(),
                                          static_cast<int>(history[ch].size()), rng, m->sample_scratch_);
            frame[ch + 1] = pred;
            history[ch].push_back(pred);
            m->lookup_row(m->aemb_[ch], pred, input.data());
            codes[static_cast<size_t>(f) * kNVq + ch] = pred;
        }
        Row next{};
        next[0] = kSlotToken;
        for (int ch = 0; ch < kNVq; ++ch) next[ch + 1] = frame[ch + 1];
        m->global_step(next, m->hidden_.data());
    }
}

// ---- kernel-level entry points (fp16.cpp, quant.cpp, gemv_avx2.cpp, sampler.cpp) ----
void ref_half_to_float_n(const uint16_t *h, int n, float *out) {
    for (int i = 0; i < n; ++i) out[i] = half_to_float(h[i]);
}

void ref_float_to_half_n(const float *f, int n, uint16_t *out) {
    for (int i = 0; i < n; ++i) out[i] = float_to_half(f[i]);
}

void ref_dequant_row_q8x4(const uint8_t *group, int nb, int k, float *out) { dequantize_row_q8_0_4x4(group, nb, k, out); }

float ref_row_dot_a16(const uint8_t *group, int nb, int k, const float *act) {
    return row_dot_q8_4x4_actf32(group, nb, k, act);
}

float ref_row_dot_a8(const uint8_t *group, int nb, int k, const float *x, int cols) {
    QuantizedActivation act;
    quantize_activation(x, act, cols);
    return row_dot_q8_4x4(group, nb, k, act);
}

void ref_quantize_act(const float *x, int n, int8_t *q, float *scales) {
    QuantizedActivation act;
    quantize_activation(x, act, n);
    for (int b = 0; b < n / 32; ++b) {
        std::memcpy(q + b * 32, act.blocks[b].qs, 32);
        scales[b] = act.scales[b];
    }
}

int ref_sample_token(const float *logits, int n, int greedy, float temperature, int top_k, float top_p, float rep,
                     const int *prev, int n_prev, uint64_t seed) {
    SampleParams p;
    p.greedy = greedy != 0;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repetition_penalty = rep;
    Rng rng;
    rng.seed(seed);
    std::vector<float> scratch;
    return sample_token(logits, n, p, prev, n_prev, rng, scratch);
}

// ---- the reference's audio codec decoder (decoder.cpp), through its public API

void *ref_codec_create(const char *path, int threads) {
    auto *d = new AudioDecoder(threads);
    std::string err;
    if (!d->load(path, &err)) {
        std::fprintf(stderr, "ref_codec_create: %s\n", err.c_str());
        delete d;
        return nullptr;
    }
    d->reset_stream();
    return d;
}

void ref_codec_destroy(void *h) { delete static_cast<AudioDecoder *>(h); }

void ref_codec_reset(void *h) { static_cast<AudioDecoder *>(h)->reset_stream(); }

// AudioDecoder::decode_chunk: codes [16][frames] (nq-major); returns the sample count written
// to out (at most cap), or -1 when out is too small.
int ref_codec_decode_chunk(void *h, const int32_t *codes, int frames, float *out, int cap) {
    const std::vector<float> y = static_cast<AudioDecoder *>(h)->decode_chunk(codes, frames);
    if (static_cast<int>(y.size()) > cap) return -1;
    std::memcpy(out, y.data(), y.size() * sizeof(float));
    return static_cast<int>(y.size());
}

// AudioDecoder::decode: a whole utterance, non-streaming
int ref_codec_decode(void *h, const int32_t *codes, int frames, float *out, int cap) {
    const std::vector<float> y = static_cast<AudioDecoder *>(h)->decode(codes, frames);
    if (static_cast<int>(y.size()) > cap) return -1;
    std::memcpy(out, y.data(), y.size() * sizeof(float));
    return static_cast<int>(y.size());
}

}  // extern "C"
