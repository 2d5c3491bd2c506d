// llm_gpu.h -- moss::gpu::LlmModel: the reference's single-stream moss::LlmModel interface
// (reference csrc/include/moss/llm.h:39-158) implemented over the C ABI in mossgpu.h.
//
// Drop-in for TtsEngine (reference engine.h:94 holds std::unique_ptr<LlmModel>): same method
// names, argument meaning and error behaviour -- load() returns false with *err set; the
// void methods throw std::runtime_error on failure like the reference's fail() (common.h:11);
// generate() stops on the end gate, at the context cap or on the cancel flag, honours
// teacher forcing, the logits dump and the gate dump.  The prefix cache files (.mosskv,
// llm.cpp:441-550) and debug state files (llm.cpp:552-632) are byte-compatible with the
// reference's, so caches written by either engine load in the other.
//
// Header-only; link with libmossgpu.so.  Several LlmModel objects may share one engine
// (one per GPU) by passing it to the constructor; each object owns one engine stream.
#pragma once

#include <array>
#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/mossgpu.h"

namespace moss {
namespace gpu {

constexpr int kHidden = 768;
constexpr int kNVq = 16;
constexpr int kCodebook = 1024;
constexpr int kSlotToken = 9;
constexpr int kLayers = 12;

using Row = std::array<int32_t, kNVq + 1>;  // [text_id, code0..code15] (llm.h:32)

struct FrameTiming {  // llm.h:34-37
    double global_ms = 0.0;
    double local_ms = 0.0;
};

struct SampleParams {  // sampler.h:8-22, same defaults
    bool greedy = true;
    float temperature = 1.0f;
    int top_k = 0;
    float top_p = 1.0f;
    float repetition_penalty = 1.0f;
    bool end_greedy = true;
    int min_frames = 0;
    int greedy_frames = 0;
};

// Where generate() reports per-frame timings: nothing (nullptr), or a std::vector of any
// struct with the members {global_ms, local_ms} -- this header's FrameTiming or the
// reference's moss::FrameTiming (llm.h:34-37), so that callers written against the reference
// pass their own vectors unchanged.
class TimingOut {
public:
    TimingOut(std::nullptr_t = nullptr) {}
    template <class T>
    TimingOut(std::vector<T> *v) {
        if (v) push_ = [v](double global_ms, double local_ms) { v->push_back(T{global_ms, local_ms}); };
    }
    void operator()(double global_ms, double local_ms) const {
        if (push_) push_(global_ms, local_ms);
    }

private:
    std::function<void(double, double)> push_;
};

class Engine {  // one mossgpu_engine per GPU, shareable by several LlmModel objects
public:
    Engine(const std::string &weights, int device, int max_streams, int max_ctx) {
        char err[1024] = {0};
        h_ = mossgpu_create(weights.c_str(), device, max_streams, max_ctx, 0, err, sizeof(err));
        if (!h_) throw std::runtime_error(err);
        max_ctx_ = max_ctx;
    }
    ~Engine() { mossgpu_destroy(h_); }
    Engine(const Engine &) = delete;
    Engine &operator=(const Engine &) = delete;
    mossgpu_engine *handle() const { return h_; }
    int max_ctx() const { return max_ctx_; }
    void check(int rc) const {
        if (rc != 0) throw std::runtime_error(mossgpu_last_error(h_));
    }

private:
    mossgpu_engine *h_ = nullptr;
    int max_ctx_ = 0;
};

class LlmModel {
public:
    // threads: accepted for signature compatibility (llm.h:42); the GPU engine ignores it.
    explicit LlmModel(int threads = 1, int device = 0, int max_ctx = 4608, std::shared_ptr<Engine> engine = nullptr)
        : device_(device), max_ctx_(max_ctx), engine_(std::move(engine)) {
        (void)threads;
    }
    ~LlmModel() {
        if (engine_ && sid_ >= 0) mossgpu_stream_close(engine_->handle(), sid_);
        if (engine_ && prefix_sid_ >= 0) mossgpu_stream_close(engine_->handle(), prefix_sid_);
    }

    // llm.h:46
    bool load(const std::string &weights_path, std::string *err) {
        try {
            // two stream slots: the model's state and its device-side prefix snapshot
            if (!engine_) engine_ = std::make_shared<Engine>(weights_path, device_, 2, max_ctx_);
            max_ctx_ = engine_->max_ctx();
            engine_->check(mossgpu_stream_open(engine_->handle(), &sid_));
            weights_fp_ = fp_weights(weights_path);
            info_ = "weights=" + weights_path + " device=" + std::to_string(device_);
            return true;
        } catch (const std::exception &e) {
            if (err) *err = e.what();
            return false;
        }
    }

    void reset() { engine_->check(mossgpu_stream_reset(engine_->handle(), sid_)); }  // llm.h:49

    // llm.h:53, llm.cpp:327-401
    void prefill(const std::vector<Row> &rows, int start = 0) {
        engine_->check(mossgpu_prefill(engine_->handle(), sid_, rows.empty() ? nullptr : rows[0].data(),
                                       static_cast<int>(rows.size()), start));
    }

    // llm.h:57-60, llm.cpp:455-483: the prefix is kept on the device as a second stream that
    // shares the KV pages (mossgpu_stream_fork); restoring forks it back, copying only the
    // partly filled last page
    void snapshot_prefix() {
        prefix_pos_ = position();
        keep_prefix_on_device();
    }
    void restore_prefix() {
        if (prefix_pos_ <= 0) {
            reset();
            return;
        }
        if (prefix_sid_ < 0) keep_prefix_on_device();
        // the prefix stream keeps the shared pages alive: close first, then fork into the slot
        engine_->check(mossgpu_stream_close(engine_->handle(), sid_));
        sid_ = -1;
        engine_->check(mossgpu_stream_fork(engine_->handle(), prefix_sid_, prefix_pos_, &sid_));
    }
    int prefix_pos() const { return prefix_pos_; }

    // llm.h:63-64, llm.cpp:485-550 (magic "MOSSPFX1")
    bool save_prefix(const std::string &path, const std::vector<Row> &rows, std::string *err) {
        return save_file(path, rows, kKvMagic, false, err);
    }
    bool load_prefix(const std::string &path, const std::vector<Row> &rows, std::string *err) {
        return load_file(path, rows, kKvMagic, false, false, err);
    }
    // llm.h:68-70, llm.cpp:560-632 (magic "MOSSST1", KV + last hidden)
    bool save_state(const std::string &path, const std::vector<Row> &rows, std::string *err) {
        return save_file(path, rows, kStateMagic, true, err);
    }
    bool load_state(const std::string &path, const std::vector<Row> &rows, bool ignore_weights_fp, std::string *err) {
        return load_file(path, rows, kStateMagic, true, ignore_weights_fp, err);
    }

    // llm.h:75-79, llm.cpp:634-733.  Params: this header's SampleParams or the reference's
    // moss::SampleParams (sampler.h:8-22) -- any struct with its eight members.
    template <class Params>
    std::vector<Row> generate(int max_frames, const Params &audio_params, uint64_t seed, TimingOut timing = nullptr,
                              const std::vector<Row> *forced = nullptr,
                              const std::function<void(int, const Row &)> &on_frame = {}) {
        using Clock = std::chrono::steady_clock;
        std::vector<Row> frames;
        std::vector<float> logits_dump, logits(static_cast<size_t>(kNVq) * kCodebook);
        std::string gate_csv;
        engine_->check(mossgpu_generate_begin(engine_->handle(), sid_, seed));
        mossgpu_sample_params p{audio_params.greedy ? 1 : 0, audio_params.temperature, audio_params.top_k,
                                audio_params.top_p, audio_params.repetition_penalty, audio_params.end_greedy ? 1 : 0,
                                audio_params.min_frames, audio_params.greedy_frames};
        for (int f = 0; f < max_frames; ++f) {
            if (position() >= max_ctx_) break;
            if (cancel_ && cancel_->load(std::memory_order_relaxed)) break;
            const auto t0 = Clock::now();
            int32_t codes[kNVq], fcodes[kNVq];
            uint8_t stop = 0;
            float gate[2] = {0.f, 0.f};
            const int32_t *fc = nullptr;
            if (forced) {
                for (int ch = 0; ch < kNVq; ++ch) fcodes[ch] = (*forced)[static_cast<size_t>(f)][ch + 1];
                fc = fcodes;
            }
            const bool last = !(f + 1 < max_frames);
            engine_->check(mossgpu_step(engine_->handle(), &sid_, 1, &p, fc, codes, &stop,
                                        logits_dump_path_.empty() ? nullptr : logits.data(), gate, last ? 0 : 1));
            const double ms = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
            if (!gate_dump_path_.empty())
                gate_csv += std::to_string(f) + "," + std::to_string(gate[1] - gate[0]) + "\n";
            if (stop) break;
            if (!logits_dump_path_.empty()) logits_dump.insert(logits_dump.end(), logits.begin(), logits.end());
            Row row{};
            for (int ch = 0; ch < kNVq; ++ch) row[ch + 1] = codes[ch];
            frames.push_back(row);
            timing(last ? 0.0 : ms, 0.0);
            if (on_frame) on_frame(f, row);
        }
        if (!logits_dump_path_.empty()) {
            if (std::FILE *fp = std::fopen(logits_dump_path_.c_str(), "wb")) {
                std::fwrite(logits_dump.data(), sizeof(float), logits_dump.size(), fp);
                std::fclose(fp);
            }
        }
        if (!gate_dump_path_.empty()) {
            if (std::FILE *fp = std::fopen(gate_dump_path_.c_str(), "wb")) {
                std::fprintf(fp, "frame,slot_minus_end\n%s", gate_csv.c_str());
                std::fclose(fp);
            }
        }
        return frames;
    }

    void set_logits_dump(const std::string &path) { logits_dump_path_ = path; }
    // CSV "frame,slot_minus_end": the gate margin of every frame.  The reference's dump adds the
    // argmax over the full 16384-row text head (llm.cpp:664-676,721-730), which this engine
    // does not compute (the gate evaluates rows 7 and 9 only, as assistant_logits does).
    void set_gate_dump(const std::string &path) { gate_dump_path_ = path; }
    void set_cancel_flag(const std::atomic<bool> *flag) { cancel_ = flag; }

    const float *hidden() const {
        hidden_.resize(kHidden);
        engine_->check(mossgpu_get_hidden(engine_->handle(), sid_, hidden_.data()));
        return hidden_.data();
    }
    int position() const {
        int p = 0;
        engine_->check(mossgpu_stream_position(engine_->handle(), sid_, &p));
        return p;
    }
    const std::string &info() const { return info_; }

private:
    static constexpr char kKvMagic[8] = {'M', 'O', 'S', 'S', 'P', 'F', 'X', '1'};
    static constexpr char kStateMagic[8] = {'M', 'O', 'S', 'S', 'S', 'T', '1', '\0'};

    struct KvHeader {  // llm.cpp:443-451
        char magic[8];
        uint32_t version = 1;
        uint32_t layers = 0;
        uint32_t n_pos = 0;
        uint32_t hidden = 0;
        uint64_t rows_fp = 0;
        uint64_t weights_fp = 0;
    };

    static uint64_t fnv(uint64_t h, const void *data, size_t n) {  // llm.cpp:410-417
        const uint8_t *p = static_cast<const uint8_t *>(data);
        for (size_t i = 0; i < n; ++i) {
            h ^= p[i];
            h *= 1099511628211ull;
        }
        return h;
    }
    static uint64_t fp_rows(const std::vector<Row> &rows) {  // llm.cpp:419-423
        uint64_t h = 1469598103934665603ull;
        for (const Row &r : rows) h = fnv(h, r.data(), sizeof(int32_t) * r.size());
        return h;
    }
    static uint64_t fp_weights(const std::string &path) {  // llm.cpp:426-439
        uint64_t h = 1469598103934665603ull;
        std::FILE *f = std::fopen(path.c_str(), "rb");
        if (!f) return 0;
        std::fseek(f, 0, SEEK_END);
        const long size = std::ftell(f);
        std::fseek(f, 0, SEEK_SET);
        uint8_t head[4096];
        const size_t got = std::fread(head, 1, sizeof(head), f);
        std::fclose(f);
        const int64_t sz = size;
        h = fnv(h, &sz, sizeof(sz));
        return fnv(h, head, got);
    }

    // K and V of positions [0, n) of every layer, fp32 [12][n][768] (fp16 cache widened)
    void keep_prefix_on_device() {
        if (prefix_sid_ >= 0) engine_->check(mossgpu_stream_close(engine_->handle(), prefix_sid_));
        prefix_sid_ = -1;
        if (prefix_pos_ > 0) engine_->check(mossgpu_stream_fork(engine_->handle(), sid_, prefix_pos_, &prefix_sid_));
    }

    void read_kv(int n, std::vector<float> *k, std::vector<float> *v) const {
        const size_t per = static_cast<size_t>(n) * kHidden;
        k->assign(kLayers * per, 0.f);
        v->assign(kLayers * per, 0.f);
        if (n <= 0) return;
        for (int l = 0; l < kLayers; ++l)
            engine_->check(mossgpu_get_kv(engine_->handle(), sid_, l, 0, n, k->data() + l * per, v->data() + l * per));
    }

    bool save_file(const std::string &path, const std::vector<Row> &rows, const char *magic, bool with_hidden,
                   std::string *err) {
        const int n = position();
        if (n <= 0) {
            if (err) *err = "empty state, nothing to save";
            return false;
        }
        std::vector<float> k, v;
        read_kv(n, &k, &v);
        std::FILE *f = std::fopen(path.c_str(), "wb");
        if (!f) {
            if (err) *err = "cannot write " + path;
            return false;
        }
        KvHeader h{};
        std::memcpy(h.magic, magic, 8);
        h.layers = kLayers;
        h.n_pos = static_cast<uint32_t>(n);
        h.hidden = kHidden;
        h.rows_fp = fp_rows(rows);
        h.weights_fp = weights_fp_;
        std::fwrite(&h, sizeof(h), 1, f);
        const size_t per = static_cast<size_t>(n) * kHidden;
        for (int l = 0; l < kLayers; ++l) {
            std::fwrite(k.data() + l * per, sizeof(float), per, f);
            std::fwrite(v.data() + l * per, sizeof(float), per, f);
        }
        if (with_hidden) std::fwrite(hidden(), sizeof(float), kHidden, f);
        std::fclose(f);
        return true;
    }

    bool load_file(const std::string &path, const std::vector<Row> &rows, const char *magic, bool with_hidden,
                   bool ignore_weights_fp, std::string *err) {
        std::FILE *f = std::fopen(path.c_str(), "rb");
        if (!f) {
            if (err) *err = "cannot open " + path;
            return false;
        }
        KvHeader h{};
        if (std::fread(&h, sizeof(h), 1, f) != 1 || std::memcmp(h.magic, magic, 8) != 0 || h.version != 1 ||
            h.layers != kLayers || h.hidden != kHidden || h.n_pos == 0 || h.n_pos > static_cast<uint32_t>(max_ctx_)) {
            std::fclose(f);
            if (err) *err = "bad file format: " + path;
            return false;
        }
        if (h.rows_fp != fp_rows(rows)) {
            std::fclose(f);
            if (err) *err = "file does not match the prompt (rows fingerprint)";
            return false;
        }
        if (!ignore_weights_fp && h.weights_fp != weights_fp_) {
            std::fclose(f);
            if (err) *err = "file does not match the loaded weights (weights fingerprint)";
            return false;
        }
        const size_t per = static_cast<size_t>(h.n_pos) * kHidden;
        std::vector<float> k(kLayers * per), v(kLayers * per), hid(kHidden);
        for (int l = 0; l < kLayers; ++l) {
            if (std::fread(k.data() + l * per, sizeof(float), per, f) != per ||
                std::fread(v.data() + l * per, sizeof(float), per, f) != per) {
                std::fclose(f);
                if (err) *err = "truncated file: " + path;
                return false;
            }
        }
        if (with_hidden && std::fread(hid.data(), sizeof(float), kHidden, f) != static_cast<size_t>(kHidden)) {
            std::fclose(f);
            if (err) *err = "file lacks the hidden state: " + path;
            return false;
        }
        std::fclose(f);
        try {
            engine_->check(mossgpu_set_state(engine_->handle(), sid_, k.data(), v.data(), static_cast<int>(h.n_pos),
                                             with_hidden ? hid.data() : nullptr));
        } catch (const std::exception &e) {
            if (err) *err = e.what();
            return false;
        }
        prefix_pos_ = static_cast<int>(h.n_pos);
        try {
            keep_prefix_on_device();
        } catch (const std::exception &e) {
            if (err) *err = e.what();
            return false;
        }
        return true;
    }

    int device_ = 0;
    int max_ctx_ = 4608;
    std::shared_ptr<Engine> engine_;
    int sid_ = -1;
    uint64_t weights_fp_ = 0;
    int prefix_pos_ = 0;
    int prefix_sid_ = -1;  // device stream holding the prefix snapshot (shared KV pages)
    mutable std::vector<float> hidden_;
    const std::atomic<bool> *cancel_ = nullptr;
    std::string info_, logits_dump_path_, gate_dump_path_;
};

}  // namespace gpu
}  // namespace moss
