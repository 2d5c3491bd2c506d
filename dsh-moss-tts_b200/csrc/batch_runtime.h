// batch_runtime.h -- moss::gpu::BatchRuntime: the reference Runtime's job API (submit / wait /
// job / cancel / queue_depth, reference csrc/include/moss/runtime.h:92-113, queue semantics
// runtime.cpp:282-336, 434-508) with its one worker thread advancing every admitted job in
// the same engine calls, where the reference's worker runs one TtsEngine::synthesize at a
// time (runtime.cpp:318-336).
//
// A job is the token-level part of TtsEngine::synthesize (engine.cpp:415-545).  For each
// text segment:
//   - the voice prefix is restored: a fork of a prefix stream (mossgpu_stream_fork), or a
//     fresh stream when the job has no prefix;
//   - the segment's suffix rows are prefilled at the prefix length;
//   - generate() runs up to max_frames, its generator seeded with the job seed;
//   - the frames go to the sink as nq-major code blocks [16][n]: the job's first block after
//     min(4, chunk_frames) frames, later blocks after chunk_frames, and each segment's
//     remainder when the segment ends (engine.cpp:480-502).
// Text splitting, tokenisation, the codec and PCM sit above this layer.  The sink receives
// the codes that the reference hands to decode_chunk.
//
// One worker iteration (run_once):
//   1. queued jobs are admitted while fewer than max_active run.  A job cancelled while
//      queued ends Cancelled without an engine call;
//   2. every running job without a live segment opens its next one.  All segments opened in
//      the iteration are prefilled by ONE mossgpu_prefill_batch call (if that call fails, each
//      segment is retried alone so that one bad job fails by itself), then
//      mossgpu_generate_begin seeds each;
//   3. live segments are grouped by sampling parameters.  Each group advances by one
//      mossgpu_step_frames call of F frames, F = min(frames_per_call, the frames any member
//      has left before max_frames or the context cap);
//   4. frames go to each job's chunk assembler and sink.  A segment ends on the end gate
//      (fewer frames done than F), at max_frames, at the context cap, or on cancel.
// Cancel is looked at once per step call, where the reference looks once per frame.  Frames of
// a call that returns after cancel() are dropped, as the reference drops the frames it pops
// after the flag is set (engine.cpp:506-513), and a cancelled segment is not flushed.  A sink
// returning false cancels its job (runtime.cpp:393-401).
//
// Ops is the engine: MossGpuOps below (the C ABI of mossgpu.h) or a test double with the same
// members.  Use either start() (a worker thread) or run_once() from one thread, not both.
// Once the worker runs, the engine is the worker's: open and prefill prefix streams before
// start(), since calls on one engine must not overlap.
#pragma once

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <utility>
#include <vector>

#include "../../include/mossgpu.h"
#include "frame_router.h"

namespace moss {
namespace gpu {

// Token-level JobRequest (runtime.h:45-62): the rows each text segment prefills instead of the
// text, and the prefix stream instead of the voice.  Zero sampling fields take the engine
// defaults (engine.h:39-42; runtime.cpp:352-356).
struct GenJobRequest {
    std::string id;                                 // empty: the runtime makes one
    int prefix_stream = -1;                         // open engine stream holding the voice prefix
    int prefix_len = 0;                             // its positions to share (fork length)
    std::vector<std::vector<FrameRow>> segments;    // suffix rows [m][17] per text segment
    uint64_t seed = 0;
    bool greedy = false;
    int max_frames = 375;                           // <= 0: 375 (runtime.cpp:348)
    int chunk_frames = 8;                           // <= 0: 8
    int min_frames = 0;
    int greedy_frames = 0;
    float temperature = 0.0f;                       // 0: 0.8
    int top_k = 0;                                  // 0: 25
    float top_p = 0.0f;                             // 0: 0.95
    float repetition_penalty = 0.0f;                // 0: 1.2
};

enum class GenJobState { Queued, Running, Completed, Cancelled, Failed };

inline const char *gen_job_state_name(GenJobState s) {  // runtime.cpp:72-81
    switch (s) {
        case GenJobState::Queued: return "queued";
        case GenJobState::Running: return "running";
        case GenJobState::Completed: return "completed";
        case GenJobState::Cancelled: return "cancelled";
        case GenJobState::Failed: return "failed";
    }
    return "unknown";
}

struct GenJobInfo {  // runtime.h:64-77, token-level
    std::string id;
    GenJobState state = GenJobState::Queued;
    int frames = 0;            // frames handed to the sink
    int segments_done = 0;
    double wall_ms = 0.0;      // submit to end
    double first_codes_ms = -1.0;
    std::string error;
};

// One nq-major block codes[16][n] of segment `segment`; returning false means the receiver
// failed, and the job is cancelled (PcmSink, runtime.h:83).
using CodeSink = std::function<bool(int segment, const int32_t *codes, int n)>;

struct BatchRuntimeOptions {
    int max_active = 64;       // jobs advanced together; each holds one engine stream
    int max_queue = 4;         // queued (not yet admitted) jobs before submit answers "busy"
    int frames_per_call = 8;   // frames per mossgpu_step_frames call (1..1024)
    // Admission hold: while other jobs run, queued jobs wait until admit_min of them are
    // queued or the oldest has waited admit_wait_ms, so that more new segments share one
    // prefill pass (at the cost of their first codes' latency).  An idle runtime admits at
    // once.  admit_min <= 1: no hold.
    int admit_min = 1;
    int admit_wait_ms = 0;
};

// The engine through the C ABI.
class MossGpuOps {
public:
    MossGpuOps(mossgpu_engine *h, int max_ctx) : h_(h), max_ctx_(max_ctx) {}
    int open(int *sid) { return mossgpu_stream_open(h_, sid); }
    int fork(int src, int n_pos, int *sid) { return mossgpu_stream_fork(h_, src, n_pos, sid); }
    int close(int sid) { return mossgpu_stream_close(h_, sid); }
    int position(int sid, int *pos) { return mossgpu_stream_position(h_, sid, pos); }
    int prefill_batch(int n, const int32_t *sids, const int32_t *m, const int32_t *start, const int32_t *rows) {
        return mossgpu_prefill_batch(h_, n, sids, m, start, rows);
    }
    int generate_begin(int sid, uint64_t seed) { return mossgpu_generate_begin(h_, sid, seed); }
    int step_frames(const int32_t *sids, int n, const mossgpu_sample_params &p, int frames, int32_t *codes,
                    int32_t *done) {
        return mossgpu_step_frames(h_, sids, n, &p, frames, codes, done);
    }
    const char *last_error() { return mossgpu_last_error(h_); }
    int max_ctx() const { return max_ctx_; }

private:
    mossgpu_engine *h_;
    int max_ctx_;
};

template <class Ops>
class BatchRuntime {
    using Clock = std::chrono::steady_clock;

public:
    static constexpr int kKeepJobs = 32;         // runtime.cpp:23
    static constexpr int kJobTtlSeconds = 600;   // runtime.cpp:24

    BatchRuntime(Ops &ops, BatchRuntimeOptions opt) : ops_(ops), opt_(opt) {
        opt_.max_active = std::max(1, opt_.max_active);
        opt_.frames_per_call = std::min(1024, std::max(1, opt_.frames_per_call));
    }
    ~BatchRuntime() { shutdown(); }
    BatchRuntime(const BatchRuntime &) = delete;
    BatchRuntime &operator=(const BatchRuntime &) = delete;

    void start() {
        std::lock_guard<std::mutex> lock(mutex_);
        if (!worker_.joinable() && !stop_) worker_ = std::thread([this] { worker_loop(); });
    }

    // Queued jobs end Cancelled ("shutting down"); running jobs run to their end first
    // (runtime.cpp:172-186).  Without a worker (run_once mode) nothing runs them: call
    // run_once until it returns false before shutting down, or their streams stay open.
    void shutdown() {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            if (!stop_) {
                stop_ = true;
                for (auto &j : queue_) {
                    j->cancel.store(true);
                    end_locked(*j, GenJobState::Cancelled, "shutting down");
                }
                queue_.clear();
            }
        }
        job_added_.notify_all();
        job_done_.notify_all();
        if (worker_.joinable()) worker_.join();
    }

    bool submit(const GenJobRequest &req, CodeSink sink, std::string *job_id, std::string *err) {
        if (req.segments.empty()) return fail_submit(err, "no segments");
        if (req.prefix_stream >= 0 && req.prefix_len <= 0) return fail_submit(err, "prefix_len must be positive");
        auto j = std::make_shared<Job>();
        j->req = req;
        j->sink = std::move(sink);
        j->submitted = Clock::now();
        if (j->req.max_frames <= 0) j->req.max_frames = 375;
        if (j->req.chunk_frames <= 0) j->req.chunk_frames = 8;
        j->assembler = ChunkAssembler(j->req.chunk_frames);
        j->params = make_params(j->req);
        j->cost = job_cost(j->req);
        {
            std::lock_guard<std::mutex> lock(mutex_);
            if (stop_) return fail_submit(err, "shutting down");
            if (static_cast<int>(queue_.size()) >= opt_.max_queue) return fail_submit(err, "busy");
            j->info.id = j->req.id.empty() ? make_job_id_locked() : j->req.id;
            queue_.push_back(j);
            jobs_.push_back(j);
            load_ += j->cost;
            prune_locked();
        }
        job_added_.notify_one();
        if (job_id) *job_id = j->info.id;
        return true;
    }

    // Blocks until the job ends or timeout_ms passes; true iff it ended.
    bool wait(const std::string &id, int timeout_ms, GenJobInfo *out) {
        std::unique_lock<std::mutex> lock(mutex_);
        auto j = find_locked(id);
        if (!j) return false;
        const auto deadline = Clock::now() + std::chrono::milliseconds(std::max(0, timeout_ms));
        job_done_.wait_until(lock, deadline, [&] { return terminal(j->info.state); });
        if (out) *out = j->info;
        return terminal(j->info.state);
    }

    bool job(const std::string &id, GenJobInfo *out) const {
        std::lock_guard<std::mutex> lock(mutex_);
        auto j = find_locked(id);
        if (!j) return false;
        if (out) *out = j->info;
        return true;
    }

    bool cancel(const std::string &id) {
        std::lock_guard<std::mutex> lock(mutex_);
        auto j = find_locked(id);
        if (!j) return false;
        j->cancel.store(true);
        return true;
    }

    int queue_depth() const {
        std::lock_guard<std::mutex> lock(mutex_);
        return static_cast<int>(queue_.size());
    }
    int max_queue() const { return opt_.max_queue; }
    int running() const { return running_count_.load(); }
    // Outstanding work: the summed job_cost of the jobs queued or running.
    int64_t load() const { return load_.load(); }

    // A job's work for load balancing: every non-empty segment attends over the prefix and its
    // own rows and generates up to max_frames frames (max_frames <= 0 counts as 375).
    static int64_t job_cost(const GenJobRequest &r) {
        const int64_t frames = r.max_frames > 0 ? r.max_frames : 375;
        int64_t c = 0;
        for (const auto &seg : r.segments)
            if (!seg.empty()) c += (r.prefix_stream >= 0 ? r.prefix_len : 0) + static_cast<int64_t>(seg.size()) + frames;
        return c;
    }

    // One scheduling iteration; false when there was nothing to do (no queued or running job).
    bool run_once() {
        bool did = admit();
        if (running_.empty()) return did;
        open_segments();
        step_groups();
        running_.erase(std::remove_if(running_.begin(), running_.end(),
                                      [](const std::shared_ptr<Job> &j) { return j->ended; }),
                       running_.end());
        running_count_.store(static_cast<int>(running_.size()));
        return true;
    }

private:
    struct Job {
        GenJobRequest req;
        CodeSink sink;
        std::atomic<bool> cancel{false};
        GenJobInfo info;
        Clock::time_point submitted, finished;
        mossgpu_sample_params params{};
        int64_t cost = 0;
        // worker-side state
        ChunkAssembler assembler{8};
        size_t seg = 0;        // next segment to open (or the live one)
        int sid = -1;
        int pos = 0;
        int seg_frames = 0;
        bool live = false;
        bool ended = false;
    };

    static bool terminal(GenJobState s) {
        return s == GenJobState::Completed || s == GenJobState::Cancelled || s == GenJobState::Failed;
    }
    static bool fail_submit(std::string *err, const char *why) {
        if (err) *err = why;
        return false;
    }
    static double ms_since(Clock::time_point t0) {
        return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    }
    static mossgpu_sample_params make_params(const GenJobRequest &r) {  // engine.cpp:415-423
        mossgpu_sample_params p{};
        p.greedy = r.greedy ? 1 : 0;
        p.temperature = r.temperature > 0.0f ? r.temperature : 0.8f;
        p.top_k = r.top_k > 0 ? r.top_k : 25;
        p.top_p = r.top_p > 0.0f ? r.top_p : 0.95f;
        p.repetition_penalty = r.repetition_penalty > 0.0f ? r.repetition_penalty : 1.2f;
        p.end_greedy = 1;
        p.min_frames = std::max(0, r.min_frames);
        p.greedy_frames = std::max(0, r.greedy_frames);
        return p;
    }
    static auto params_key(const mossgpu_sample_params &p) {
        return std::make_tuple(p.greedy, p.temperature, p.top_k, p.top_p, p.repetition_penalty, p.end_greedy,
                               p.min_frames, p.greedy_frames);
    }

    std::string make_job_id_locked() {  // runtime.cpp:273-280
        ++counter_;
        char buf[32];
        std::snprintf(buf, sizeof(buf), "%08llx%04llx", static_cast<unsigned long long>(counter_),
                      static_cast<unsigned long long>(Clock::now().time_since_epoch().count() & 0xFFFF));
        return buf;
    }
    std::shared_ptr<Job> find_locked(const std::string &id) const {
        for (auto &j : jobs_)
            if (j->info.id == id) return j;
        return nullptr;
    }
    void prune_locked() {  // runtime.cpp:446-467
        const auto now = Clock::now();
        jobs_.erase(std::remove_if(jobs_.begin(), jobs_.end(),
                                   [&](const std::shared_ptr<Job> &j) {
                                       return terminal(j->info.state) &&
                                              std::chrono::duration<double>(now - j->finished).count() >
                                                  kJobTtlSeconds;
                                   }),
                    jobs_.end());
        while (static_cast<int>(jobs_.size()) > kKeepJobs && terminal(jobs_.front()->info.state))
            jobs_.erase(jobs_.begin());
    }
    void end_locked(Job &j, GenJobState s, const std::string &error) {
        if (!j.ended) load_ -= j.cost;
        j.info.state = s;
        j.info.error = error;
        j.finished = Clock::now();
        j.info.wall_ms = ms_since(j.submitted);
        j.ended = true;
    }
    void end_job(Job &j, GenJobState s, const std::string &error) {
        if (j.live) {
            ops_.close(j.sid);
            j.live = false;
            j.sid = -1;
        }
        {
            std::lock_guard<std::mutex> lock(mutex_);
            end_locked(j, s, error);
        }
        job_done_.notify_all();
    }

    void worker_loop() {
        while (true) {
            if (run_once()) continue;
            std::unique_lock<std::mutex> lock(mutex_);
            job_added_.wait(lock, [this] { return stop_ || !queue_.empty(); });
            if (stop_ && queue_.empty()) return;
        }
    }

    bool admit() {
        bool did = false;
        std::vector<std::shared_ptr<Job>> admitted;
        {
            std::lock_guard<std::mutex> lock(mutex_);
            const bool hold = !running_.empty() && !queue_.empty() && static_cast<int>(queue_.size()) < opt_.admit_min &&
                              ms_since(queue_.front()->submitted) < static_cast<double>(opt_.admit_wait_ms);
            while (!hold && !queue_.empty() && static_cast<int>(running_.size() + admitted.size()) < opt_.max_active) {
                auto j = queue_.front();
                queue_.pop_front();
                did = true;
                if (j->cancel.load()) {
                    end_locked(*j, GenJobState::Cancelled, "cancelled");
                    continue;
                }
                j->info.state = GenJobState::Running;
                admitted.push_back(j);
            }
        }
        if (did) job_done_.notify_all();
        for (auto &j : admitted) running_.push_back(j);
        running_count_.store(static_cast<int>(running_.size()));
        return did;
    }

    // Step 2: next segments of jobs without a live one, prefilled in one batched call.
    void open_segments() {
        std::vector<Job *> opening;
        for (auto &jp : running_) {
            Job &j = *jp;
            if (j.live || j.ended) continue;
            while (j.seg < j.req.segments.size() && j.req.segments[j.seg].empty()) ++j.seg;  // engine.cpp:455
            if (j.cancel.load()) {
                end_job(j, GenJobState::Cancelled, "cancelled");
                continue;
            }
            if (j.seg >= j.req.segments.size()) {
                end_job(j, GenJobState::Completed, "");
                continue;
            }
            int sid = -1;
            const int rc = j.req.prefix_stream >= 0 ? ops_.fork(j.req.prefix_stream, j.req.prefix_len, &sid)
                                                    : ops_.open(&sid);
            if (rc != 0) {
                end_job(j, GenJobState::Failed, ops_.last_error());
                continue;
            }
            j.sid = sid;
            j.live = true;
            j.seg_frames = 0;
            opening.push_back(&j);
        }
        if (opening.empty()) return;
        std::vector<Job *> ok;
        if (prefill(opening) == 0) {
            ok = opening;
        } else if (opening.size() == 1) {
            end_job(*opening[0], GenJobState::Failed, ops_.last_error());
        } else {
            for (Job *j : opening) {  // isolate the failing segment(s)
                if (prefill({j}) == 0)
                    ok.push_back(j);
                else
                    end_job(*j, GenJobState::Failed, ops_.last_error());
            }
        }
        for (Job *j : ok) {
            if (ops_.generate_begin(j->sid, j->req.seed) != 0 || ops_.position(j->sid, &j->pos) != 0)
                end_job(*j, GenJobState::Failed, ops_.last_error());
        }
    }

    int prefill(const std::vector<Job *> &jobs) {
        std::vector<int32_t> sids, m, start, rows;
        for (Job *j : jobs) {
            const auto &seg = j->req.segments[j->seg];
            sids.push_back(j->sid);
            m.push_back(static_cast<int32_t>(seg.size()));
            start.push_back(j->req.prefix_stream >= 0 ? j->req.prefix_len : 0);
            for (const auto &r : seg) rows.insert(rows.end(), r.begin(), r.end());
        }
        return ops_.prefill_batch(static_cast<int>(jobs.size()), sids.data(), m.data(), start.data(), rows.data());
    }

    // Steps 3 and 4.
    void step_groups() {
        std::vector<std::vector<Job *>> groups;
        for (auto &jp : running_) {
            Job &j = *jp;
            if (!j.live || j.ended) continue;
            if (j.cancel.load()) {
                end_job(j, GenJobState::Cancelled, "cancelled");
                continue;
            }
            if (j.pos >= ops_.max_ctx()) {  // a prompt that filled the context: no frames (llm.cpp:644)
                end_segment(j);
                continue;
            }
            auto it = std::find_if(groups.begin(), groups.end(), [&](const std::vector<Job *> &g) {
                return params_key(g[0]->params) == params_key(j.params);
            });
            if (it == groups.end())
                groups.push_back({&j});
            else
                it->push_back(&j);
        }
        for (auto &g : groups) step_group(g);
    }

    void step_group(const std::vector<Job *> &g) {
        const int n = static_cast<int>(g.size());
        int frames = opt_.frames_per_call;
        for (Job *j : g) {
            frames = std::min(frames, j->req.max_frames - j->seg_frames);
            frames = std::min(frames, ops_.max_ctx() - j->pos);
        }
        frames = std::max(frames, 1);  // a segment at either limit has already ended
        std::vector<int32_t> sids(static_cast<size_t>(n)), done(static_cast<size_t>(n), 0);
        std::vector<int32_t> codes(static_cast<size_t>(frames) * n * kRouterNVq, -1);
        for (int i = 0; i < n; ++i) sids[static_cast<size_t>(i)] = g[static_cast<size_t>(i)]->sid;
        if (ops_.step_frames(sids.data(), n, g[0]->params, frames, codes.data(), done.data()) != 0) {
            const std::string err = ops_.last_error();
            for (Job *j : g) end_job(*j, GenJobState::Failed, err);
            return;
        }
        for (int i = 0; i < n; ++i) {
            Job &j = *g[static_cast<size_t>(i)];
            if (j.cancel.load()) {  // frames of this call are dropped, the segment is not flushed
                end_job(j, GenJobState::Cancelled, "cancelled");
                continue;
            }
            const int got = std::min(std::max(done[static_cast<size_t>(i)], 0), frames);
            bool sink_ok = true;
            std::vector<int32_t> block;
            int bn = 0;
            for (int f = 0; f < got && sink_ok; ++f) {
                FrameRow row{};
                const int32_t *c = codes.data() + (static_cast<size_t>(f) * n + i) * kRouterNVq;
                for (int ch = 0; ch < kRouterNVq; ++ch) row[static_cast<size_t>(ch) + 1] = c[ch];
                if (j.assembler.push(row, &block, &bn)) sink_ok = deliver(j, block, bn);
            }
            j.seg_frames += got;
            j.pos += got;
            if (!sink_ok) {
                j.cancel.store(true);
                end_job(j, GenJobState::Cancelled, "cancelled");
                continue;
            }
            if (got < frames || j.seg_frames >= j.req.max_frames || j.pos >= ops_.max_ctx()) end_segment(j);
        }
    }

    bool deliver(Job &j, const std::vector<int32_t> &block, int n) {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            j.info.frames += n;
            if (j.info.first_codes_ms < 0.0) j.info.first_codes_ms = ms_since(j.submitted);
        }
        if (!j.sink) return true;
        try {
            return j.sink(static_cast<int>(j.seg), block.data(), n);
        } catch (...) {
            return false;  // a throwing receiver fails like one returning false
        }
    }

    // The segment ended normally: its remainder goes out, its stream closes, and the job ends
    // when no segment is left (engine.cpp:515-530).
    void end_segment(Job &j) {
        std::vector<int32_t> block;
        int bn = 0;
        const bool sink_ok = !j.assembler.flush(&block, &bn) || deliver(j, block, bn);
        ops_.close(j.sid);
        j.live = false;
        j.sid = -1;
        ++j.seg;
        {
            std::lock_guard<std::mutex> lock(mutex_);
            ++j.info.segments_done;
        }
        if (!sink_ok) {
            j.cancel.store(true);
            end_job(j, GenJobState::Cancelled, "cancelled");
            return;
        }
        size_t next = j.seg;
        while (next < j.req.segments.size() && j.req.segments[next].empty()) ++next;
        if (next >= j.req.segments.size()) end_job(j, GenJobState::Completed, "");
    }

    Ops &ops_;
    BatchRuntimeOptions opt_;
    mutable std::mutex mutex_;
    std::condition_variable job_added_, job_done_;
    std::deque<std::shared_ptr<Job>> queue_;
    std::vector<std::shared_ptr<Job>> jobs_;     // recent jobs, for job() / wait()
    std::vector<std::shared_ptr<Job>> running_;  // worker-side
    std::atomic<int> running_count_{0};
    std::atomic<int64_t> load_{0};
    bool stop_ = false;
    std::thread worker_;
    uint64_t counter_ = 0;
};

// Several engines (one per GPU) behind one job API.  Each shard is a BatchRuntime with its own
// worker thread, so every GPU has its own scheduler thread and stream of engine calls; the
// streams of an utterance never leave their GPU and no data crosses between GPUs.  A new job
// goes to the shard with the least outstanding work (longest-processing-time greedy on
// BatchRuntime::job_cost; a shard whose queue is full is passed over).  A voice prefix lives on
// every shard: set_prefix registers its stream on each engine under one slot number, and a
// request's prefix_stream names that slot.
template <class Ops>
class ShardedRuntime {
public:
    ShardedRuntime(const std::vector<Ops *> &engines, BatchRuntimeOptions opt) {
        for (Ops *o : engines) rts_.push_back(std::make_unique<BatchRuntime<Ops>>(*o, opt));
    }
    int shards() const { return static_cast<int>(rts_.size()); }
    BatchRuntime<Ops> &shard(int i) { return *rts_[static_cast<size_t>(i)]; }
    void start() {
        for (auto &r : rts_) r->start();
    }
    void shutdown() {
        for (auto &r : rts_) r->shutdown();
    }

    // Prefix slot `slot`: stream stream_per_shard[i] on engine i, its first `len` positions.
    void set_prefix(int slot, const std::vector<int> &stream_per_shard, int len) {
        if (stream_per_shard.size() != rts_.size()) throw std::invalid_argument("one prefix stream per shard");
        std::lock_guard<std::mutex> lock(mutex_);
        prefixes_[slot] = {stream_per_shard, len};
    }

    // As BatchRuntime::submit; shard_out (may be null) receives the shard that took the job.
    bool submit(const GenJobRequest &req, CodeSink sink, std::string *job_id, std::string *err,
                int *shard_out = nullptr) {
        std::vector<int> order(rts_.size());
        for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int>(i);
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int b) { return rts_[size_t(a)]->load() < rts_[size_t(b)]->load(); });
        GenJobRequest r = req;
        std::vector<int> prefix_streams;
        {
            std::lock_guard<std::mutex> lock(mutex_);
            if (r.id.empty()) r.id = make_id_locked();
            if (req.prefix_stream >= 0) {
                auto it = prefixes_.find(req.prefix_stream);
                if (it == prefixes_.end()) {
                    if (err) *err = "unknown prefix slot";
                    return false;
                }
                prefix_streams = it->second.first;
                r.prefix_len = it->second.second;
            }
        }
        std::string why = "busy";
        for (int s : order) {
            if (req.prefix_stream >= 0) r.prefix_stream = prefix_streams[static_cast<size_t>(s)];
            std::string e;
            if (rts_[static_cast<size_t>(s)]->submit(r, sink, job_id, &e)) {
                std::lock_guard<std::mutex> lock(mutex_);
                where_[r.id] = s;
                prune_locked();
                if (shard_out) *shard_out = s;
                return true;
            }
            if (e != "busy") why = e;
        }
        if (err) *err = why;
        return false;
    }

    bool wait(const std::string &id, int timeout_ms, GenJobInfo *out) {
        const int s = find(id);
        return s >= 0 && rts_[static_cast<size_t>(s)]->wait(id, timeout_ms, out);
    }
    bool job(const std::string &id, GenJobInfo *out) const {
        const int s = find(id);
        return s >= 0 && rts_[static_cast<size_t>(s)]->job(id, out);
    }
    bool cancel(const std::string &id) {
        const int s = find(id);
        return s >= 0 && rts_[static_cast<size_t>(s)]->cancel(id);
    }
    int queue_depth() const {
        int d = 0;
        for (auto &r : rts_) d += r->queue_depth();
        return d;
    }

private:
    int find(const std::string &id) const {
        std::lock_guard<std::mutex> lock(mutex_);
        auto it = where_.find(id);
        return it == where_.end() ? -1 : it->second;
    }
    std::string make_id_locked() {
        ++counter_;
        char buf[40];
        std::snprintf(buf, sizeof(buf), "s%08llx%04llx", static_cast<unsigned long long>(counter_),
                      static_cast<unsigned long long>(std::chrono::steady_clock::now().time_since_epoch().count() & 0xFFFF));
        return buf;
    }
    // forget jobs their shard no longer keeps (BatchRuntime keeps the recent kKeepJobs)
    void prune_locked() {
        if (where_.size() <= 4 * rts_.size() * BatchRuntime<Ops>::kKeepJobs) return;
        for (auto it = where_.begin(); it != where_.end();)
            it = rts_[static_cast<size_t>(it->second)]->job(it->first, nullptr) ? std::next(it) : where_.erase(it);
    }

    std::vector<std::unique_ptr<BatchRuntime<Ops>>> rts_;
    mutable std::mutex mutex_;
    std::map<int, std::pair<std::vector<int>, int>> prefixes_;
    std::map<std::string, int> where_;
    uint64_t counter_ = 0;
};

}  // namespace gpu
}  // namespace moss
