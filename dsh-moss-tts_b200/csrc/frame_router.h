// frame_router.h -- the hand-off between the batched LLM step and the per-utterance codec
// decoders, for a Runtime that advances many jobs with one mossgpu_step / mossgpu_step_frames
// call.  Header-only C++17, host side.
//
// The reference hands frames from one LlmModel::generate thread to one decoder through a
// bounded queue (engine.cpp:91-124): the producer blocks while the queue is full,
// the consumer pops rows and, once enough are pending, turns them into an nq-major code block
// [16][n] for decode_chunk -- the first block after min(4, chunk_frames) frames, later blocks
// after chunk_frames frames, the remainder when the stream ends (engine.cpp:480-502).
//
// Here one batched step produces a frame for every live job at once:
//   FrameQueue     - a stream's bounded ring of Row = [text id, code0..15], filled in bulk
//                    straight from a step result's code array;
//   FrameRouter    - one FrameQueue per stream id; dispatch() pushes the rows of a
//                    mossgpu_step result (codes [n][16], stop[n]) or of a mossgpu_step_frames
//                    result (codes [frames][n][16], frames_done[n]) to their streams' queues and
//                    closes the queue of every stream whose utterance ended;
//   ChunkAssembler - the consumer side: collects rows and emits nq-major blocks with the
//                    reference's first-block rule.
// A stream's queue is closed when its generate would have returned: on the end gate (stop) or
// when step_frames stopped early for it; close() also lets a consumer that cancelled drain.
#pragma once

#include <algorithm>
#include <array>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <vector>

namespace moss {
namespace gpu {

constexpr int kRouterNVq = 16;
using FrameRow = std::array<int32_t, kRouterNVq + 1>;  // [text id, code0..15], as moss::Row

// A stream's frames between the batched step and its codec consumer: a fixed ring of
// `capacity` rows, allocated once, that a step result is copied into straight from its code
// array (append(), many frames at a time for a mossgpu_step_frames result).  The writer
// blocks while the ring is full, so a slow decoder holds back its own stream only; the reader
// blocks while it is empty.  finish() marks the end of the utterance: the reader drains what
// is left and then sees the end, and a writer that is still waiting gives up (the rows it had
// not written are dropped, as after a cancel).  One mutex guards the ring and one condition
// variable wakes both sides: each side waits for a different predicate on the same counters.
class FrameQueue {
public:
    explicit FrameQueue(size_t capacity) : ring_(capacity ? capacity : 1) {}

    // Appends `frames` rows whose 16 codes start at codes + f * stride, each behind the text
    // id `text` (0 in generate's rows).  Returns the rows written (< frames once finished).
    size_t append(const int32_t *codes, size_t frames, size_t stride, int32_t text = 0) {
        std::unique_lock<std::mutex> lk(mu_);
        size_t done = 0;
        while (done < frames) {
            cv_.wait(lk, [&] { return ended_ || count_ < ring_.size(); });
            if (ended_) break;
            const size_t room = std::min(ring_.size() - count_, frames - done);
            for (size_t k = 0; k < room; ++k, ++done) {
                FrameRow &row = ring_[(head_ + count_ + k) % ring_.size()];
                row[0] = text;
                std::copy(codes + done * stride, codes + done * stride + kRouterNVq, row.begin() + 1);
            }
            count_ += room;
            cv_.notify_all();
        }
        return done;
    }
    // One complete row (text id included).
    void push(const FrameRow &row) { append(row.data() + 1, 1, 0, row[0]); }

    // Takes the oldest row; false once the utterance ended and the ring is drained.
    bool pop(FrameRow *row) {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return ended_ || count_ > 0; });
        if (count_ == 0) return false;
        *row = ring_[head_];
        head_ = (head_ + 1) % ring_.size();
        --count_;
        cv_.notify_all();
        return true;
    }
    void finish() {
        std::lock_guard<std::mutex> lk(mu_);
        ended_ = true;
        cv_.notify_all();
    }
    void close() { finish(); }
    bool closed() const {
        std::lock_guard<std::mutex> lk(mu_);
        return ended_;
    }
    size_t size() const {
        std::lock_guard<std::mutex> lk(mu_);
        return count_;
    }

private:
    mutable std::mutex mu_;
    std::condition_variable cv_;
    std::vector<FrameRow> ring_;
    size_t head_ = 0, count_ = 0;
    bool ended_ = false;
};

class FrameRouter {
public:
    explicit FrameRouter(size_t capacity_per_stream) : capacity_(capacity_per_stream) {}

    // A queue for a stream that is about to generate (replaces a closed one).
    FrameQueue &open(int stream_id) {
        std::lock_guard<std::mutex> lock(mutex_);
        auto &q = queues_[stream_id];
        q = std::make_shared<FrameQueue>(capacity_);
        return *q;
    }
    // The stream's queue; throws if the stream was never opened.
    FrameQueue &queue(int stream_id) { return *get(stream_id); }
    void close(int stream_id) { get(stream_id)->close(); }

    // One mossgpu_step result: codes[n][16] the model's predictions, stop[n] the end gate.
    // Rows of streams that did not stop go to their queues; a stopped stream's queue closes.
    void dispatch(const int32_t *stream_ids, int n, const int32_t *codes, const uint8_t *stop) {
        for (int i = 0; i < n; ++i) {
            auto q = get(stream_ids[i]);
            if (stop && stop[i]) {
                q->close();
                continue;
            }
            q->append(codes + static_cast<size_t>(i) * kRouterNVq, 1, 0);
        }
    }
    // One mossgpu_step_frames result: codes[frames][n][16], frames_done[n] (the frames each
    // stream completed; fewer than `frames` means it ended inside the call).
    void dispatch_frames(const int32_t *stream_ids, int n, int frames, const int32_t *codes,
                         const int32_t *frames_done) {
        for (int i = 0; i < n; ++i) {
            auto q = get(stream_ids[i]);
            const int done = frames_done ? frames_done[i] : frames;
            // the stream's rows sit n rows apart in the [frames][n][16] result
            q->append(codes + static_cast<size_t>(i) * kRouterNVq, static_cast<size_t>(std::min(done, frames)),
                      static_cast<size_t>(n) * kRouterNVq);
            if (done < frames) q->close();
        }
    }

private:
    std::shared_ptr<FrameQueue> get(int stream_id) {
        std::lock_guard<std::mutex> lock(mutex_);
        auto it = queues_.find(stream_id);
        if (it == queues_.end() || !it->second) throw std::runtime_error("frame router: stream not opened");
        return it->second;
    }
    size_t capacity_;
    std::mutex mutex_;
    std::map<int, std::shared_ptr<FrameQueue>> queues_;
};

// Consumer side (engine.cpp:480-502): rows in, nq-major code blocks [16][n] out for
// decode_chunk.  The first block is emitted once min(4, chunk_frames) rows are pending, later
// ones at chunk_frames rows; flush() emits the remainder.
class ChunkAssembler {
public:
    explicit ChunkAssembler(int chunk_frames) : chunk_frames_(chunk_frames > 0 ? chunk_frames : 1) {}

    // Adds a row; returns true with the block in `codes` (size 16 n) when one is ready.
    bool push(const FrameRow &row, std::vector<int32_t> *codes, int *n) {
        pending_.push_back(row);
        const size_t want = emitted_ == 0 ? std::min<size_t>(4, static_cast<size_t>(chunk_frames_))
                                          : static_cast<size_t>(chunk_frames_);
        if (pending_.size() < want) return false;
        return take(codes, n);
    }
    // The rows still pending, if any.
    bool flush(std::vector<int32_t> *codes, int *n) {
        if (pending_.empty()) return false;
        return take(codes, n);
    }
    int frames_emitted() const { return emitted_; }

private:
    bool take(std::vector<int32_t> *codes, int *n) {
        const int m = static_cast<int>(pending_.size());
        codes->assign(static_cast<size_t>(m) * kRouterNVq, 0);
        for (int ch = 0; ch < kRouterNVq; ++ch)
            for (int j = 0; j < m; ++j)
                (*codes)[static_cast<size_t>(ch) * m + j] = pending_[static_cast<size_t>(j)][static_cast<size_t>(ch) + 1];
        *n = m;
        emitted_ += m;
        pending_.clear();
        return true;
    }
    int chunk_frames_;
    int emitted_ = 0;
    std::vector<FrameRow> pending_;
};

}  // namespace gpu
}  // namespace moss
