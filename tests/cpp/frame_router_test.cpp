// Host test of moss::gpu::FrameRouter / ChunkAssembler (frame_router.h): batched step results
// routed to per-stream bounded queues, consumed by one thread per stream that assembles
// nq-major code blocks as the reference's TtsEngine does (first block 4 frames, then
// chunk_frames).  Prints one line per stream: id, frames, block sizes; exits 1 on a mismatch.
#include <cstdio>
#include <thread>
#include <vector>

#include "frame_router.h"

using moss::gpu::ChunkAssembler;
using moss::gpu::FrameRouter;
using moss::gpu::FrameRow;

static int code_of(int sid, int frame, int ch) { return (sid * 131 + frame * 17 + ch * 7) % 1024; }

int main() {
    const std::vector<int> sids = {5, 9, 11, 2};
    const int chunk = 8;
    FrameRouter router(3);  // small queues: the producer must block and resume
    for (int s : sids) router.open(s);
    std::vector<std::vector<int>> blocks(sids.size());
    std::vector<int> frames(sids.size(), 0), bad(sids.size(), 0);
    std::vector<std::thread> consumers;
    for (size_t k = 0; k < sids.size(); ++k) {
        consumers.emplace_back([&, k] {
            ChunkAssembler asm_(chunk);
            FrameRow row;
            std::vector<int32_t> codes;
            int n = 0;
            auto check = [&](int first) {
                for (int ch = 0; ch < 16; ++ch)
                    for (int j = 0; j < n; ++j)
                        if (codes[static_cast<size_t>(ch) * n + j] != code_of(sids[k], first + j, ch)) bad[k] = 1;
                blocks[k].push_back(n);
            };
            while (router.queue(sids[k]).pop(&row)) {
                const int first = asm_.frames_emitted();
                if (asm_.push(row, &codes, &n)) check(first);
                ++frames[k];
            }
            const int first = asm_.frames_emitted();
            if (asm_.flush(&codes, &n)) check(first);
        });
    }
    // producer: 3 step_frames calls of 6 frames, then single steps; stream 9 ends inside the
    // second call (frames_done 4), stream 11 on the end gate at its frame 20, stream 2 when
    // the caller closes it after 22 frames, stream 5 runs to 25 frames
    int frame_of[4] = {0, 0, 0, 0};
    bool live[4] = {true, true, true, true};
    for (int call = 0; call < 3; ++call) {
        std::vector<int32_t> ids, codes, done;
        std::vector<int> idx;
        for (int k = 0; k < 4; ++k)
            if (live[k]) {
                ids.push_back(sids[static_cast<size_t>(k)]);
                idx.push_back(k);
            }
        const int n = static_cast<int>(ids.size());
        codes.assign(static_cast<size_t>(6) * n * 16, 0);
        for (int f = 0; f < 6; ++f)
            for (int i = 0; i < n; ++i)
                for (int ch = 0; ch < 16; ++ch)
                    codes[(static_cast<size_t>(f) * n + i) * 16 + ch] = code_of(ids[static_cast<size_t>(i)], frame_of[idx[static_cast<size_t>(i)]] + f, ch);
        for (int i = 0; i < n; ++i) {
            const int k = idx[static_cast<size_t>(i)];
            const int d = (sids[static_cast<size_t>(k)] == 9 && call == 1) ? 4 : 6;
            done.push_back(d);
            frame_of[k] += d;
            if (d < 6) live[k] = false;
        }
        router.dispatch_frames(ids.data(), n, 6, codes.data(), done.data());
    }
    for (int step = 0; step < 8; ++step) {
        std::vector<int32_t> ids, codes;
        std::vector<uint8_t> stop;
        std::vector<int> idx;
        for (int k = 0; k < 4; ++k)
            if (live[k]) {
                ids.push_back(sids[static_cast<size_t>(k)]);
                idx.push_back(k);
            }
        if (ids.empty()) break;
        for (size_t i = 0; i < ids.size(); ++i) {
            const int k = idx[i];
            for (int ch = 0; ch < 16; ++ch) codes.push_back(code_of(ids[i], frame_of[k], ch));
            const bool gate = sids[static_cast<size_t>(k)] == 11 && frame_of[k] == 20;
            stop.push_back(gate ? 1 : 0);
            if (gate) live[k] = false;
            else ++frame_of[k];
        }
        router.dispatch(ids.data(), static_cast<int>(ids.size()), codes.data(), stop.data());
        for (size_t i = 0; i < ids.size(); ++i) {
            const int k = idx[i];
            if (!live[k]) continue;
            if ((sids[static_cast<size_t>(k)] == 2 && frame_of[k] == 22) || (sids[static_cast<size_t>(k)] == 5 && frame_of[k] == 25)) {
                router.close(sids[static_cast<size_t>(k)]);
                live[k] = false;
            }
        }
    }
    for (auto &t : consumers) t.join();
    int rc = 0;
    for (size_t k = 0; k < sids.size(); ++k) {
        std::printf("%d %d", sids[k], frames[k]);
        for (int b : blocks[k]) std::printf(" %d", b);
        std::printf("\n");
        rc |= bad[k];
    }
    return rc;
}
