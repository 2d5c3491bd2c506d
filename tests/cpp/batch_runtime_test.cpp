// BatchRuntime (batch_runtime.h) on a host-only test double of the engine.  The double's
// codes and end gate depend only on a stream's own contents, the frame index, the sampling
// parameters and the seed, so a job must produce the same blocks however the runtime
// batches it.  Expected blocks come from a sequential restatement of TtsEngine::synthesize's
// frame loop (one frame per call, reference engine.cpp:455-530) with its own chunking
// (decode_pending, engine.cpp:480-502).  Exit 0 = all checks passed; failures print and exit 1.
#include "batch_runtime.h"
#include "fake_engine.h"

#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

using namespace moss::gpu;

namespace {

int g_failures = 0;
#define CHECK(cond, ...)                                   \
    do {                                                   \
        if (!(cond)) {                                     \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                      \
            std::printf("\n");                             \
            ++g_failures;                                  \
        }                                                  \
    } while (0)

using namespace fake;

std::vector<GenJobRequest> mixed_jobs(int prefix_sid, int prefix_len) {
    std::vector<GenJobRequest> jobs;
    for (int i = 0; i < 12; ++i) {
        GenJobRequest r;
        r.seed = 100 + static_cast<uint64_t>(i);
        const int nseg = 1 + i % 3;
        for (int k = 0; k < nseg; ++k) r.segments.push_back(rows_of(3 + (i * 5 + k * 7) % 17, static_cast<uint64_t>(i * 10 + k)));
        if (i == 4) r.segments.insert(r.segments.begin() + 1, std::vector<FrameRow>{});  // empty text segment
        r.greedy = i % 2 == 0;
        r.repetition_penalty = i % 4 == 1 ? 1.1f : 0.0f;
        r.min_frames = i % 5 == 0 ? 3 : 0;
        r.chunk_frames = (i % 4 == 0) ? 1 : (i % 4 == 1) ? 3 : (i % 4 == 2) ? 0 : 8;
        r.max_frames = (i % 3 == 0) ? 5 : (i % 3 == 1) ? 40 : 0;
        if (i % 2 == 1) {
            r.prefix_stream = prefix_sid;
            r.prefix_len = prefix_len - (i % 3);
        }
        jobs.push_back(r);
    }
    return jobs;
}

struct Collected {  // sinks of several worker threads (one per shard) write here
    std::map<std::string, std::vector<Block>> blocks;
    std::mutex mu;
    CodeSink sink_for(const std::string &key) {
        {
            std::lock_guard<std::mutex> lock(mu);
            blocks[key];  // the entry exists before any worker writes
        }
        return [this, key](int segment, const int32_t *codes, int n) {
            std::lock_guard<std::mutex> lock(mu);
            blocks[key].push_back(Block{segment, std::vector<int32_t>(codes, codes + 16 * n)});
            return true;
        };
    }
};

void drain(BatchRuntime<FakeOps> &rt) {
    for (int it = 0; it < 100000 && rt.run_once(); ++it) {
    }
}

// A: batched results equal the sequential ones; calls really batch; every stream closes.
void test_batched_equals_sequential() {
    FakeOps eng(16, 4096), ref(16, 4096);
    const int psid = setup_prefix(eng, 20), rsid = setup_prefix(ref, 20);
    CHECK(psid == rsid, "prefix stream ids differ");
    auto jobs = mixed_jobs(psid, 20);
    BatchRuntime<FakeOps> rt(eng, BatchRuntimeOptions{8, 64, 4});
    Collected got;
    std::vector<std::string> ids;
    for (size_t i = 0; i < jobs.size(); ++i) {
        std::string id, err;
        jobs[i].id = "job" + std::to_string(i);
        CHECK(rt.submit(jobs[i], got.sink_for(jobs[i].id), &id, &err), "submit %zu: %s", i, err.c_str());
        CHECK(id == jobs[i].id, "job id");
        ids.push_back(id);
    }
    drain(rt);
    int total_frames = 0;
    for (size_t i = 0; i < jobs.size(); ++i) {
        GenJobInfo info;
        CHECK(rt.job(ids[i], &info), "job %zu missing", i);
        CHECK(info.state == GenJobState::Completed, "job %zu state %s (%s)", i, gen_job_state_name(info.state), info.error.c_str());
        const auto want = expected_blocks(ref, jobs[i]);
        CHECK(got.blocks[ids[i]] == want, "job %zu: %zu blocks, expected %zu", i, got.blocks[ids[i]].size(), want.size());
        int frames = 0;
        for (auto &b : want) frames += static_cast<int>(b.codes.size() / 16);
        CHECK(info.frames == frames, "job %zu frames %d vs %d", i, info.frames, frames);
        const int nonempty = static_cast<int>(jobs[i].segments.size()) - (i == 4 ? 1 : 0);
        CHECK(info.segments_done == nonempty, "job %zu segments %d", i, info.segments_done);
        total_frames += frames;
    }
    CHECK(eng.open_streams() == 1, "streams left open: %d", eng.open_streams() - 1);
    int pmax = 0, smax = 0, fmax = 0;
    for (int n : eng.prefill_n) pmax = std::max(pmax, n);
    for (int n : eng.step_n) smax = std::max(smax, n);
    for (int n : eng.step_frames_n) fmax = std::max(fmax, n);
    CHECK(pmax > 1 && smax > 1, "no batching: prefill %d step %d", pmax, smax);
    CHECK(smax <= 8 && fmax <= 4, "limits: %d streams, %d frames per call", smax, fmax);
    std::printf("A frames=%d prefill_calls=%zu prefill_max=%d step_calls=%zu step_max=%d\n", total_frames,
                eng.prefill_n.size(), pmax, eng.step_n.size(), smax);
}

// B: queue limit, cancel while queued, cancel while running, a failing sink, shutdown.
void test_queue_cancel_sink() {
    FakeOps eng(8, 4096);
    BatchRuntime<FakeOps> rt(eng, BatchRuntimeOptions{1, 2, 2});
    GenJobRequest r;
    r.segments.push_back(rows_of(6, 1));
    r.max_frames = 300;
    r.min_frames = 200;  // no end gate before frame 200
    std::string a, b, c, err;
    Collected got;
    CHECK(rt.submit(r, got.sink_for("a"), &a, &err), "submit a");
    CHECK(rt.submit(r, got.sink_for("b"), &b, &err), "submit b");
    CHECK(!rt.submit(r, nullptr, &c, &err) && err == "busy", "third submit: %s", err.c_str());
    CHECK(rt.queue_depth() == 2, "queue depth %d", rt.queue_depth());
    CHECK(a != b && a.size() == 12, "generated ids");
    rt.run_once();  // admits a (max_active 1), prefills, one 2-frame call
    CHECK(rt.queue_depth() == 1 && rt.running() == 1, "after one iteration");
    CHECK(rt.cancel(b), "cancel b");
    rt.run_once();
    CHECK(rt.cancel(a), "cancel a");
    drain(rt);
    GenJobInfo ia, ib;
    rt.job(a, &ia);
    rt.job(b, &ib);
    // a: two 2-frame calls made its first 4-frame block; the frames after cancel are dropped
    CHECK(ia.state == GenJobState::Cancelled && ia.frames == 4, "a: %s %d", gen_job_state_name(ia.state), ia.frames);
    CHECK(ib.state == GenJobState::Cancelled && ib.frames == 0, "b: %s", gen_job_state_name(ib.state));
    CHECK(eng.prefill_n.size() == 1, "b never reached the engine");
    CHECK(eng.open_streams() == 0, "cancelled stream left open");

    // a sink that fails on its second block
    GenJobRequest s = r;
    s.chunk_frames = 2;
    int calls = 0;
    std::string d;
    CHECK(rt.submit(s, [&](int, const int32_t *, int) { return ++calls < 2; }, &d, &err), "submit d");
    drain(rt);
    GenJobInfo id_;
    rt.job(d, &id_);
    CHECK(id_.state == GenJobState::Cancelled && calls == 2 && id_.frames == 4, "d: %s calls %d frames %d",
          gen_job_state_name(id_.state), calls, id_.frames);
    CHECK(eng.open_streams() == 0, "sink-cancelled stream left open");

    // a throwing sink fails the same way
    std::string t;
    CHECK(rt.submit(s, [&](int, const int32_t *, int) -> bool { throw std::runtime_error("x"); }, &t, &err), "submit t");
    drain(rt);
    GenJobInfo it_;
    rt.job(t, &it_);
    CHECK(it_.state == GenJobState::Cancelled, "throwing sink: %s", gen_job_state_name(it_.state));

    // shutdown cancels queued jobs
    std::string e1, e2;
    rt.submit(r, nullptr, &e1, &err);
    rt.submit(r, nullptr, &e2, &err);
    rt.shutdown();
    GenJobInfo ie;
    rt.job(e2, &ie);
    CHECK(ie.state == GenJobState::Cancelled && ie.error == "shutting down", "shutdown: %s", ie.error.c_str());
    CHECK(!rt.submit(r, nullptr, &e1, &err) && err == "shutting down", "submit after shutdown");
    std::printf("B ok\n");
}

// C: a bad segment fails its own job only; the context cap ends a segment without error.
void test_failures_and_context_cap() {
    FakeOps eng(8, 4096), ref(8, 4096);
    BatchRuntime<FakeOps> rt(eng, BatchRuntimeOptions{8, 8, 16});
    std::vector<GenJobRequest> jobs(3);
    for (int i = 0; i < 3; ++i) {
        jobs[static_cast<size_t>(i)].segments.push_back(rows_of(5 + i, static_cast<uint64_t>(40 + i), i == 1 ? 2 : -1));
        jobs[static_cast<size_t>(i)].greedy = true;
        jobs[static_cast<size_t>(i)].seed = static_cast<uint64_t>(i);
    }
    Collected got;
    std::vector<std::string> ids(3);
    std::string err;
    for (int i = 0; i < 3; ++i) rt.submit(jobs[static_cast<size_t>(i)], got.sink_for(std::to_string(i)), &ids[static_cast<size_t>(i)], &err);
    drain(rt);
    for (int i = 0; i < 3; ++i) {
        GenJobInfo info;
        rt.job(ids[static_cast<size_t>(i)], &info);
        if (i == 1) {
            CHECK(info.state == GenJobState::Failed && info.error == "text id out of range", "bad job: %s %s",
                  gen_job_state_name(info.state), info.error.c_str());
        } else {
            CHECK(info.state == GenJobState::Completed, "good job %d: %s", i, info.error.c_str());
            CHECK(got.blocks[std::to_string(i)] == expected_blocks(ref, jobs[static_cast<size_t>(i)]), "good job %d blocks", i);
        }
    }
    CHECK(eng.open_streams() == 0, "failed job's stream left open");

    // context of 17 positions: 10 prompt rows leave 7 frames
    FakeOps small(4, 17), small_ref(4, 17);
    BatchRuntime<FakeOps> rt2(small, BatchRuntimeOptions{4, 4, 5});
    GenJobRequest r;
    r.segments.push_back(rows_of(10, 3));
    r.segments.push_back(rows_of(17, 4));  // fills the context: no frames
    r.min_frames = 100;
    r.chunk_frames = 3;
    std::string id;
    rt2.submit(r, got.sink_for("cap"), &id, &err);
    drain(rt2);
    GenJobInfo info;
    rt2.job(id, &info);
    CHECK(info.state == GenJobState::Completed && info.frames == 7 && info.segments_done == 2, "cap: %s frames %d (%s)",
          gen_job_state_name(info.state), info.frames, info.error.c_str());
    CHECK(got.blocks["cap"] == expected_blocks(small_ref, r), "cap blocks");
    std::printf("C ok\n");
}

// D: the worker thread with wait().
void test_worker_thread() {
    FakeOps eng(16, 4096), ref(16, 4096);
    const int psid = setup_prefix(eng, 12);
    setup_prefix(ref, 12);
    auto jobs = mixed_jobs(psid, 12);
    jobs.resize(8);
    BatchRuntime<FakeOps> rt(eng, BatchRuntimeOptions{4, 16, 8});
    Collected got;
    std::vector<std::string> ids(jobs.size());
    std::string err;
    for (size_t i = 0; i < jobs.size(); ++i)
        CHECK(rt.submit(jobs[i], got.sink_for(std::to_string(i)), &ids[i], &err), "submit %zu", i);
    rt.start();
    for (size_t i = 0; i < jobs.size(); ++i) {
        GenJobInfo info;
        CHECK(rt.wait(ids[i], 20000, &info), "wait %zu timed out", i);
        CHECK(info.state == GenJobState::Completed, "job %zu: %s", i, info.error.c_str());
    }
    rt.shutdown();
    for (size_t i = 0; i < jobs.size(); ++i)
        CHECK(got.blocks[std::to_string(i)] == expected_blocks(ref, jobs[i]), "threaded job %zu blocks", i);
    std::printf("D ok\n");
}

// E: two engines behind one ShardedRuntime: jobs spread by outstanding work, a voice prefix
// registered on both, every job's blocks as if run alone, loads back to zero at the end.
void test_sharded() {
    FakeOps e0(16, 4096), e1(16, 4096), ref(16, 4096);
    int busy = -1;
    e1.open(&busy);  // stream 0 of engine 1 is taken, so its prefix gets another stream id
    const int p0 = setup_prefix(e0, 9), p1 = setup_prefix(e1, 9), pref = setup_prefix(ref, 9);
    CHECK(p0 == 0 && p1 == 1 && pref == 0, "prefix streams %d %d %d", p0, p1, pref);
    ShardedRuntime<FakeOps> rt({&e0, &e1}, BatchRuntimeOptions{4, 16, 3});
    rt.set_prefix(7, {p0, p1}, 9);
    auto jobs = mixed_jobs(0, 9);
    for (auto &j : jobs) {
        if (j.prefix_stream >= 0) j.prefix_stream = 7;  // the slot
        j.prefix_len = 0;
    }
    Collected got;
    std::vector<std::string> ids(jobs.size());
    std::vector<int> where(jobs.size(), -1);
    int64_t cost[2] = {0, 0}, most = 0;
    std::string err;
    for (size_t i = 0; i < jobs.size(); ++i) {
        CHECK(rt.submit(jobs[i], got.sink_for(std::to_string(i)), &ids[i], &err, &where[i]), "submit %zu: %s", i, err.c_str());
        GenJobRequest as_run = jobs[i];
        if (as_run.prefix_stream >= 0) as_run.prefix_len = 9;
        const int64_t c = BatchRuntime<FakeOps>::job_cost(as_run);
        cost[where[i]] += c;
        most = std::max(most, c);
    }
    CHECK(rt.shard(0).load() == cost[0] && rt.shard(1).load() == cost[1], "loads before start");
    CHECK(std::llabs(cost[0] - cost[1]) <= most, "unbalanced: %lld vs %lld", (long long)cost[0], (long long)cost[1]);
    GenJobRequest bad = jobs[1];
    bad.prefix_stream = 3;
    std::string bid;
    CHECK(!rt.submit(bad, nullptr, &bid, &err) && err == "unknown prefix slot", "unknown slot: %s", err.c_str());
    rt.start();
    for (size_t i = 0; i < jobs.size(); ++i) {
        GenJobInfo info;
        CHECK(rt.wait(ids[i], 20000, &info), "wait %zu", i);
        CHECK(info.state == GenJobState::Completed, "sharded job %zu: %s", i, info.error.c_str());
        GenJobRequest as_run = jobs[i];
        if (as_run.prefix_stream >= 0) {
            as_run.prefix_stream = pref;
            as_run.prefix_len = 9;
        }
        CHECK(got.blocks[std::to_string(i)] == expected_blocks(ref, as_run), "sharded job %zu blocks", i);
    }
    rt.shutdown();
    CHECK(rt.shard(0).load() == 0 && rt.shard(1).load() == 0, "loads after the end");
    CHECK(e0.open_streams() == 1 && e1.open_streams() == 2, "streams left open");
    std::printf("E shard0_cost=%lld shard1_cost=%lld\n", (long long)cost[0], (long long)cost[1]);
}

// F: the admission hold groups late arrivals into one prefill pass.
void test_admission_hold() {
    FakeOps eng(16, 4096);
    BatchRuntimeOptions opt{8, 16, 2};
    opt.admit_min = 3;
    opt.admit_wait_ms = 600000;  // never expires within the test
    BatchRuntime<FakeOps> rt(eng, opt);
    GenJobRequest r;
    r.segments.push_back(rows_of(5, 11));
    r.min_frames = 1000;
    r.max_frames = 1000;
    std::string a, b, c, d, err;
    rt.submit(r, nullptr, &a, &err);
    rt.run_once();  // idle: admitted at once
    CHECK(rt.running() == 1 && eng.prefill_n.size() == 1, "idle runtime admits at once");
    rt.submit(r, nullptr, &b, &err);
    rt.submit(r, nullptr, &c, &err);
    rt.run_once();
    CHECK(rt.queue_depth() == 2 && rt.running() == 1, "two queued jobs are held");
    rt.submit(r, nullptr, &d, &err);
    rt.run_once();
    CHECK(rt.queue_depth() == 0 && rt.running() == 4, "the third releases them");
    CHECK(eng.prefill_n.size() == 2 && eng.prefill_n.back() == 3, "one prefill call for the three");
    for (const std::string &id : {a, b, c, d}) rt.cancel(id);
    drain(rt);
    CHECK(eng.open_streams() == 0, "streams left open");

    // no hold by default
    FakeOps eng2(16, 4096);
    BatchRuntime<FakeOps> rt2(eng2, BatchRuntimeOptions{8, 16, 2});
    rt2.submit(r, nullptr, &a, &err);
    rt2.run_once();
    rt2.submit(r, nullptr, &b, &err);
    rt2.run_once();
    CHECK(rt2.running() == 2 && eng2.prefill_n.size() == 2, "default admits every iteration");
    rt2.cancel(a);
    rt2.cancel(b);
    drain(rt2);
    std::printf("F ok\n");
}

}  // namespace

int main() {
    test_batched_equals_sequential();
    test_queue_cancel_sink();
    test_failures_and_context_cap();
    test_worker_thread();
    test_sharded();
    test_admission_hold();
    if (g_failures) {
        std::printf("%d failures\n", g_failures);
        return 1;
    }
    return 0;
}
