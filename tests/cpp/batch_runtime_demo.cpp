// BatchRuntime over the real engine (MossGpuOps, the C ABI): reads a job file, runs every job
// through the runtime's worker thread, and writes what each job's sink received.
//
//   batch_runtime_demo <weights.moss> <jobs.bin> <out.txt> <max_active> <frames_per_call> [n_gpus]
//
// With n_gpus > 1 the jobs go through ShardedRuntime over one engine per GPU (devices
// 0..n_gpus-1), the prefix prefilled on each and registered as slot 0.
//
// jobs.bin (int32 little endian): n_jobs, prefix_m, prefix rows [prefix_m][17], then per job
// seed, greedy, rep_x1000, min_frames, max_frames, chunk_frames, use_prefix, m, rows [m][17].
// out.txt: per job "job <i> <state> <frames> <shard>", then one "blk <segment> <n> <16 n codes>" line
// per block.  Exit 0 when every job ended (in any state), 2 on a load or input error.
//
// With MOSS_DEMO_DECODER=<decoder .moss> in the environment (one GPU), every job's sink also
// decodes its blocks through its own stream of one GPU codec (CodecStreams, codec_gpu.h), and
// each job's samples go to <out.txt>.pcm<i> (float32, interleaved stereo).
#include "batch_runtime.h"
#include "codec_gpu.h"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

using namespace moss::gpu;

namespace {

constexpr int kMaxCtx = 512;
constexpr int kMaxStreams = 16;

bool read_ints(std::ifstream &f, int32_t *v, size_t n) {
    f.read(reinterpret_cast<char *>(v), static_cast<std::streamsize>(n * sizeof(int32_t)));
    return static_cast<size_t>(f.gcount()) == n * sizeof(int32_t);
}

bool read_rows(std::ifstream &f, int m, std::vector<FrameRow> *rows) {
    rows->resize(static_cast<size_t>(m));
    for (auto &r : *rows)
        if (!read_ints(f, r.data(), r.size())) return false;
    return true;
}

}  // namespace

int main(int argc, char **argv) {
    if (argc != 6 && argc != 7) {
        std::fprintf(stderr, "usage: %s weights jobs.bin out.txt max_active frames_per_call [n_gpus]\n", argv[0]);
        return 2;
    }
    const int n_gpus = argc == 7 ? std::atoi(argv[6]) : 1;
    if (n_gpus < 1 || n_gpus > 8) return 2;
    std::ifstream in(argv[2], std::ios::binary);
    int32_t hdr[2];
    if (!in || !read_ints(in, hdr, 2)) {
        std::fprintf(stderr, "bad job file\n");
        return 2;
    }
    std::vector<FrameRow> prefix;
    if (!read_rows(in, hdr[1], &prefix)) return 2;
    std::vector<GenJobRequest> jobs(static_cast<size_t>(hdr[0]));
    std::vector<int> use_prefix(jobs.size());
    for (size_t i = 0; i < jobs.size(); ++i) {
        int32_t v[8];
        if (!read_ints(in, v, 8)) return 2;
        GenJobRequest &r = jobs[i];
        r.id = "job" + std::to_string(i);
        r.seed = static_cast<uint64_t>(v[0]);
        r.greedy = v[1] != 0;
        r.repetition_penalty = static_cast<float>(v[2]) / 1000.0f;
        r.min_frames = v[3];
        r.max_frames = v[4];
        r.chunk_frames = v[5];
        use_prefix[i] = v[6];
        r.segments.emplace_back();
        if (!read_rows(in, v[7], &r.segments.back())) return 2;
    }

    std::vector<mossgpu_engine *> hs;
    std::vector<int> prefix_sid;
    for (int d = 0; d < n_gpus; ++d) {
        char err[1024] = {0};
        mossgpu_engine *h = mossgpu_create(argv[1], d, kMaxStreams, kMaxCtx, 0, err, sizeof(err));
        if (!h) {
            std::fprintf(stderr, "load failed on device %d: %s\n", d, err);
            for (auto *o : hs) mossgpu_destroy(o);
            return 2;
        }
        hs.push_back(h);
        int sid = -1;
        if (!prefix.empty()) {
            if (mossgpu_stream_open(h, &sid) != 0 ||
                mossgpu_prefill(h, sid, prefix[0].data(), static_cast<int>(prefix.size()), 0) != 0) {
                std::fprintf(stderr, "prefix: %s\n", mossgpu_last_error(h));
                for (auto *o : hs) mossgpu_destroy(o);
                return 2;
            }
        }
        prefix_sid.push_back(sid);
    }
    int rc = 0;
    {
        std::vector<MossGpuOps> ops;
        for (auto *h : hs) ops.emplace_back(h, kMaxCtx);
        const BatchRuntimeOptions opt{std::atoi(argv[4]), 64, std::atoi(argv[5])};
        std::unique_ptr<BatchRuntime<MossGpuOps>> single;
        std::unique_ptr<ShardedRuntime<MossGpuOps>> sharded;
        if (n_gpus == 1) {
            single = std::make_unique<BatchRuntime<MossGpuOps>>(ops[0], opt);
        } else {
            std::vector<MossGpuOps *> ptrs;
            for (auto &o : ops) ptrs.push_back(&o);
            sharded = std::make_unique<ShardedRuntime<MossGpuOps>>(ptrs, opt);
            sharded->set_prefix(0, prefix_sid, static_cast<int>(prefix.size()));
        }
        for (size_t i = 0; i < jobs.size(); ++i)
            if (use_prefix[i]) {
                jobs[i].prefix_stream = single ? prefix_sid[0] : 0;  // sharded: the slot
                jobs[i].prefix_len = static_cast<int>(prefix.size());
            }
        std::vector<std::vector<std::string>> blocks(jobs.size());
        std::vector<std::string> ids(jobs.size());
        std::vector<int> shard(jobs.size(), 0);
        const char *dec_path = std::getenv("MOSS_DEMO_DECODER");
        std::unique_ptr<CodecStreams> codec;
        std::vector<std::unique_ptr<CodecStreams::Stream>> dec(jobs.size());
        std::vector<std::vector<float>> pcm(jobs.size());
        if (dec_path && *dec_path && n_gpus == 1) {
            codec = std::make_unique<CodecStreams>(dec_path, 0, static_cast<int>(jobs.size()), 16);
            for (auto &d : dec) d = codec->open();
        }
        for (size_t i = 0; i < jobs.size(); ++i) {
            std::string e;
            auto sink = [&blocks, &dec, &pcm, i](int segment, const int32_t *codes, int n) {
                std::string line = "blk " + std::to_string(segment) + " " + std::to_string(n);
                for (int k = 0; k < 16 * n; ++k) line += " " + std::to_string(codes[k]);
                blocks[i].push_back(line);
                if (dec[i]) {  // the job's codec stream, in block order (engine.cpp:480-502)
                    std::vector<float> audio;
                    std::string why;
                    if (!dec[i]->decode(segment, codes, n, &audio, &why)) {
                        std::fprintf(stderr, "decode %zu: %s\n", i, why.c_str());
                        return false;
                    }
                    pcm[i].insert(pcm[i].end(), audio.begin(), audio.end());
                }
                return true;
            };
            const bool ok = single ? single->submit(jobs[i], sink, &ids[i], &e)
                                   : sharded->submit(jobs[i], sink, &ids[i], &e, &shard[i]);
            if (!ok) {
                std::fprintf(stderr, "submit %zu: %s\n", i, e.c_str());
                rc = 2;
            }
        }
        if (single)
            single->start();
        else
            sharded->start();
        std::ofstream out(argv[3]);
        for (size_t i = 0; i < jobs.size() && rc == 0; ++i) {
            GenJobInfo info;
            const bool ended = single ? single->wait(ids[i], 120000, &info) : sharded->wait(ids[i], 120000, &info);
            if (!ended) {
                std::fprintf(stderr, "job %zu did not end\n", i);
                rc = 2;
                break;
            }
            out << "job " << i << " " << gen_job_state_name(info.state) << " " << info.frames << " " << shard[i] << "\n";
            if (!info.error.empty()) std::fprintf(stderr, "job %zu: %s\n", i, info.error.c_str());
            for (auto &l : blocks[i]) out << l << "\n";
        }
        if (single)
            single->shutdown();
        else
            sharded->shutdown();
        for (size_t i = 0; i < jobs.size() && codec; ++i) {
            std::ofstream f(std::string(argv[3]) + ".pcm" + std::to_string(i), std::ios::binary);
            f.write(reinterpret_cast<const char *>(pcm[i].data()), static_cast<std::streamsize>(pcm[i].size() * 4));
        }
    }
    for (auto *h : hs) mossgpu_destroy(h);
    return rc;
}
