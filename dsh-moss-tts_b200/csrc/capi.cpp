// capi.cpp -- the extern "C" boundary (include/mossgpu.h) over mossgpu::Engine.
// Every entry point catches C++ exceptions and turns them into a non-zero status with the
// message kept on the handle, as the reference's capi.cpp does (capi.cpp:16-23,109).
#include "../../include/mossgpu.h"

#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>

#include "engine.h"

struct mossgpu_engine {
    std::unique_ptr<mossgpu::Engine> eng;
    std::string error;
};

namespace {

// The engine's device becomes the calling thread's current device first: a handle is used
// from threads other than its creator (a runtime worker, the reference's generate producer
// thread, engine.cpp:466-475), whose current device starts at 0.
void make_current(const mossgpu::Engine &g) {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d != g.device()) {
        const cudaError_t rc = cudaSetDevice(g.device());
        if (rc != cudaSuccess) throw std::runtime_error(std::string("cudaSetDevice: ") + cudaGetErrorString(rc));
    }
}

template <class F>
int guarded(mossgpu_engine *e, F &&f) {
    if (!e || !e->eng) return 1;
    try {
        make_current(*e->eng);
        f(*e->eng);
        e->error.clear();
        return 0;
    } catch (const std::exception &ex) {
        e->error = ex.what();
    } catch (...) {
        e->error = "unknown error";
    }
    return 1;
}

void copy_err(char *err, int errlen, const std::string &msg) {
    if (err && errlen > 0) {
        std::strncpy(err, msg.c_str(), size_t(errlen) - 1);
        err[errlen - 1] = 0;
    }
}

}  // namespace

extern "C" {

mossgpu_engine *mossgpu_create(const char *weights_path, int device_id, int max_streams, int max_ctx, int kv_pages,
                               char *err, int errlen) {
    return mossgpu_create_rows(weights_path, device_id, max_streams, max_ctx, kv_pages, 0, err, errlen);
}

mossgpu_engine *mossgpu_create_rows(const char *weights_path, int device_id, int max_streams, int max_ctx, int kv_pages,
                                    int max_rows, char *err, int errlen) {
    if (!weights_path) {
        copy_err(err, errlen, "weights_path is NULL");
        return nullptr;
    }
    try {
        auto *h = new mossgpu_engine();
        h->eng = std::make_unique<mossgpu::Engine>(weights_path, device_id, max_streams, max_ctx, kv_pages, max_rows);
        return h;
    } catch (const std::exception &ex) {
        copy_err(err, errlen, ex.what());
    } catch (...) {
        copy_err(err, errlen, "unknown error");
    }
    return nullptr;
}

void mossgpu_destroy(mossgpu_engine *e) { delete e; }

const char *mossgpu_last_error(mossgpu_engine *e) { return e ? e->error.c_str() : "null engine"; }

const char *mossgpu_version(void) { return "moss-b200 0.1.0 (sm_100a)"; }

int mossgpu_set_cuda_stream(mossgpu_engine *e, void *s) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_cuda_stream(s); });
}

int mossgpu_stream_open(mossgpu_engine *e, int *stream_id) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!stream_id) throw std::runtime_error("stream_id is NULL");
        *stream_id = g.open_stream();
    });
}

int mossgpu_stream_close(mossgpu_engine *e, int stream_id) {
    return guarded(e, [&](mossgpu::Engine &g) { g.close_stream(stream_id); });
}

int mossgpu_stream_reset(mossgpu_engine *e, int stream_id) {
    return guarded(e, [&](mossgpu::Engine &g) { g.reset_stream(stream_id); });
}

int mossgpu_stream_fork(mossgpu_engine *e, int src_stream, int n_pos, int *new_stream) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!new_stream) throw std::runtime_error("new_stream is NULL");
        *new_stream = g.fork_stream(src_stream, n_pos);
    });
}

int mossgpu_stream_position(mossgpu_engine *e, int stream_id, int *position) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!position) throw std::runtime_error("position is NULL");
        *position = g.position(stream_id);
    });
}

int mossgpu_prefill(mossgpu_engine *e, int stream_id, const int32_t *rows, int m, int start) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!rows && m > 0) throw std::runtime_error("rows is NULL");
        g.prefill(stream_id, rows, m, start);
    });
}

int mossgpu_prefill_embeds(mossgpu_engine *e, int stream_id, const float *x, int m, int start) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!x && m > 0) throw std::runtime_error("x is NULL");
        g.prefill_embeds(stream_id, x, m, start);
    });
}

int mossgpu_prefill_batch(mossgpu_engine *e, int n, const int32_t *stream_ids, const int32_t *m, const int32_t *start,
                          const int32_t *rows) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (n > 0 && (!stream_ids || !m || !start || !rows)) throw std::runtime_error("NULL argument");
        g.prefill_batch(n, stream_ids, m, start, rows, nullptr);
    });
}

int mossgpu_prefill_embeds_batch(mossgpu_engine *e, int n, const int32_t *stream_ids, const int32_t *m,
                                 const int32_t *start, const float *x) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (n > 0 && (!stream_ids || !m || !start || !x)) throw std::runtime_error("NULL argument");
        g.prefill_batch(n, stream_ids, m, start, nullptr, x);
    });
}

int mossgpu_set_tc_policy(mossgpu_engine *e, int direct_min_rows, int direct_rows) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_tc_policy(direct_min_rows, direct_rows); });
}

int mossgpu_generate_begin(mossgpu_engine *e, int stream_id, uint64_t seed) {
    return guarded(e, [&](mossgpu::Engine &g) { g.generate_begin(stream_id, seed); });
}

int mossgpu_step(mossgpu_engine *e, const int32_t *stream_ids, int n, const mossgpu_sample_params *params,
                 const int32_t *forced, int32_t *out_codes, uint8_t *out_stop, float *out_logits, float *out_gate,
                 int run_global) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!stream_ids || !params) throw std::runtime_error("stream_ids and params are required");
        mossgpu::SampleParamsC p{params->greedy,           params->temperature, params->top_k,
                                 params->top_p,            params->repetition_penalty, params->end_greedy,
                                 params->min_frames,       params->greedy_frames};
        g.step(stream_ids, n, p, forced, out_codes, out_stop, out_logits, out_gate, run_global != 0);
    });
}

int mossgpu_step_frames(mossgpu_engine *e, const int32_t *stream_ids, int n, const mossgpu_sample_params *params,
                        int n_frames, int32_t *out_codes, int32_t *out_frames_done) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!stream_ids || !params) throw std::runtime_error("stream_ids and params are required");
        mossgpu::SampleParamsC p{params->greedy,           params->temperature, params->top_k,
                                 params->top_p,            params->repetition_penalty, params->end_greedy,
                                 params->min_frames,       params->greedy_frames};
        g.step_frames(stream_ids, n, p, n_frames, out_codes, out_frames_done);
    });
}

int mossgpu_global_step_embed(mossgpu_engine *e, const int32_t *stream_ids, int n, const float *x, float *hidden_out) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!stream_ids || !x) throw std::runtime_error("stream_ids and x are required");
        g.global_step_embed(stream_ids, n, x, hidden_out);
    });
}

int mossgpu_set_state(mossgpu_engine *e, int stream_id, const float *k, const float *v, int n_pos,
                      const float *hidden) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!k || !v) throw std::runtime_error("k and v are required");
        g.set_state(stream_id, k, v, n_pos, hidden);
    });
}

int mossgpu_get_kv(mossgpu_engine *e, int stream_id, int layer, int p0, int n, float *k, float *v) {
    return guarded(e, [&](mossgpu::Engine &g) { g.get_kv(stream_id, layer, p0, n, k, v); });
}

int mossgpu_get_hidden(mossgpu_engine *e, int stream_id, float *hidden) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!hidden) throw std::runtime_error("hidden is NULL");
        g.get_hidden(stream_id, hidden);
    });
}

int mossgpu_debug_matrix_bytes(mossgpu_engine *e, const char *name, uint8_t *out, size_t out_bytes) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!name || !out) throw std::runtime_error("name and out are required");
        g.debug_matrix_bytes(name, out, out_bytes);
    });
}

int mossgpu_last_launch_count(mossgpu_engine *e) { return (e && e->eng) ? e->eng->last_launches() : -1; }

int mossgpu_fill_state_random(mossgpu_engine *e, int stream_id, int n_pos, uint64_t seed) {
    return guarded(e, [&](mossgpu::Engine &g) { g.fill_state_random(stream_id, n_pos, seed); });
}

int mossgpu_set_graphs(mossgpu_engine *e, int enable) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_use_graphs(enable != 0); });
}

int mossgpu_debug_inject_wait_timeout(mossgpu_engine *e, int enable) {
    return guarded(e, [&](mossgpu::Engine &g) { g.debug_inject_wait_timeout(enable != 0); });
}

int mossgpu_set_local_path(mossgpu_engine *e, int mode) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_local_path(mode); });
}

int mossgpu_set_small_layers(mossgpu_engine *e, int mode) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_small_layers(mode); });
}

int mossgpu_debug_small_layer_stamps(mossgpu_engine *e, unsigned long long *out, size_t n) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!out) throw std::runtime_error("out is required");
        g.small_layer_stamps(out, n);
    });
}

int mossgpu_set_gemm_path(mossgpu_engine *e, int mode) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_gemm_path(mode); });
}

int mossgpu_debug_matrix_tile_bytes(mossgpu_engine *e, const char *name, uint8_t *out, size_t out_bytes) {
    return guarded(e, [&](mossgpu::Engine &g) {
        if (!name || !out) throw std::runtime_error("name and out are required");
        g.debug_matrix_tile_bytes(name, out, out_bytes);
    });
}

int mossgpu_kernel_profile(mossgpu_engine *e, int enable) {
    return guarded(e, [&](mossgpu::Engine &g) { g.set_kernel_timing(enable != 0); });
}

int mossgpu_kernel_profile_read(mossgpu_engine *e, float *total_ms, int *launches, int max_kinds, int *n_kinds) {
    return guarded(e, [&](mossgpu::Engine &g) { g.read_kernel_timing(total_ms, launches, max_kinds, n_kinds); });
}

const char *mossgpu_kernel_name(int kind) { return mossgpu::kernel_kind_name(kind); }

}  // extern "C"
