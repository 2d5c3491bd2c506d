// engine.h -- the B200 engine behind include/mossgpu.h.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <array>
#include <string>
#include <unordered_map>
#include <vector>

#include "types.h"

namespace mossgpu {

struct SampleParamsC {
    int greedy;
    float temperature;
    int top_k;
    float top_p;
    float repetition_penalty;
    int end_greedy;
    int min_frames;
    int greedy_frames;
};

struct DevMat {
    int8_t *qs = nullptr;   // GEMV planes: [rows/4][cols/32][4][32] int8
    __half *sc = nullptr;   //              [rows/4][cols/32][4] fp16
    int8_t *qt = nullptr;   // tensor-core tiles: [rows/128][cols/64][128][64] int8 (swizzled pieces)
    __half *st = nullptr;   //                    [rows/128][cols/64][128][2] fp16
    int8_t *qm = nullptr;   // MMA fragment records (local layer, audio heads): [rows/16][cols/32][512] int8
    __half *sm = nullptr;   //                                                  [rows/16][cols/32][16] fp16
    int rows = 0, cols = 0;
};

struct Layer {
    DevMat attn, proj, fc_in, fc_out;
    float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
    float *attn_b = nullptr, *proj_b = nullptr, *fc_in_b = nullptr, *fc_out_b = nullptr;
};

// Kernel classes reported by the per-kernel timing (mossgpu_kernel_profile_read).
enum KernelKind {
    KK_PAGES, KK_GATHER, KK_LOOKUP, KK_EMBED, KK_PLAN,
    KK_QKV_G, KK_ATTN_DECODE, KK_PROJ_G, KK_FCIN_G, KK_FCOUT_G, KK_LNF,
    KK_QKV_L, KK_ATTN_LOCAL, KK_PROJ_L, KK_FCIN_L, KK_FCOUT_L, KK_GATE, KK_HEADS, KK_SAMPLE, KK_COMMIT,
    KK_BIMG, KK_ATTN_COMBINE, KK_ATTN_PREFILL, KK_QKV_ROPE, KK_LOCAL_FUSED, KK_SMALL_ATTN, KK_SMALL_MLP,
    KK_COUNT
};
const char *kernel_kind_name(int kind);

// One captured launch sequence (a frame, or a global step) for a fixed row count.
struct CapturedGraph {
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    std::vector<cudaEvent_t> events;  // timed graphs: one before the first kernel, one after each
    std::vector<int> kinds;
};

class Engine {
public:
    static constexpr int kPrefillRows = 256;    // rows per prefill pass unless max_rows says otherwise
    static constexpr int kMaxRowsLimit = 16384;
    static constexpr int kAttnGrid = 148;       // decode-attention CTAs: one per SM (205 KB smem each)
    static constexpr int kAttnItems = kAttnGrid * 8 * kHeads;  // split-K partials: ~8 chunks per CTA

    // max_rows: rows of one pass through the layers (a prefill pass over one or several
    // streams, or a decode batch); 0 = max(max_streams, kPrefillRows)
    Engine(const std::string &weights_path, int device, int max_streams, int max_ctx, int kv_pages, int max_rows = 0);
    ~Engine();
    Engine(const Engine &) = delete;
    Engine &operator=(const Engine &) = delete;

    int open_stream();
    int fork_stream(int src, int n_pos);
    void close_stream(int sid);
    void reset_stream(int sid);
    int position(int sid) const;
    void prefill(int sid, const int32_t *rows, int m, int start);
    void prefill_embeds(int sid, const float *x, int m, int start);
    // Several streams' prompts in shared passes of up to max_rows rows: stream sids[i] gets
    // m[i] rows at positions start[i].., its rows taken in order from rows ([.][17]) or x
    // ([.][768]), stream after stream.
    void prefill_batch(int n, const int32_t *sids, const int32_t *m, const int32_t *start, const int32_t *rows,
                       const float *x);
    void generate_begin(int sid, uint64_t seed);
    void step(const int32_t *sids, int n, const SampleParamsC &p, const int32_t *forced, int32_t *out_codes,
              uint8_t *out_stop, float *out_logits, float *out_gate, bool run_global);
    static constexpr int kMaxFramesPerCall = 1024;
    void step_frames(const int32_t *sids, int n, const SampleParamsC &p, int n_frames, int32_t *out_codes,
                     int32_t *out_frames_done);
    void global_step_embed(const int32_t *sids, int n, const float *x, float *hidden_out);
    void set_state(int sid, const float *k, const float *v, int n_pos, const float *hidden);
    void get_kv(int sid, int layer, int p0, int n, float *k, float *v);
    void get_hidden(int sid, float *out);
    void debug_matrix_bytes(const std::string &name, uint8_t *out, size_t out_bytes);
    void debug_matrix_tile_bytes(const std::string &name, uint8_t *out, size_t out_bytes);
    // Fault injection for the time-out test: while on, the first global layer's split-K decode
    // attention leaves one ring stage unfilled, so its bounded wait runs out (code 7).
    void debug_inject_wait_timeout(bool on);
    // Local decoder: 0 = the fused cluster kernel for greedy frames, 1 = the chain of per-step
    // kernels for every frame (default: measured as fast at 64 streams and faster above).
    void set_local_path(int mode);
    int local_cluster() const { return lf_cluster_; }
    // Global layers of decode batches of at most kGemvMaxRows rows: 1 = two launches per layer
    // (layer_small.cuh, the default), 0 = the five CUDA-core GEMV / attention launches.
    void set_small_layers(int mode);
    // Phase stamps of the last small-layer step (builds with -DMOSSGPU_PHASE_STAMPS): copies
    // [24 launches][96 CTAs][12 phases] %globaltimer values into out; throws in other builds.
    void small_layer_stamps(unsigned long long *out, size_t n);
    void set_cuda_stream(void *s);
    void fill_state_random(int sid, int n_pos, uint64_t seed);
    void set_kernel_timing(bool on);
    void read_kernel_timing(float *total_ms, int *launches, int max_kinds, int *n_kinds) const;
    void set_use_graphs(bool on) { use_graphs_ = on; }
    // 0 = automatic (tensor cores above kGemvMaxRows rows), 1 = CUDA-core GEMV, 2 = tensor cores
    void set_gemm_path(int mode);
    static constexpr int kGemvMaxRows = 8;
    // decode batches up to this many rows on the tensor-core path also use k_attn_rows (one
    // launch per layer; measured faster than plan + split-K decode + combine at 32 and 64 rows,
    // slower at 256, where the split-K kernel's page ring keeps HBM busier)
    static constexpr int kAttnRowsMaxTc = 96;
    int max_rows() const { return r_max_; }
    // tensor-core GEMM form: batches of at least direct_min_rows padded rows run one CTA per
    // (weight tile, slice of <= direct_rows rows) with no split-K (0 = never)
    void set_tc_policy(int direct_min_rows, int direct_rows);
    int last_launches() const { return launches_; }
    uint64_t weights_fingerprint() const { return weights_fp_; }
    int device() const { return device_; }

private:
    struct Slot {
        bool open = false;
        int pos = 0;
        int frame = 0;
        uint64_t seed = 0;
        std::vector<int> pages;
    };

    void load_weights(const std::string &path);
    void allocate_state();
    void set_smem_limits();
    QMat qm(const DevMat &m) const;
    EmbedTables tables() const;
    void block(const Layer &L, int li, bool local, int R, const int *row_slot, const int *row_pos, int lpos, float *x);
    bool use_tc(int R) const;
    void block_tc(const Layer &L, int li, bool local, int R, const int *row_slot, const int *row_pos, int lpos, float *x);
    void block_small(const Layer &L, int li, int R, const int *row_slot, const int *row_pos);
    void heads_tc(int ch, int R);
    void check_device_error();
    void drop_graphs();
    void global_layers(int R, const int *row_slot, const int *row_pos);
    void issue_frame(int R, bool run_global);
    void issue_global_embed(int R);
    // Launch the sequence `issue` for key: replay its CUDA graph (captured on first use), or
    // launch it directly when graphs are off.
    template <class F>
    void run_captured(uint64_t key, F &&issue);
    void mark(int kind);
    void accumulate_timing();
    void check_slot(int sid) const;
    void ensure_pages(int sid, int from_pos, int upto_pos, std::vector<int> &updates);
    int alloc_page();
    void copy_page(int dst, int src);
    void release_pages(Slot &s);
    void upload_page_updates(const std::vector<int> &updates);
    // flash-prefill work list of one pass (rows' slots and positions on the host)
    void plan_prefill_attention(int R, const int *slot, const int *pos);

    // control-block layout (ints) for R = r_max_ rows
    int off_slot() const { return 0; }
    int off_pos() const { return r_max_; }
    int off_frame() const { return 2 * r_max_; }
    int off_forced() const { return 3 * r_max_; }
    int off_pages() const { return 19 * r_max_; }  // [count][slot, index, page] x r_max_
    int off_fctl() const { return 22 * r_max_ + 1; }   // FrameCtl (kFrameCtlInts reserved)
    int off_active_in() const { return off_fctl() + kFrameCtlInts; }
    int off_fslot() const { return off_active_in() + r_max_; }  // frames committed in this call

    int device_ = 0;
    int max_streams_ = 0, max_ctx_ = 0, pages_per_stream_ = 0, n_pages_ = 0, r_max_ = 0;
    int tc_direct_min_rows_ = 256, tc_direct_rows_ = 0;  // 0: slice rows by batch size
    // flash-prefill tiles of the current pass (int4 each) on the device, with a pinned staging
    // copy; active while a prefill pass runs on the tensor-core path
    int4 *pf_items_ = nullptr;
    int4 *h_pf_items_ = nullptr;
    bool pf_active_ = false;
    int pf_tc_items_ = 0;
    // a direct-form fc_out stored its output here; the next layer's LN1 kernel adds it to x
    const float *pending_resid_ = nullptr;
    int pending_parts_ = 1;
    bool ln1_prebuilt_ = false;  // the next local block's LN1 image was written by k_sample
    // direct-form proj / fc_out split K in kTcKParts parts (their 768-row GEMMs have 96 tiles
    // for 148 SMs) and store the parts part_stride() floats apart in mlp_ ([R][3072] floats)
    static constexpr int kTcKParts = 3;
    size_t part_stride() const { return size_t(r_max_) * kHidden; }
    // a global step that starts without the plan kernel launches its first kernel plainly
    bool plain_first_ = false;
    cudaStream_t stream_ = nullptr, own_stream_ = nullptr;
    std::vector<void *> owned_, pinned_;
    size_t weights_bytes_ = 0;
    uint64_t weights_fp_ = 0;

    std::array<Layer, kLayers> global_{};
    Layer local_{};
    float *lnf_w_ = nullptr, *lnf_b_ = nullptr, *llnf_w_ = nullptr, *llnf_b_ = nullptr;
    DevMat wte_{};
    std::array<DevMat, kNVq> aemb_{};
    std::unordered_map<std::string, DevMat> mats_;

    // persistent per-stream state
    __half *kv_ = nullptr;
    int *page_table_ = nullptr;
    float *hidden_ = nullptr, *lkv_ = nullptr;
    uint16_t *counts_ = nullptr;
    uint32_t *rng_ = nullptr;  // [slot][4] xoshiro128** state of the stream's generate() call
    float2 *rope_ = nullptr;
    // row-batch scratch
    float *x_ = nullptr, *lx_ = nullptr, *q_ = nullptr, *attn_ = nullptr, *mlp_ = nullptr, *logits_ = nullptr;
    int *plan_ = nullptr, *work_ = nullptr, *active_ = nullptr, *codes_ = nullptr, *used_ = nullptr;
    float *part_ = nullptr, *gate_ = nullptr;
    int4 *desc_ = nullptr;  // decode-attention chunk descriptors
    int attn_items_ = 0;    // split-K partial capacity (chunks x heads)
    int *rows17_ = nullptr;
    int *codes_hist_ = nullptr;  // [kMaxFramesPerCall][max_streams][16] codes of a multi-frame call
    uint8_t *bimg_a_ = nullptr;    // activation image, K = 768, up to 256 rows
    uint8_t *bimg_mlp_ = nullptr;  // activation image, K = 3072 (fc_in output -> fc_out input)
    int *dev_err_ = nullptr;       // [0]: kernels' time-out flag; [1]: fault-injection word
    float *h_x_ = nullptr;         // pinned staging of global_step_embed's input rows
    int *h_err_ = nullptr;         // pinned host copy of it
    int gemm_path_ = 0;
    // small-batch layers: the three int64 residual accumulators D ([3][kGemvMaxRows][768]);
    // lnf_xfix_ is the one the ln_f after the layers reads its rows from (null on the other
    // paths, whose rows are in x_)
    int small_layers_ = 1;
    int attn_rows_max_ = kAttnRowsMaxTc;  // MOSSGPU_ATTN_ROWS_MAX overrides it (measurement)
    bool in_prefill_ = false;
    long long *sd_ = nullptr;
    const long long *lnf_xfix_ = nullptr;
    int local_path_ = 1;     // set_local_path (the fused kernel is opt-in)
    int lf_cluster_ = 0;     // CTAs per cluster of the fused local decoder (16 or 8; 0 = unavailable)
    bool frame_fused_ = false;  // the frame being issued runs the fused local decoder
    void launch_local_fused(int R, int step0, int step1);
    bool fused_ok(const SampleParamsC &p) const {
        return local_path_ == 0 && lf_cluster_ > 0 && (p.greedy != 0 || p.top_k == 1);
    }
    int *d_ctl_ = nullptr, *h_ctl_ = nullptr;
    int ctl_ints_ = 0;
    uint8_t *h_out_ = nullptr;

    std::vector<Slot> slots_;
    std::vector<int> free_pages_;
    std::vector<int> page_ref_;  // streams using each KV page (prefix sharing)
    int launches_ = 0;

    // CUDA graphs, programmatic dependent launch and per-kernel timing
    bool use_graphs_ = true;
    bool pdl_ = true;  // MOSSGPU_PDL=0 in the environment turns it off (A/B measurements)
    bool timing_ = false;
    std::unordered_map<uint64_t, CapturedGraph> graphs_;
    CapturedGraph *capturing_ = nullptr;
    CapturedGraph *last_graph_ = nullptr;
    double prof_ms_[KK_COUNT] = {};
    int prof_n_[KK_COUNT] = {};
};

}  // namespace mossgpu
