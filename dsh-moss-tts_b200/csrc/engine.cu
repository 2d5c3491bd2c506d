// engine.cu -- host side of the B200 engine: .moss upload + repack, the paged KV cache,
// stream slots, and the launch sequences of one frame (local decoder, gate, codes, global
// step) and of a prefill.  Exposed through the C ABI in capi.cpp (include/mossgpu.h).
#include "engine.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels.cuh"
#include "gemm_tc.cuh"
#include "attn_tc.cuh"
#include "local_fused.cuh"
#include "layer_small.cuh"

namespace mossgpu {

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            throw std::runtime_error(std::string(#call) + ": " + cudaGetErrorString(e_));          \
    } while (0)

namespace {

template <class T>
T *dalloc(size_t n, std::vector<void *> &owned) {
    void *p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    owned.push_back(p);
    return static_cast<T *>(p);
}

struct Entry {
    int dtype = 0, rows = 0, cols = 0;
    uint64_t off = 0, nbytes = 0;
};

uint64_t fnv(uint64_t h, const void *data, size_t n) {
    const uint8_t *p = static_cast<const uint8_t *>(data);
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

}  // namespace

// ------------------------------------------------------------------ construction

Engine::Engine(const std::string &path, int device, int max_streams, int max_ctx, int kv_pages, int max_rows)
    : device_(device), max_streams_(max_streams), max_ctx_(max_ctx) {
    if (max_streams <= 0 || max_ctx <= 0) throw std::runtime_error("max_streams and max_ctx must be positive");
    if (max_rows < 0 || max_rows > kMaxRowsLimit)
        throw std::runtime_error("max_rows must be in 0.." + std::to_string(kMaxRowsLimit));
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&own_stream_, cudaStreamNonBlocking));
    stream_ = own_stream_;
    if (const char *v = std::getenv("MOSSGPU_PDL")) pdl_ = std::strcmp(v, "0") != 0;
    if (const char *v = std::getenv("MOSSGPU_ATTN_ROWS_MAX")) attn_rows_max_ = std::atoi(v);
    load_weights(path);
    pages_per_stream_ = (max_ctx + kPage - 1) / kPage;
    n_pages_ = kv_pages > 0 ? kv_pages : max_streams * pages_per_stream_;
    r_max_ = std::max(max_streams, max_rows > 0 ? max_rows : kPrefillRows);
    allocate_state();
}

Engine::~Engine() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (auto &kv : graphs_) {
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
        for (cudaEvent_t ev : kv.second.events) cudaEventDestroy(ev);
    }
    for (void *p : owned_) cudaFree(p);
    for (void *p : pinned_) cudaFreeHost(p);
    if (own_stream_) cudaStreamDestroy(own_stream_);
}

void Engine::load_weights(const std::string &path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open weights: " + path);
    const std::streamsize size = f.tellg();
    if (size <= 16) throw std::runtime_error("weights file too small: " + path);
    std::vector<uint8_t> file(static_cast<size_t>(size));
    f.seekg(0);
    if (!f.read(reinterpret_cast<char *>(file.data()), size)) throw std::runtime_error("short read: " + path);
    // llm.cpp:426-439: weights fingerprint = FNV-1a over the file size and the first 4 KB
    const int64_t sz = size;
    weights_fp_ = fnv(fnv(1469598103934665603ull, &sz, sizeof(sz)), file.data(), std::min<size_t>(4096, file.size()));
    // weights.cpp:27-126: header, 80-byte entries, payload bounds
    if (std::memcmp(file.data(), "MOSW", 4) != 0) throw std::runtime_error("bad magic (not a .moss file)");
    uint32_t version = 0, n_tensors = 0;
    std::memcpy(&version, file.data() + 4, 4);
    std::memcpy(&n_tensors, file.data() + 8, 4);
    if (version != 1) throw std::runtime_error("unsupported .moss version " + std::to_string(version));
    if (16 + size_t(n_tensors) * 80 > file.size()) throw std::runtime_error("tensor table out of bounds");
    std::unordered_map<std::string, Entry> ents;
    for (uint32_t i = 0; i < n_tensors; ++i) {
        const uint8_t *b = file.data() + 16 + size_t(i) * 80;
        std::string name(reinterpret_cast<const char *>(b), strnlen(reinterpret_cast<const char *>(b), 48));
        Entry e;
        e.dtype = b[48];
        uint32_t dims[3];
        std::memcpy(dims, b + 52, 12);
        std::memcpy(&e.off, b + 64, 8);
        std::memcpy(&e.nbytes, b + 72, 8);
        if (e.off + e.nbytes > file.size()) throw std::runtime_error("tensor out of bounds: " + name);
        e.rows = int(dims[0]);
        e.cols = int(dims[1]);
        ents[name] = e;
    }
    uint8_t *staging = nullptr;
    CK(cudaMalloc(&staging, file.size()));
    CK(cudaMemcpy(staging, file.data(), file.size(), cudaMemcpyHostToDevice));

    auto mat = [&](const std::string &name, int rows, int cols) -> DevMat {
        auto it = ents.find(name);
        if (it == ents.end()) throw std::runtime_error("missing matrix: " + name);
        const Entry &e = it->second;
        if (e.dtype != 4 || e.rows != rows || e.cols != cols || e.nbytes != uint64_t(rows / 4) * (cols / 32) * 136)
            throw std::runtime_error("matrix is not q8_0_4x4 [" + std::to_string(rows) + "x" + std::to_string(cols) +
                                     "]: " + name);
        DevMat m;
        m.rows = rows;
        m.cols = cols;
        const long long nblocks = (long long)(rows / 4) * (cols / 32);
        m.qs = dalloc<int8_t>(size_t(nblocks) * 128, owned_);
        m.sc = dalloc<__half>(size_t(nblocks) * 4, owned_);
        const long long words = nblocks * 17;
        k_repack_q8x4<<<unsigned((words + 255) / 256), 256>>>(staging + e.off, m.qs, m.sc, nblocks);
        CK(cudaGetLastError());
        if (rows % kTcM == 0 && cols % kTcK == 0) {  // every matrix of this model qualifies
            m.qt = dalloc<int8_t>(size_t(rows) * cols, owned_);
            m.st = dalloc<__half>(size_t(rows) * (cols / 32), owned_);
            const long long items = (long long)rows * (cols / 32);
            k_repack_tiles<<<unsigned((items + 255) / 256), 256>>>(staging + e.off, rows, cols, m.qt, m.st);
            CK(cudaGetLastError());
        }
        mats_[name] = m;
        return m;
    };
    std::vector<std::pair<std::string, int>> vec_list;
    auto vec = [&](const std::string &name, int n) -> float * {
        auto it = ents.find(name);
        if (it == ents.end()) throw std::runtime_error("missing vector: " + name);
        const Entry &e = it->second;
        if (e.dtype != 3 || e.rows * e.cols != n || e.nbytes != uint64_t(n) * 4)
            throw std::runtime_error("vector is not f32[" + std::to_string(n) + "]: " + name);
        float *d = dalloc<float>(n, owned_);
        CK(cudaMemcpy(d, staging + e.off, size_t(n) * 4, cudaMemcpyDeviceToDevice));
        return d;
    };
    auto layer = [&](const std::string &p) {
        Layer L;
        L.ln1_w = vec(p + "ln1.w", kHidden);
        L.ln1_b = vec(p + "ln1.b", kHidden);
        L.ln2_w = vec(p + "ln2.w", kHidden);
        L.ln2_b = vec(p + "ln2.b", kHidden);
        L.attn = mat(p + "attn.w", kQKV, kHidden);
        L.attn_b = vec(p + "attn.b", kQKV);
        L.proj = mat(p + "proj.w", kHidden, kHidden);
        L.proj_b = vec(p + "proj.b", kHidden);
        L.fc_in = mat(p + "fc_in.w", kFF, kHidden);
        L.fc_in_b = vec(p + "fc_in.b", kFF);
        L.fc_out = mat(p + "fc_out.w", kHidden, kFF);
        L.fc_out_b = vec(p + "fc_out.b", kHidden);
        return L;
    };
    for (int i = 0; i < kLayers; ++i) global_[i] = layer("g" + std::to_string(i) + ".");
    local_ = layer("local.");
    lnf_w_ = vec("lnf.w", kHidden);
    lnf_b_ = vec("lnf.b", kHidden);
    llnf_w_ = vec("local.lnf.w", kHidden);
    llnf_b_ = vec("local.lnf.b", kHidden);
    wte_ = mat("wte", kVocab, kHidden);
    for (int ch = 0; ch < kNVq; ++ch) aemb_[ch] = mat("aemb." + std::to_string(ch), kCodebook, kHidden);
    // the fused local decoder reads the local layer and the audio heads, the small-batch global
    // layers (layer_small.cuh) every global matrix, as MMA fragment records
    auto mma_copy = [&](DevMat &m) {
        const long long threads = (long long)(m.rows / 16) * (m.cols / 32) * 32;
        m.qm = dalloc<int8_t>(size_t(m.rows) * m.cols, owned_);
        m.sm = dalloc<__half>(size_t(m.rows) * (m.cols / 32), owned_);
        k_repack_mma<<<unsigned((threads + 255) / 256), 256>>>(m.qs, m.sc, m.rows, m.cols, m.qm, m.sm);
        CK(cudaGetLastError());
    };
    for (DevMat *m : {&local_.attn, &local_.proj, &local_.fc_in, &local_.fc_out}) mma_copy(*m);
    for (Layer &L : global_)
        for (DevMat *m : {&L.attn, &L.proj, &L.fc_in, &L.fc_out}) mma_copy(*m);
    for (int ch = 0; ch < kNVq; ++ch) mma_copy(aemb_[ch]);
    CK(cudaDeviceSynchronize());
    CK(cudaFree(staging));
    weights_bytes_ = file.size();
}

void Engine::allocate_state() {
    kv_ = dalloc<__half>(size_t(kLayers) * n_pages_ * kPageHalfs, owned_);
    page_table_ = dalloc<int>(size_t(max_streams_) * pages_per_stream_, owned_);
    CK(cudaMemset(page_table_, 0, size_t(max_streams_) * pages_per_stream_ * sizeof(int)));
    hidden_ = dalloc<float>(size_t(max_streams_) * kHidden, owned_);
    CK(cudaMemset(hidden_, 0, size_t(max_streams_) * kHidden * sizeof(float)));
    lkv_ = dalloc<float>(size_t(max_streams_) * 2 * kLocalLen * kHidden, owned_);
    counts_ = dalloc<uint16_t>(size_t(max_streams_) * kNVq * kCodebook, owned_);
    CK(cudaMemset(counts_, 0, size_t(max_streams_) * kNVq * kCodebook * sizeof(uint16_t)));
    rng_ = dalloc<uint32_t>(size_t(max_streams_) * 4, owned_);
    CK(cudaMemset(rng_, 0, size_t(max_streams_) * 4 * sizeof(uint32_t)));

    const size_t R = size_t(r_max_);
    x_ = dalloc<float>(R * kHidden, owned_);
    lx_ = dalloc<float>(R * kHidden, owned_);
    q_ = dalloc<float>(R * kHidden, owned_);
    attn_ = dalloc<float>(R * kHidden, owned_);
    mlp_ = dalloc<float>(R * kFF, owned_);
    logits_ = dalloc<float>(size_t(max_streams_) * kNVq * kCodebook, owned_);
    plan_ = dalloc<int>(R + 3, owned_);
    // split-K capacity: ~8 chunks per CTA, and never less than one chunk per row
    attn_items_ = std::max(kAttnItems, r_max_ * kHeads);
    part_ = dalloc<float>(size_t(attn_items_) * kPartStride, owned_);
    desc_ = dalloc<int4>(attn_items_ / kHeads, owned_);
    work_ = dalloc<int>(kLayers, owned_);  // per-layer chunk counters of the decode attention
    // flash-prefill tiles: at most one per row
    pf_items_ = dalloc<int4>(size_t(r_max_), owned_);
    {
        void *hp = nullptr;
        CK(cudaMallocHost(&hp, size_t(r_max_) * sizeof(int4)));
        pinned_.push_back(hp);
        h_pf_items_ = static_cast<int4 *>(hp);
    }
    CK(cudaMemset(work_, 0, kLayers * sizeof(int)));
    active_ = dalloc<int>(R, owned_);
    codes_ = dalloc<int>(R * kNVq, owned_);
    used_ = dalloc<int>(R * kNVq, owned_);
    gate_ = dalloc<float>(R * 2, owned_);
    rows17_ = dalloc<int>(R * (kNVq + 1), owned_);
    codes_hist_ = dalloc<int>(size_t(kMaxFramesPerCall) * max_streams_ * kNVq, owned_);
    const size_t rows16 = (R + 15) / 16 * 16;  // padded batch rows of an activation image
    bimg_a_ = dalloc<uint8_t>(2 * size_t(kHidden) * rows16 * 2, owned_);  // hi and lo parts
    bimg_mlp_ = dalloc<uint8_t>(2 * size_t(kFF) * rows16 * 2, owned_);
    dev_err_ = dalloc<int>(4, owned_);
    CK(cudaMemset(dev_err_, 0, 4 * sizeof(int)));
    sd_ = dalloc<long long>(size_t(3) * kSlMaxRows * kHidden, owned_);
    CK(cudaMemset(sd_, 0, size_t(3) * kSlMaxRows * kHidden * sizeof(long long)));
    {
        void *he = nullptr;
        CK(cudaMallocHost(&he, 4 * sizeof(int)));
        pinned_.push_back(he);
        h_err_ = static_cast<int *>(he);
        *h_err_ = 0;
    }

    // control block: [slot R][pos R][frame R][forced 16R][page updates 1 + 3R][FrameCtl]
    ctl_ints_ = off_fslot() + 4;
    d_ctl_ = dalloc<int>(ctl_ints_, owned_);
    void *hp = nullptr;
    CK(cudaMallocHost(&hp, size_t(ctl_ints_) * sizeof(int)));
    pinned_.push_back(hp);
    h_ctl_ = static_cast<int *>(hp);
    std::memset(h_ctl_, 0, size_t(ctl_ints_) * sizeof(int));
    const size_t out_bytes = R * kNVq * 4 * 2 + R * 4 + R * 2 * 4 + size_t(max_streams_) * kNVq * kCodebook * 4 +
                             R * kHidden * 4;
    CK(cudaMallocHost(&hp, out_bytes));
    pinned_.push_back(hp);
    h_out_ = static_cast<uint8_t *>(hp);
    // pinned staging of a global step's input rows, so that their copy is asynchronous (a copy
    // from pageable memory would first wait for the stream's earlier work)
    CK(cudaMallocHost(&hp, R * kHidden * sizeof(float)));
    pinned_.push_back(hp);
    h_x_ = static_cast<float *>(hp);

    // RoPE table in double precision, cast to fp32 (llm.cpp:90-102)
    // rows for every global position and for the 17 local positions
    const int rope_rows = std::max(max_ctx_, kLocalLen);
    std::vector<float2> rope(size_t(rope_rows) * (kHeadDim / 2));
    for (int pos = 0; pos < rope_rows; ++pos)
        for (int i = 0; i < kHeadDim / 2; ++i) {
            const double inv = 1.0 / std::pow(10000.0, double(2 * i) / kHeadDim);
            const double ang = double(pos) * inv;
            rope[size_t(pos) * (kHeadDim / 2) + i] = make_float2(float(std::cos(ang)), float(std::sin(ang)));
        }
    rope_ = dalloc<float2>(rope.size(), owned_);
    CK(cudaMemcpy(rope_, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));

    slots_.assign(size_t(max_streams_), Slot{});
    free_pages_.clear();
    for (int p = n_pages_ - 1; p >= 0; --p) free_pages_.push_back(p);
    page_ref_.assign(size_t(n_pages_), 0);

    set_smem_limits();
    // the set-up copies and memsets above ran on the legacy stream; finish them before any
    // work is issued on the engine's (non-blocking) stream
    CK(cudaDeviceSynchronize());
}

namespace {

// Kernel launch with programmatic dependent launch (PDL) allowed: the kernel may begin while
// the previous kernel on the stream is still running, and orders itself with pdl_wait()
// (every kernel of the frame calls it before touching data an earlier kernel produced).
template <typename... KArgs, typename... Args>
void launch_kc(bool pdl, int cluster, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster > 0) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    CK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

template <typename... KArgs, typename... Args>
void launch_k(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
              Args &&...args) {
    launch_kc(pdl, 0, kernel, grid, block, smem, st, std::forward<Args>(args)...);
}

}  // namespace

// ------------------------------------------------------------------ GEMV launch

namespace {

struct GemvShape {
    int ks, gpc;
};

GemvShape shape_for(int cols) {
    // 2 chunks of 16 B per lane: K=768 -> 3 slices of 8 blocks, 2 groups per CTA (6 warps);
    // K=3072 -> 12 slices of 8 blocks, 1 group per CTA (12 warps)
    return cols == kFF ? GemvShape{12, 1} : GemvShape{3, 2};
}

template <int PRO, int EPI, int MAXR>
void set_attr() {
    CK(cudaFuncSetAttribute(k_gemv<PRO, EPI, MAXR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

template <int PRO, int EPI>
void set_attr_all() {
    set_attr<PRO, EPI, 1>();
    set_attr<PRO, EPI, 2>();
    set_attr<PRO, EPI, 4>();
    set_attr<PRO, EPI, 8>();
}

template <int PRO, int EPI, int MAXR>
void launch_gemv_r(const GemvArgs &a, cudaStream_t st, bool pdl) {
    const GemvShape s{a.ks, a.gpc};
    const int warps = s.ks * s.gpc;
    const int groups = a.w.rows / 4;
    dim3 grid((groups + s.gpc - 1) / s.gpc, (a.nrows + MAXR - 1) / MAXR);
    const size_t smem = (size_t(MAXR) * a.w.cols + size_t(warps) * 4 * MAXR + size_t(s.gpc) * 4 * MAXR) * sizeof(float);
    launch_k(pdl, k_gemv<PRO, EPI, MAXR>, grid, dim3(warps * 32), smem, st, a);
}

template <int PRO, int EPI>
void launch_gemv(GemvArgs a, cudaStream_t st, bool pdl) {
    const GemvShape s = shape_for(a.w.cols);
    a.ks = s.ks;
    a.gpc = s.gpc;
    if (a.nrows <= 1) launch_gemv_r<PRO, EPI, 1>(a, st, pdl);
    else if (a.nrows <= 2) launch_gemv_r<PRO, EPI, 2>(a, st, pdl);
    else if (a.nrows <= 4) launch_gemv_r<PRO, EPI, 4>(a, st, pdl);
    else launch_gemv_r<PRO, EPI, 8>(a, st, pdl);
}

// largest footprint over the batch slices a launch may use (16..64 rows split-K, 16..256
// direct, most stages)
template <int EPI>
void set_tc_attr() {
    int s1 = 0, s3 = 0, d1 = 0, d3 = 0;
    for (int n = 16; n <= kTcMaxNS; n += 16) {
        s1 = std::max(s1, tc_smem_bytes(n, TC_F16, tc_max_stages(n, TC_F16)));
        s3 = std::max(s3, tc_smem_bytes(n, TC_F16X3, tc_max_stages(n, TC_F16X3)));
    }
    for (int n = 16; n <= kTcMaxND; n += 16) {
        d1 = std::max(d1, tc_smem_bytes_direct(n, TC_F16, tc_max_stages_direct(n, TC_F16)));
        d3 = std::max(d3, tc_smem_bytes_direct(n, TC_F16X3, tc_max_stages_direct(n, TC_F16X3)));
    }
    CK(cudaFuncSetAttribute(k_gemm_tc<EPI, TC_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
    CK(cudaFuncSetAttribute(k_gemm_tc<EPI, TC_F16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    CK(cudaFuncSetAttribute(k_gemm_tc<EPI, TC_F16X3>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    CK(cudaFuncSetAttribute(k_gemm_tc<EPI, TC_F16X3>, cudaFuncAttributeMaxDynamicSharedMemorySize, s3));
    CK(cudaFuncSetAttribute(k_gemm_tp<EPI, TC_F16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, d1));
    CK(cudaFuncSetAttribute(k_gemm_tp<EPI, TC_F16X3, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, d3));
    int m1 = 0, m3 = 0;
    for (int n = 16; n <= 128; n += 16) {
        m1 = std::max(m1, tc_smem_bytes_atm(n, TC_F16, tc_max_stages_atm(n, TC_F16)));
        m3 = std::max(m3, tc_smem_bytes_atm(n, TC_F16X3, tc_max_stages_atm(n, TC_F16X3)));
    }
    CK(cudaFuncSetAttribute(k_gemm_tp<EPI, TC_F16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, m1));
    CK(cudaFuncSetAttribute(k_gemm_tp<EPI, TC_F16X3, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, m3));
}

}  // namespace

void Engine::set_smem_limits() {
    CK(cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    CK(cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kPtSmem));
    set_attr_all<PRO_LN, EPI_QKV>();
    set_attr_all<PRO_NONE, EPI_RESID>();
    set_attr_all<PRO_LN, EPI_GELU>();
    set_attr_all<PRO_LN, EPI_STORE>();
    set_tc_attr<TC_STORE>();
    set_tc_attr<TC_QKV>();
    set_tc_attr<TC_RESID>();
    set_tc_attr<TC_GELU_B>();
    // fused local decoder: 16-CTA clusters (a non-portable size) when the device can co-schedule
    // one, else 8
    CK(cudaFuncSetAttribute(k_small_attn<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlAttnSmem<1>::total));
    CK(cudaFuncSetAttribute(k_small_attn<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlAttnSmem<2>::total));
    CK(cudaFuncSetAttribute(k_small_attn<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlAttnSmem<4>::total));
    CK(cudaFuncSetAttribute(k_small_attn<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlAttnSmem<8>::total));
    CK(cudaFuncSetAttribute(k_small_mlp<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlMlpSmem<1>::total));
    CK(cudaFuncSetAttribute(k_small_mlp<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlMlpSmem<2>::total));
    CK(cudaFuncSetAttribute(k_small_mlp<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlMlpSmem<4>::total));
    CK(cudaFuncSetAttribute(k_small_mlp<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, SlMlpSmem<8>::total));
    // the SMs keep the full shared-memory split, so a launch's CTAs can be resident beside its
    // predecessor's (programmatic dependent launch) rather than wait for an SM to reconfigure
    for (const void *f : {(const void *)k_small_attn<1>, (const void *)k_small_attn<2>, (const void *)k_small_attn<4>,
                          (const void *)k_small_attn<8>, (const void *)k_small_mlp<1>, (const void *)k_small_mlp<2>,
                          (const void *)k_small_mlp<4>, (const void *)k_small_mlp<8>})
        CK(cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared));
    CK(cudaFuncSetAttribute(k_local_fused<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, LfSmem<16>::total));
    CK(cudaFuncSetAttribute(k_local_fused<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    CK(cudaFuncSetAttribute(k_local_fused<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, LfSmem<8>::total));
    lf_cluster_ = 0;
    int only = 0;  // MOSSGPU_LOCAL_CLUSTER=8 or 16 pins the cluster size (A/B measurements)
    if (const char *v = std::getenv("MOSSGPU_LOCAL_CLUSTER")) only = std::atoi(v);
    for (int C : {16, 8}) {
        if (only && C != only) continue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(C);
        cfg.blockDim = dim3(kLfThreads);
        cfg.dynamicSmemBytes = C == 16 ? LfSmem<16>::total : LfSmem<8>::total;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = C;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        const cudaError_t rc = C == 16 ? cudaOccupancyMaxActiveClusters(&n, k_local_fused<16>, &cfg)
                                       : cudaOccupancyMaxActiveClusters(&n, k_local_fused<8>, &cfg);
        if (rc == cudaSuccess && n > 0) {
            lf_cluster_ = C;
            break;
        }
        cudaGetLastError();  // a refused size is not an engine error
    }
}

void Engine::set_local_path(int mode) {
    if (mode < 0 || mode > 1) throw std::runtime_error("local path must be 0 (fused for greedy frames) or 1 (per-step kernels)");
    local_path_ = mode;
}

void Engine::launch_local_fused(int R, int step0, int step1) {
    const int *d_slot = d_ctl_ + off_slot();
    LfArgs a{};
    auto lm = [](const DevMat &m) { return LfMat{m.qm, m.sm, m.cols / 32}; };
    a.attn = lm(local_.attn);
    a.proj = lm(local_.proj);
    a.fc_in = lm(local_.fc_in);
    a.fc_out = lm(local_.fc_out);
    for (int ch = 0; ch < kNVq; ++ch) {
        a.head[ch] = lm(aemb_[ch]);
        a.aemb[ch] = qm(aemb_[ch]);
    }
    a.attn_b = local_.attn_b;
    a.proj_b = local_.proj_b;
    a.fc_in_b = local_.fc_in_b;
    a.fc_out_b = local_.fc_out_b;
    a.ln1_w = local_.ln1_w;
    a.ln1_b = local_.ln1_b;
    a.ln2_w = local_.ln2_w;
    a.ln2_b = local_.ln2_b;
    a.lnf_w = llnf_w_;
    a.lnf_b = llnf_b_;
    a.rope = rope_;
    a.wte = qm(wte_);
    a.hidden = hidden_;
    a.row_slot = d_slot;
    a.R = R;
    a.lkv = lkv_;
    a.qbuf = q_;
    a.lx_out = lx_;
    a.logits = logits_;
    a.counts = counts_;
    a.ctl = reinterpret_cast<const FrameCtl *>(d_ctl_ + off_fctl());
    a.forced = d_ctl_ + off_forced();
    a.active = active_;
    a.codes_out = codes_;
    a.used_out = used_;
    a.step0 = step0;
    a.step1 = step1;
    a.err = dev_err_;
    const int clusters = (R + kLfG - 1) / kLfG;
    if (lf_cluster_ == 16)
        launch_kc(pdl_, 16, k_local_fused<16>, dim3(clusters * 16), dim3(kLfThreads), LfSmem<16>::total, stream_, a);
    else
        launch_kc(pdl_, 8, k_local_fused<8>, dim3(clusters * 8), dim3(kLfThreads), LfSmem<8>::total, stream_, a);
    mark(KK_LOCAL_FUSED);
}

void Engine::set_small_layers(int mode) {
    if (mode < 0 || mode > 1) throw std::runtime_error("small layers must be 0 (five launches a layer) or 1 (two)");
    if (mode == small_layers_) return;
    small_layers_ = mode;
    drop_graphs();
}

// captured sequences hold the launch shapes of the policy they were captured under
void Engine::drop_graphs() {
    CK(cudaStreamSynchronize(stream_));
    for (auto &kv : graphs_) {
        if (kv.second.exec) CK(cudaGraphExecDestroy(kv.second.exec));
        for (cudaEvent_t ev : kv.second.events) CK(cudaEventDestroy(ev));
    }
    graphs_.clear();
    last_graph_ = nullptr;
}

void Engine::set_gemm_path(int mode) {
    if (mode < 0 || mode > 3)
        throw std::runtime_error("gemm path must be 0 (auto), 1 (CUDA cores), 2 (tensor cores, fp16x3) or 3 (tensor "
                                 "cores, fp16)");
    gemm_path_ = mode;
}

void Engine::set_tc_policy(int direct_min_rows, int direct_rows) {
    if (direct_min_rows < 0 || (direct_rows != 0 && (direct_rows < 16 || direct_rows > kTcMaxND || direct_rows % 16)))
        throw std::runtime_error("direct rows must be 0 (by batch size) or a multiple of 16 in 16..256");
    if (direct_min_rows == tc_direct_min_rows_ && direct_rows == tc_direct_rows_) return;
    tc_direct_min_rows_ = direct_min_rows;
    tc_direct_rows_ = direct_rows;
    drop_graphs();
}

bool Engine::use_tc(int R) const {
    if (gemm_path_ == 1) return false;
    return gemm_path_ >= 2 || R > kGemvMaxRows;
}

namespace {

// Decode batches (split-K form): grid = weight tiles x cluster CTAs x batch slices of <= 64
// rows.  At 64 rows a QKV GEMM has 18 weight tiles; clusters of 8 give it 144 CTAs streaming
// 1-2 K chunks each.  Batches of at least direct_min padded rows take the direct form instead:
// weight tiles x slices of <= direct_ns rows (x K parts), every K chunk of a part in one CTA.
// direct_ns = 0 sizes the slices by the batch: 256 rows from 1024 rows on (prefill passes);
// below that the smallest of 64 / 128 / 256 rows whose tiles fit one wave of the SMs, and the
// split-K form when even 64-row slices leave fewer than 96 tiles and the output is not stored
// in K parts (a 768-row matrix with a residual epilogue, the audio heads; QKV below 384 rows).
// Measured per GEMM on a 512-stream frame (one B200, ms per frame, split-K / 128-row / 64-row
// slices): global QKV 0.35 / 0.20 / 0.18, fc_in 0.55 / 0.26 / 0.35, local fc_out 0.51 / 0.81 /
// 0.78, audio heads 0.21 / 0.27 / 0.24; at 256 rows (split-K / 64-row): fc_in 0.39 / 0.29,
// local QKV 0.26 / 0.36.
template <int EPI>
void launch_tc(TcArgs a, int prec, cudaStream_t st, bool pdl, int direct_min, int direct_ns) {
    const int tiles = a.rows / kTcM, nchunks = a.K / kTcK;
    const int ks = (EPI == TC_STORE && a.ksplit > 1 && nchunks % a.ksplit == 0) ? a.ksplit : 1;
    bool direct = direct_min > 0 && a.N >= direct_min;
    int ns = 0;
    if (direct && direct_ns > 0) {
        ns = std::min(a.N, direct_ns);
    } else if (direct && a.N >= 1024) {
        ns = std::min(a.N, kTcMaxND);
    } else if (direct) {
        for (int cand : {64, 128, 256}) {
            ns = std::min(a.N, cand);
            if (tiles * ((a.N + ns - 1) / ns) * ks <= kNumSMs) break;
        }
        // a STORE in K parts stays direct: its consumer adds the parts, split-K writes one
        if (ks == 1 && tiles * ((a.N + 63) / 64) < 96) direct = false;
    }
    if (direct) {
        while (a.N % ns) ns -= 16;
        // the per-matrix choice keeps slices of >= 64 rows (a padded batch that 64 does not
        // divide, such as 304 rows, takes split-K), except for a STORE in K parts, whose
        // consumer adds the parts; an explicit direct_ns is taken as given
        if (direct_ns == 0 && a.N < 1024 && ns < 64 && ks == 1) direct = false;
    }
    if (direct) {
        a.nsub = ns;
        a.csize = 1;
        // tile-persistent: at most one CTA per SM walks the (weight tile, slice) tiles; slices
        // of <= 128 rows keep A in tensor memory beside the two accumulators
        a.ksplit = ks;
        const dim3 grid(std::min(tiles * (a.N / ns) * ks, kNumSMs));
        const bool atm = ns <= 128;
        a.stages = atm ? tc_max_stages_atm(ns, prec) : tc_max_stages_direct(ns, prec);
        const size_t smem = atm ? tc_smem_bytes_atm(ns, prec, a.stages) : tc_smem_bytes_direct(ns, prec, a.stages);
        if (prec == TC_F16X3)
            launch_kc(pdl, 0, atm ? k_gemm_tp<EPI, TC_F16X3, true> : k_gemm_tp<EPI, TC_F16X3, false>, grid,
                      dim3(kTpThreads), smem, st, a);
        else
            launch_kc(pdl, 0, atm ? k_gemm_tp<EPI, TC_F16, true> : k_gemm_tp<EPI, TC_F16, false>, grid, dim3(kTpThreads),
                      smem, st, a);
        return;
    }
    int nsub = std::min(a.N, kTcMaxNS);
    while (a.N % nsub) nsub -= 16;  // N is a multiple of 16
    const int nz = a.N / nsub;
    // split K over the largest cluster (<= 16) that keeps every CTA of the grid resident
    int C = kTcMaxCluster;
    while (C > 1 && (tiles * C * nz > 148 || C > nchunks)) C >>= 1;
    const int per = (nchunks + C - 1) / C;  // most chunks one CTA handles
    a.nsub = nsub;
    a.csize = C;
    a.stages = std::min(per, tc_max_stages(nsub, prec));
    const dim3 grid(tiles * C, 1, nz);
    if (prec == TC_F16X3)
        launch_kc(pdl, C, k_gemm_tc<EPI, TC_F16X3>, grid, dim3(kTcThreads), tc_smem_bytes(nsub, TC_F16X3, a.stages), st,
                  a);
    else
        launch_kc(pdl, C, k_gemm_tc<EPI, TC_F16>, grid, dim3(kTcThreads), tc_smem_bytes(nsub, TC_F16, a.stages), st, a);
}

}  // namespace

// The block of llm.cpp:230-246 on tensor cores (R > 8 rows): activation images built by
// k_build_bimg (LayerNorm fused), tcgen05 GEMMs with cluster split-K and fused epilogues.
void Engine::block_tc(const Layer &L, int li, bool local, int R, const int *row_slot, const int *row_pos, int lpos,
                      float *x) {
    const int N = (R + 15) / 16 * 16;
    const int prec = gemm_path_ == 3 ? TC_F16 : TC_F16X3;
    // GEMMs in the direct form (prefill passes) store plain outputs; the QKV epilogue (RoPE, KV
    // append) runs as its own pass and residual adds move into the next LayerNorm kernel, which
    // reads x anyway.  The last global layer's fc_out keeps its residual epilogue (ln_f reads x).
    const bool direct = !local && tc_direct_min_rows_ > 0 && N >= tc_direct_min_rows_;
    // From the direct-form batch size on, proj and fc_out store their outputs in K parts (more
    // tiles to fill the SMs) and the next activation-image builder adds them to x: LN2 for
    // proj; for fc_out the next layer's LN1, or in the local decoder the audio head's ln_f
    // (heads_tc).  Kept as a residual epilogue: the last global layer's fc_out (ln_f reads x)
    // and local step 0's (the end gate reads x).  The local decoder stores parts from twice the
    // direct-form batch on (measured per 512-stream frame: local proj + fc_out 0.51 against
    // 0.74 ms, the builders' adds 0.08 ms more; at 256 streams the frame was 1% slower).
    const bool parts = tc_direct_min_rows_ > 0 && N >= (local ? 2 : 1) * tc_direct_min_rows_;
    const float *add1 = pending_resid_;
    const int nadd1 = pending_parts_;
    pending_resid_ = nullptr;
    if (local && ln1_prebuilt_) {  // k_sample wrote this step's LN1 image with its input row
        if (add1) throw std::logic_error("local LN1 image prebuilt with a residual add pending");
        ln1_prebuilt_ = false;
    } else {
        launch_k(pdl_ && !(plain_first_ && li == 0 && !local), k_build_bimg, dim3((N + 7) / 8), dim3(256), 0, stream_,
                 x, kHidden, R, N, L.ln1_w, L.ln1_b, tc_parts(prec), bimg_a_, add1, nadd1, part_stride());
        if (!local && li == 0) plain_first_ = false;
        mark(KK_BIMG);
    }
    TcArgs a{};
    a.N = N;
    a.R = R;
    a.err = dev_err_;
    a.bimg = bimg_a_;
    a.qt = L.attn.qt;
    a.st = L.attn.st;
    a.rows = kQKV;
    a.K = kHidden;
    a.bias = L.attn_b;
    a.q_out = q_;
    a.row_slot = row_slot;
    a.row_pos = local ? nullptr : row_pos;
    a.fixed_pos = lpos;
    a.rope = rope_;
    if (local) {
        a.lkv = lkv_;
    } else {
        a.kv = kv_ + size_t(li) * n_pages_ * kPageHalfs;
        a.page_table = page_table_;
        a.pages_per_stream = pages_per_stream_;
    }
    if (direct) {
        a.out = mlp_;  // raw [R][2304], bias included
        a.ldo = kQKV;
        launch_tc<TC_STORE>(a, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
        mark(KK_QKV_G);
        launch_k(pdl_, k_qkv_rope, dim3(unsigned(R)), dim3(kQkvRopeThreads), 0, stream_, mlp_, R,
                 row_slot, row_pos, rope_, q_, a.kv, page_table_, pages_per_stream_);
        mark(KK_QKV_ROPE);
    } else {
        launch_tc<TC_QKV>(a, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
        mark(local ? KK_QKV_L : KK_QKV_G);
    }
    // attention writes straight into proj's activation image; its padding rows are still
    // zero from the LN1 image built above with the same N
    if (local) {
        const int warps = R * kHeads;
        launch_k(pdl_, k_attn_local, dim3((warps + 11) / 12), dim3(384), 0, stream_, q_, lkv_, row_slot, lpos, R,
                 attn_, bimg_a_, N, tc_parts(prec));
        mark(KK_ATTN_LOCAL);
    } else {
        AttnArgs t{};
        t.q = q_;
        t.kv = a.kv;
        t.page_table = page_table_;
        t.pages_per_stream = pages_per_stream_;
        t.row_slot = row_slot;
        t.row_pos = row_pos;
        t.plan = plan_;
        t.R = R;
        t.part = part_;
        t.desc = desc_;
        t.out = attn_;
        t.bimg = bimg_a_;
        t.bimg_N = N;
        t.bimg_parts = tc_parts(prec);
        t.work = work_ + li;
        t.err = dev_err_;
        t.inject = li == 0 ? dev_err_ + 1 : nullptr;
        if (pf_active_) {
            PtArgs f{};
            f.q = q_;
            f.kv = t.kv;
            f.page_table = page_table_;
            f.pages_per_stream = pages_per_stream_;
            f.items = pf_items_;
            f.bimg = bimg_a_;
            f.bimg_N = N;
            f.bimg_parts = tc_parts(prec);
            f.err = dev_err_;
            launch_k(pdl_, k_attn_prefill_tc, dim3(unsigned(pf_tc_items_), kHeads), dim3(kPtThreads), kPtSmem, stream_, f);
            mark(KK_ATTN_PREFILL);
        } else if (R <= attn_rows_max_) {
            launch_k(pdl_, k_attn_rows, dim3(R * kHeads), dim3(kArWarps * 32), 0, stream_, q_,
                     static_cast<const __half *>(t.kv), page_table_, pages_per_stream_, row_slot, row_pos, attn_,
                     bimg_a_, N, tc_parts(prec));
            mark(KK_ATTN_DECODE);
        } else {
            launch_k(pdl_, k_attn_decode, dim3(kAttnGrid), dim3(kAttnThreads), kAttnSmem, stream_, t);
            mark(KK_ATTN_DECODE);
            launch_k(pdl_, k_attn_combine, dim3((R * kHeads + 7) / 8), dim3(256), 0, stream_, t);
            mark(KK_ATTN_COMBINE);
        }
    }
    TcArgs p{};
    p.N = N;
    p.R = R;
    p.err = dev_err_;
    p.bimg = bimg_a_;
    p.qt = L.proj.qt;
    p.st = L.proj.st;
    p.rows = kHidden;
    p.K = kHidden;
    p.bias = L.proj_b;
    p.out = parts ? mlp_ : x;  // parts: kTcKParts K parts at mlp_ + part_stride() apart
    p.ldo = kHidden;
    p.ksplit = parts ? kTcKParts : 1;
    p.part_stride = part_stride();
    if (parts)
        launch_tc<TC_STORE>(p, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
    else
        launch_tc<TC_RESID>(p, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
    mark(local ? KK_PROJ_L : KK_PROJ_G);
    launch_k(pdl_, k_build_bimg, dim3((N + 7) / 8), dim3(256), 0, stream_, x, kHidden, R, N, L.ln2_w, L.ln2_b,
             tc_parts(prec), bimg_a_, parts ? static_cast<const float *>(mlp_) : nullptr, kTcKParts, part_stride());
    mark(KK_BIMG);
    TcArgs f{};
    f.N = N;
    f.R = R;
    f.err = dev_err_;
    f.bimg = bimg_a_;
    f.qt = L.fc_in.qt;
    f.st = L.fc_in.st;
    f.rows = kFF;
    f.K = kHidden;
    f.bias = L.fc_in_b;
    f.bimg_out = bimg_mlp_;
    launch_tc<TC_GELU_B>(f, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
    mark(local ? KK_FCIN_L : KK_FCIN_G);
    TcArgs o{};
    o.N = N;
    o.R = R;
    o.err = dev_err_;
    o.bimg = bimg_mlp_;
    o.qt = L.fc_out.qt;
    o.st = L.fc_out.st;
    o.rows = kHidden;
    o.K = kFF;
    o.bias = L.fc_out_b;
    o.ldo = kHidden;
    if (parts && (local ? lpos > 0 : li < kLayers - 1)) {  // the next builder adds the K parts to x
        o.out = mlp_;
        o.ksplit = kTcKParts;
        o.part_stride = part_stride();
        launch_tc<TC_STORE>(o, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
        pending_resid_ = mlp_;
        pending_parts_ = kTcKParts;
    } else {
        o.out = x;
        launch_tc<TC_RESID>(o, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
    }
    mark(local ? KK_FCOUT_L : KK_FCOUT_G);
}

// audio head ch on tensor cores: logits[r][ch] = aemb[ch] . LN(lx[r]) (llm.cpp:268-270)
void Engine::heads_tc(int ch, int R) {
    const int N = (R + 15) / 16 * 16;
    const int prec = gemm_path_ == 3 ? TC_F16 : TC_F16X3;
    // the local block's fc_out K parts, when it stored them, are added to lx_ here
    const float *add = pending_resid_;
    const int nadd = pending_parts_;
    pending_resid_ = nullptr;
    launch_k(pdl_, k_build_bimg, dim3((N + 7) / 8), dim3(256), 0, stream_, lx_, kHidden, R, N, llnf_w_, llnf_b_,
             tc_parts(prec), bimg_a_, add, add ? nadd : 0, part_stride());
    mark(KK_BIMG);
    TcArgs h{};
    h.N = N;
    h.R = R;
    h.err = dev_err_;
    h.bimg = bimg_a_;
    h.qt = aemb_[ch].qt;
    h.st = aemb_[ch].st;
    h.rows = kCodebook;
    h.K = kHidden;
    h.out = logits_ + size_t(ch) * kCodebook;
    h.ldo = kNVq * kCodebook;
    launch_tc<TC_STORE>(h, prec, stream_, pdl_, tc_direct_min_rows_, tc_direct_rows_);
    mark(KK_HEADS);
}

// A kernel that timed out on one of its barriers (tensor-core GEMM, decode attention) leaves
// a code in dev_err_.
// Callers enqueue the copy of the flag into h_err_ before their final synchronisation.
void Engine::check_device_error() {
    const int e = *h_err_;
    if (e != 0) {
        *h_err_ = 0;
        CK(cudaMemsetAsync(dev_err_, 0, sizeof(int), stream_));
        // a step cut short may leave a small-batch residual accumulator non-zero
        CK(cudaMemsetAsync(sd_, 0, size_t(3) * kSlMaxRows * kHidden * sizeof(long long), stream_));
        CK(cudaStreamSynchronize(stream_));
        const char *what = e == 7 || e == 8 ? "decode-attention page ring"
                           : (e >= 31 && e <= 33) ? "fused local decoder barrier"
                                                  : "tensor-core GEMM barrier";
        throw std::runtime_error(std::string(what) + " wait timed out (code " + std::to_string(e) + ")");
    }
}

QMat Engine::qm(const DevMat &m) const { return QMat{m.qs, m.sc, m.rows, m.cols}; }

EmbedTables Engine::tables() const {
    EmbedTables t;
    t.wte = qm(wte_);
    for (int ch = 0; ch < kNVq; ++ch) t.aemb[ch] = qm(aemb_[ch]);
    return t;
}

// ------------------------------------------------------------------ launch sequences

// One transformer block over the row batch (llm.cpp:230-246).  local=false: global layer
// `li` with the paged KV at row_pos; local=true: the local layer at local position lpos.
void Engine::block(const Layer &L, int li, bool local, int R, const int *row_slot, const int *row_pos, int lpos,
                   float *x) {
    if (use_tc(R)) {
        block_tc(L, li, local, R, row_slot, row_pos, lpos, x);
        return;
    }
    GemvArgs a{};
    a.nrows = R;
    // LN1 -> QKV + bias + RoPE + KV append
    a.w = qm(L.attn);
    a.bias = L.attn_b;
    a.x = x;
    a.ldx = kHidden;
    a.ln_w = L.ln1_w;
    a.ln_b = L.ln1_b;
    a.q_out = q_;
    a.row_slot = row_slot;
    a.row_pos = local ? nullptr : row_pos;
    a.fixed_pos = lpos;
    a.rope = rope_;
    if (local) {
        a.kv = nullptr;
        a.lkv = lkv_;
    } else {
        a.kv = kv_ + size_t(li) * n_pages_ * kPageHalfs;
        a.page_table = page_table_;
        a.pages_per_stream = pages_per_stream_;
    }
    // the first kernel of a global step without the plan kernel follows host-to-device copies
    launch_gemv<PRO_LN, EPI_QKV>(a, stream_, pdl_ && !(plain_first_ && li == 0 && !local));
    if (!local && li == 0) plain_first_ = false;
    mark(local ? KK_QKV_L : KK_QKV_G);
    // attention
    if (local) {
        const int warps = R * kHeads;
        launch_k(pdl_, k_attn_local, dim3((warps + 11) / 12), dim3(384), 0, stream_, q_, lkv_, row_slot, lpos, R,
                 attn_, static_cast<uint8_t *>(nullptr), 0, 0);
        mark(KK_ATTN_LOCAL);
    } else {
        AttnArgs t{};
        t.q = q_;
        t.kv = a.kv;
        t.page_table = page_table_;
        t.pages_per_stream = pages_per_stream_;
        t.row_slot = row_slot;
        t.row_pos = row_pos;
        t.plan = plan_;
        t.R = R;
        t.part = part_;
        t.desc = desc_;
        t.out = attn_;
        t.work = work_ + li;
        t.err = dev_err_;
        t.inject = li == 0 ? dev_err_ + 1 : nullptr;
        if (R <= kGemvMaxRows) {
            launch_k(pdl_, k_attn_rows, dim3(R * kHeads), dim3(kArWarps * 32), 0, stream_, q_,
                     static_cast<const __half *>(a.kv), page_table_, pages_per_stream_, row_slot, row_pos, attn_,
                     static_cast<uint8_t *>(nullptr), 0, 0);
            mark(KK_ATTN_DECODE);
        } else {
            launch_k(pdl_, k_attn_decode, dim3(kAttnGrid), dim3(kAttnThreads), kAttnSmem, stream_, t);
            mark(KK_ATTN_DECODE);
            launch_k(pdl_, k_attn_combine, dim3((R * kHeads + 7) / 8), dim3(256), 0, stream_, t);
            mark(KK_ATTN_COMBINE);
        }
    }
    // proj + residual
    GemvArgs p{};
    p.nrows = R;
    p.w = qm(L.proj);
    p.bias = L.proj_b;
    p.x = attn_;
    p.ldx = kHidden;
    p.out = x;
    p.ldo = kHidden;
    launch_gemv<PRO_NONE, EPI_RESID>(p, stream_, pdl_);
    mark(local ? KK_PROJ_L : KK_PROJ_G);
    // LN2 -> fc_in + gelu
    GemvArgs f{};
    f.nrows = R;
    f.w = qm(L.fc_in);
    f.bias = L.fc_in_b;
    f.x = x;
    f.ldx = kHidden;
    f.ln_w = L.ln2_w;
    f.ln_b = L.ln2_b;
    f.out = mlp_;
    f.ldo = kFF;
    launch_gemv<PRO_LN, EPI_GELU>(f, stream_, pdl_);
    mark(local ? KK_FCIN_L : KK_FCIN_G);
    // fc_out + residual
    GemvArgs o{};
    o.nrows = R;
    o.w = qm(L.fc_out);
    o.bias = L.fc_out_b;
    o.x = mlp_;
    o.ldx = kFF;
    o.out = x;
    o.ldo = kHidden;
    launch_gemv<PRO_NONE, EPI_RESID>(o, stream_, pdl_);
    mark(local ? KK_FCOUT_L : KK_FCOUT_G);
}

// 12 global layers over rows already embedded in x_ (row_pos = positions being written).
void Engine::global_layers(int R, const int *row_slot, const int *row_pos) {
    pending_resid_ = nullptr;
    lnf_xfix_ = nullptr;
    if (small_layers_ && !in_prefill_ && !use_tc(R) && R <= kSlMaxRows) {  // decode rows, one per stream
        plain_first_ = true;
        for (int li = 0; li < kLayers; ++li) block_small(global_[li], li, R, row_slot, row_pos);
        lnf_xfix_ = sd_;  // the layers' output is in D[0] after the 24 launches
        return;
    }
    if (pf_active_) {  // a prefill pass: the host-built flash-prefill plan is already on the device
        for (int li = 0; li < kLayers; ++li) block(global_[li], li, false, R, row_slot, row_pos, 0, x_);
        return;
    }
    if (use_tc(R) ? R <= attn_rows_max_ : R <= kGemvMaxRows) {  // every layer on k_attn_rows: no plan
        plain_first_ = true;
        for (int li = 0; li < kLayers; ++li) block(global_[li], li, false, R, row_slot, row_pos, 0, x_);
        return;
    }
    // ordinary launch: in a global step alone this kernel follows a host-to-device copy
    launch_k(false, k_attn_plan, dim3(1), dim3(kPlanThreads), 0, stream_, row_pos, row_slot, pages_per_stream_, R, attn_items_,
             plan_, desc_, work_, kLayers);
    mark(KK_PLAN);
    for (int li = 0; li < kLayers; ++li) block(global_[li], li, false, R, row_slot, row_pos, 0, x_);
}

// One global layer of a decode batch of R <= 8 rows (one row per stream) in two launches
// (layer_small.cuh): attention half (launch p = 2 li) and MLP half (p = 2 li + 1), the residual
// stream passed in the int64 accumulators D[p % 3] (launch 0 reads the embeddings in x_).
void Engine::block_small(const Layer &L, int li, int R, const int *row_slot, const int *row_pos) {
    long long *D[3];
    for (int i = 0; i < 3; ++i) D[i] = sd_ + size_t(i) * kSlMaxRows * kHidden;
    SmallArgs a{};
    auto lm = [](const DevMat &m) { return LfMat{m.qm, m.sm, m.cols / 32}; };
    a.attn = lm(L.attn);
    a.proj = lm(L.proj);
    a.fc_in = lm(L.fc_in);
    a.fc_out = lm(L.fc_out);
    a.attn_b = L.attn_b;
    a.proj_b = L.proj_b;
    a.fc_in_b = L.fc_in_b;
    a.fc_out_b = L.fc_out_b;
    a.kv = kv_ + size_t(li) * n_pages_ * kPageHalfs;
    a.page_table = page_table_;
    a.pages_per_stream = pages_per_stream_;
    a.row_slot = row_slot;
    a.row_pos = row_pos;
    a.rope = rope_;
    a.R = R;
    const int R2 = R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8;
    for (int half = 0; half < 2; ++half) {
        const int p = 2 * li + half;
        a.launch = p;
        a.ln_w = half ? L.ln2_w : L.ln1_w;
        a.ln_b = half ? L.ln2_b : L.ln1_b;
        a.x0 = x_;
        a.d_in = p == 0 ? nullptr : D[p % 3];
        a.d_out = D[(p + 1) % 3];
        a.d_zero = D[(p + 2) % 3];
        // the first launch of a step follows host-to-device copies or the embedding kernel
        const bool pdl = pdl_ && !(plain_first_ && p == 0);
        const dim3 grid(kSlCtas), block(kSlThreads);
        if (half == 0) {
            switch (R2) {
            case 1: launch_kc(pdl, kSlCluster, k_small_attn<1>, grid, block, SlAttnSmem<1>::total, stream_, a); break;
            case 2: launch_kc(pdl, kSlCluster, k_small_attn<2>, grid, block, SlAttnSmem<2>::total, stream_, a); break;
            case 4: launch_kc(pdl, kSlCluster, k_small_attn<4>, grid, block, SlAttnSmem<4>::total, stream_, a); break;
            default: launch_kc(pdl, kSlCluster, k_small_attn<8>, grid, block, SlAttnSmem<8>::total, stream_, a); break;
            }
            mark(KK_SMALL_ATTN);
        } else {
            switch (R2) {
            case 1: launch_kc(pdl, kSlCluster, k_small_mlp<1>, grid, block, SlMlpSmem<1>::total, stream_, a); break;
            case 2: launch_kc(pdl, kSlCluster, k_small_mlp<2>, grid, block, SlMlpSmem<2>::total, stream_, a); break;
            case 4: launch_kc(pdl, kSlCluster, k_small_mlp<4>, grid, block, SlMlpSmem<4>::total, stream_, a); break;
            default: launch_kc(pdl, kSlCluster, k_small_mlp<8>, grid, block, SlMlpSmem<8>::total, stream_, a); break;
            }
            mark(KK_SMALL_MLP);
        }
    }
    if (li == 0) plain_first_ = false;
}

void Engine::small_layer_stamps(unsigned long long *out, size_t n) {
#ifdef MOSSGPU_PHASE_STAMPS
    const size_t total = size_t(kSlStampLaunches) * kSlCtas * kSlStampPhases;
    if (n < total) throw std::runtime_error("phase stamps need " + std::to_string(total) + " entries");
    CK(cudaStreamSynchronize(stream_));
    CK(cudaMemcpyFromSymbol(out, g_sl_stamps, total * sizeof(unsigned long long)));
#else
    (void)out;
    (void)n;
    throw std::runtime_error("this library was built without phase stamps (-DMOSSGPU_PHASE_STAMPS)");
#endif
}

// ------------------------------------------------------------------ host helpers

void Engine::check_slot(int sid) const {
    if (sid < 0 || sid >= max_streams_ || !slots_[size_t(sid)].open)
        throw std::runtime_error("stream " + std::to_string(sid) + " is not open");
}

int Engine::alloc_page() {
    if (free_pages_.empty()) throw std::runtime_error("KV page pool exhausted");
    const int page = free_pages_.back();
    free_pages_.pop_back();
    page_ref_[size_t(page)] = 1;
    return page;
}

// All 12 layers of one page (48 KB each, n_pages_ pages apart): one strided device copy.
void Engine::copy_page(int dst, int src) {
    const size_t bytes = size_t(kPageHalfs) * sizeof(__half);
    const size_t pitch = size_t(n_pages_) * bytes;
    CK(cudaMemcpy2DAsync(kv_ + size_t(dst) * kPageHalfs, pitch, kv_ + size_t(src) * kPageHalfs, pitch, bytes, kLayers,
                         cudaMemcpyDeviceToDevice, stream_));
}

// Pages for positions from_pos..upto_pos of a stream that is about to write them: a page
// still shared with another stream (after mossgpu_stream_fork) is copied first, so a write
// never reaches another stream's KV; missing pages are allocated.
void Engine::ensure_pages(int sid, int from_pos, int upto_pos, std::vector<int> &updates) {
    Slot &s = slots_[size_t(sid)];
    const int need = upto_pos / kPage + 1;
    if (upto_pos >= max_ctx_) throw std::runtime_error("stream " + std::to_string(sid) + " reached max_ctx");
    for (int i = std::max(0, from_pos) / kPage; i < std::min(need, int(s.pages.size())); ++i) {
        const int old = s.pages[size_t(i)];
        if (page_ref_[size_t(old)] <= 1) continue;
        const int page = alloc_page();
        copy_page(page, old);
        --page_ref_[size_t(old)];
        s.pages[size_t(i)] = page;
        updates.push_back(sid);
        updates.push_back(i);
        updates.push_back(page);
    }
    while (int(s.pages.size()) < need) {
        const int page = alloc_page();
        updates.push_back(sid);
        updates.push_back(int(s.pages.size()));
        updates.push_back(page);
        s.pages.push_back(page);
    }
}

void Engine::release_pages(Slot &s) {
    for (int p : s.pages)
        if (--page_ref_[size_t(p)] == 0) free_pages_.push_back(p);
    s.pages.clear();
}

// A new stream whose first n_pos positions are those of src: the full pages are shared
// (reference-counted), the partly filled last page is copied, and the hidden state is
// src's.  Writes of either stream to a shared page go through ensure_pages' copy.
int Engine::fork_stream(int src, int n_pos) {
    check_slot(src);
    const Slot &s = slots_[size_t(src)];
    if (n_pos < 0 || n_pos > s.pos) throw std::runtime_error("fork length outside the source stream's positions");
    const int dst = open_stream();
    std::vector<int> upd;
    try {
        Slot &d = slots_[size_t(dst)];
        const int full = n_pos / kPage;
        for (int i = 0; i < full; ++i) {
            const int page = s.pages[size_t(i)];
            ++page_ref_[size_t(page)];
            d.pages.push_back(page);
            upd.push_back(dst);
            upd.push_back(i);
            upd.push_back(page);
        }
        if (n_pos % kPage) {
            const int page = alloc_page();
            copy_page(page, s.pages[size_t(full)]);
            d.pages.push_back(page);
            upd.push_back(dst);
            upd.push_back(full);
            upd.push_back(page);
        }
        d.pos = n_pos;
        CK(cudaMemcpyAsync(hidden_ + size_t(dst) * kHidden, hidden_ + size_t(src) * kHidden, kHidden * sizeof(float),
                           cudaMemcpyDeviceToDevice, stream_));
        upload_page_updates(upd);
        CK(cudaStreamSynchronize(stream_));
    } catch (...) {
        close_stream(dst);
        throw;
    }
    return dst;
}

// Page-table entries reach the device through the control block (no allocation): at most
// r_max_ entries per pass, applied by k_page_updates before the pass's kernels.
void Engine::upload_page_updates(const std::vector<int> &updates) {
    const size_t n = updates.size() / 3;
    int *h = h_ctl_ + off_pages();
    for (size_t done = 0; done < n;) {
        const size_t m = std::min(n - done, size_t(r_max_));
        h[0] = int(m);
        std::memcpy(h + 1, updates.data() + 3 * done, m * 3 * sizeof(int));
        CK(cudaMemcpyAsync(d_ctl_ + off_pages(), h, (1 + 3 * m) * sizeof(int), cudaMemcpyHostToDevice, stream_));
        k_page_updates<<<unsigned((m + 127) / 128), 128, 0, stream_>>>(d_ctl_ + off_pages(), page_table_,
                                                                      pages_per_stream_);
        CK(cudaStreamSynchronize(stream_));  // the pinned staging is reused by the next pass
        done += m;
    }
    h[0] = 0;
}

// ------------------------------------------------------------------ public API

int Engine::open_stream() {
    for (int i = 0; i < max_streams_; ++i) {
        if (!slots_[size_t(i)].open) {
            slots_[size_t(i)] = Slot{};
            slots_[size_t(i)].open = true;
            return i;
        }
    }
    throw std::runtime_error("no free stream slot (max_streams reached)");
}

void Engine::close_stream(int sid) {
    check_slot(sid);
    release_pages(slots_[size_t(sid)]);
    slots_[size_t(sid)] = Slot{};
}

void Engine::reset_stream(int sid) {
    check_slot(sid);
    slots_[size_t(sid)].pos = 0;
}

int Engine::position(int sid) const {
    check_slot(sid);
    return slots_[size_t(sid)].pos;
}

// The flash-prefill work list of a pass whose row k has slot[k] and position pos[k]: runs of
// consecutive positions of one stream cut into tiles of <= 128 rows (k_attn_prefill_tc, one
// CTA per tile and head), longest key range first.
void Engine::plan_prefill_attention(int R, const int *slot, const int *pos) {
    std::vector<int4> tiles;
    for (int k = 0; k < R;) {
        int n = 1;
        while (k + n < R && n < kPtRows && slot[k + n] == slot[k] && pos[k + n] == pos[k] + n) ++n;
        tiles.push_back(make_int4(k, n, pos[k], slot[k]));
        k += n;
    }
    std::stable_sort(tiles.begin(), tiles.end(), [](const int4 &a, const int4 &b) { return a.z + a.y > b.z + b.y; });
    for (size_t i = 0; i < tiles.size(); ++i) h_pf_items_[i] = tiles[i];
    pf_tc_items_ = int(tiles.size());
    CK(cudaMemcpyAsync(pf_items_, h_pf_items_, tiles.size() * sizeof(int4), cudaMemcpyHostToDevice, stream_));
}

// LlmModel::prefill (llm.cpp:327-401) for several streams at once.  Each stream's rows are
// clamped as the reference clamps them (llm.cpp:329-331); the rows of all streams form one
// sequence that runs through the layers in passes of up to r_max_ rows (a pass may hold
// rows of several streams and a stream may span passes: each row attends to its own
// stream's positions <= its own, all of which are in the KV cache by the time its layer's
// attention runs).  The ln_f of a stream's last row becomes its hidden state.
void Engine::prefill_batch(int n, const int32_t *sids, const int32_t *m_in, const int32_t *start_in,
                           const int32_t *rows, const float *xin) {
    if (n <= 0) return;
    std::vector<int> sid(static_cast<size_t>(n)), m(static_cast<size_t>(n)), start(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
        check_slot(sids[i]);
        for (int j = 0; j < i; ++j)
            if (sids[j] == sids[i]) throw std::runtime_error("stream " + std::to_string(sids[i]) + " repeated in a prefill batch");
        sid[size_t(i)] = sids[i];
        start[size_t(i)] = std::max(0, std::min(start_in[i], max_ctx_));
        m[size_t(i)] = std::max(0, std::min(m_in[i], max_ctx_ - start[size_t(i)]));
    }
    // input row of stream i's first row (rows are taken stream after stream, before clamping)
    std::vector<size_t> src0(static_cast<size_t>(n) + 1, 0);
    for (int i = 0; i < n; ++i) src0[size_t(i) + 1] = src0[size_t(i)] + size_t(std::max(0, m_in[i]));
    if (rows) {
        for (int i = 0; i < n; ++i)
            for (int r = 0; r < std::max(0, m_in[i]); ++r) {
                const int v = rows[(src0[size_t(i)] + size_t(r)) * (kNVq + 1)];
                if (v < 0 || v >= kVocab)
                    throw std::runtime_error("text id out of range in prefill row " + std::to_string(r));
            }
    }
    std::vector<int> upd;
    for (int i = 0; i < n; ++i)
        if (m[size_t(i)] > 0) ensure_pages(sid[size_t(i)], start[size_t(i)], start[size_t(i)] + m[size_t(i)] - 1, upd);
    upload_page_updates(upd);
    // flat row list: (stream index, row within the stream)
    std::vector<std::pair<int, int>> flat;
    for (int i = 0; i < n; ++i)
        for (int r = 0; r < m[size_t(i)]; ++r) flat.emplace_back(i, r);
    const size_t total = flat.size();
    for (size_t c0 = 0; c0 < total; c0 += size_t(r_max_)) {
        const int R = int(std::min(size_t(r_max_), total - c0));
        int *slot = h_ctl_, *pos = h_ctl_ + r_max_;
        for (int k = 0; k < R; ++k) {
            const auto &fr = flat[c0 + size_t(k)];
            slot[k] = sid[size_t(fr.first)];
            pos[k] = start[size_t(fr.first)] + fr.second;
        }
        CK(cudaMemcpyAsync(d_ctl_, h_ctl_, size_t(2 * r_max_) * sizeof(int), cudaMemcpyHostToDevice, stream_));
        // the pass's inputs: runs of consecutive rows of one stream are contiguous in the input
        for (int k = 0; k < R;) {
            const auto &fr = flat[c0 + size_t(k)];
            int len = 1;
            while (k + len < R && flat[c0 + size_t(k + len)].first == fr.first) ++len;
            const size_t src = src0[size_t(fr.first)] + size_t(fr.second);
            if (rows)
                CK(cudaMemcpyAsync(rows17_ + size_t(k) * (kNVq + 1), rows + src * (kNVq + 1),
                                   size_t(len) * (kNVq + 1) * sizeof(int), cudaMemcpyHostToDevice, stream_));
            else
                CK(cudaMemcpyAsync(x_ + size_t(k) * kHidden, xin + src * kHidden, size_t(len) * kHidden * sizeof(float),
                                   cudaMemcpyHostToDevice, stream_));
            k += len;
        }
        if (rows) launch_k(false, k_embed_rows, dim3(R), dim3(256), 0, stream_, tables(), rows17_, R, x_);
        pf_active_ = use_tc(R);
        if (pf_active_) plan_prefill_attention(R, slot, pos);
        in_prefill_ = true;  // rows of one stream attend to each other: not the small-batch layers
        try {
            global_layers(R, d_ctl_, d_ctl_ + r_max_);
        } catch (...) {
            pf_active_ = false;
            in_prefill_ = false;
            throw;
        }
        pf_active_ = false;
        in_prefill_ = false;
        // ln_f of each stream's last row in this pass becomes its hidden state (llm.cpp:395-399),
        // all of them in one launch; the (row, slot) pairs go into rows17_, which the pass has
        // consumed (k_embed_rows ran before the layers on this stream)
        std::vector<int> pick;  // [rows of the pass..., their slots...]
        for (int k = 0; k < R; ++k) {
            const auto &fr = flat[c0 + size_t(k)];
            if (fr.second == m[size_t(fr.first)] - 1) pick.push_back(k);
        }
        const int np = static_cast<int>(pick.size());
        if (np > 0) {
            for (int i = 0; i < np; ++i) pick.push_back(sid[size_t(flat[c0 + size_t(pick[size_t(i)])].first)]);
            CK(cudaMemcpyAsync(rows17_, pick.data(), pick.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
            launch_k(pdl_, k_layernorm_pick, dim3(np), dim3(256), 0, stream_, static_cast<const float *>(x_),
                     static_cast<const int *>(rows17_), static_cast<const int *>(rows17_ + np), np, lnf_w_, lnf_b_,
                     hidden_);
        }
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(h_err_, dev_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        check_device_error();
    }
    for (int i = 0; i < n; ++i)
        if (m[size_t(i)] > 0) slots_[size_t(sid[size_t(i)])].pos = start[size_t(i)] + m[size_t(i)];
}

void Engine::prefill(int sid, const int32_t *rows, int m, int start) {
    const int32_t s = sid, mm = m, st = start;
    prefill_batch(1, &s, &mm, &st, rows, nullptr);
}

void Engine::prefill_embeds(int sid, const float *x, int m, int start) {
    const int32_t s = sid, mm = m, st = start;
    prefill_batch(1, &s, &mm, &st, nullptr, x);
}

namespace {
// The sampler's generator as generate() seeds it (sampler.h:28-48): xoshiro128** with the
// seed's two halves in the first words, two fixed words, then 8 draws discarded.
void seed_xoshiro(uint32_t st[4], uint64_t v) {
    st[0] = uint32_t(v);
    st[1] = uint32_t(v >> 32) ^ 0x9E3779B9u;
    st[2] = 0x243F6A88u;
    st[3] = 0xB7E15162u;
    auto rotl = [](uint32_t x, int k) { return (x << k) | (x >> (32 - k)); };
    for (int i = 0; i < 8; ++i) {
        const uint32_t t = st[1] << 9;
        st[2] ^= st[0];
        st[3] ^= st[1];
        st[1] ^= st[2];
        st[0] ^= st[3];
        st[2] ^= t;
        st[3] = rotl(st[3], 11);
    }
}
}  // namespace

void Engine::generate_begin(int sid, uint64_t seed) {
    check_slot(sid);
    Slot &s = slots_[size_t(sid)];
    s.frame = 0;
    s.seed = seed;
    uint32_t st[4];
    seed_xoshiro(st, seed);
    CK(cudaMemsetAsync(counts_ + size_t(sid) * kNVq * kCodebook, 0, size_t(kNVq) * kCodebook * sizeof(uint16_t), stream_));
    CK(cudaMemcpyAsync(rng_ + size_t(sid) * 4, st, sizeof(st), cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));
}

void Engine::step(const int32_t *sids, int n, const SampleParamsC &p, const int32_t *forced, int32_t *out_codes,
                  uint8_t *out_stop, float *out_logits, float *out_gate, bool run_global) {
    if (n <= 0) return;
    if (n > max_streams_) throw std::runtime_error("batch larger than max_streams");
    launches_ = 0;
    std::vector<int> upd;
    std::vector<char> seen(size_t(max_streams_), 0);
    for (int r = 0; r < n; ++r) {
        const int sid = sids[r];
        check_slot(sid);
        if (seen[size_t(sid)]) throw std::runtime_error("stream listed twice in one step");
        seen[size_t(sid)] = 1;
        if (run_global) ensure_pages(sid, slots_[size_t(sid)].pos, slots_[size_t(sid)].pos, upd);
    }
    if (forced) {
        for (int i = 0; i < n * kNVq; ++i)
            if (forced[i] < 0 || forced[i] >= kCodebook) throw std::runtime_error("forced code out of range");
    }
    const int R = n;
    int *slot = h_ctl_ + off_slot(), *pos = h_ctl_ + off_pos(), *frame = h_ctl_ + off_frame();
    int *frc = h_ctl_ + off_forced();
    FrameCtl *fc = reinterpret_cast<FrameCtl *>(h_ctl_ + off_fctl());
    for (int r = 0; r < R; ++r) {
        const Slot &s = slots_[size_t(sids[r])];
        slot[r] = sids[r];
        pos[r] = s.pos;
        frame[r] = s.frame;
        h_ctl_[off_active_in() + r] = 1;
        if (forced) std::memcpy(frc + r * kNVq, forced + size_t(r) * kNVq, kNVq * sizeof(int));
    }
    h_ctl_[off_fslot()] = 0;
    fc->min_frames = p.min_frames;
    fc->greedy_frames = p.greedy_frames;
    fc->rep_penalty = p.repetition_penalty;
    fc->end_greedy = p.end_greedy;
    fc->greedy = p.greedy;
    fc->temperature = p.temperature;
    fc->top_k = p.top_k;
    fc->top_p = p.top_p;
    fc->has_forced = forced ? 1 : 0;
    // page updates ride in the same control block copy (decode adds at most one page per row)
    h_ctl_[off_pages()] = int(upd.size() / 3);
    std::memcpy(h_ctl_ + off_pages() + 1, upd.data(), upd.size() * sizeof(int));
    CK(cudaMemcpyAsync(d_ctl_, h_ctl_, size_t(ctl_ints_) * sizeof(int), cudaMemcpyHostToDevice, stream_));
    frame_fused_ = fused_ok(p);
    run_captured((uint64_t(1) << 40) | (uint64_t(frame_fused_) << 36) | (uint64_t(run_global) << 32) | uint64_t(R),
                 [&] { issue_frame(R, run_global); });
    // ---- outputs
    uint8_t *ho = h_out_;
    int *h_codes = reinterpret_cast<int *>(ho);
    int *h_active = h_codes + R * kNVq;
    float *h_gate = reinterpret_cast<float *>(h_active + R);
    float *h_logits = h_gate + 2 * R;
    CK(cudaMemcpyAsync(h_codes, codes_, size_t(R) * kNVq * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(h_active, active_, size_t(R) * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(h_gate, gate_, size_t(R) * 2 * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    if (out_logits)
        CK(cudaMemcpyAsync(h_logits, logits_, size_t(R) * kNVq * kCodebook * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(h_err_, dev_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    check_device_error();
    accumulate_timing();
    for (int r = 0; r < R; ++r) {
        const bool act = h_active[r] != 0;
        if (out_codes) std::memcpy(out_codes + size_t(r) * kNVq, h_codes + size_t(r) * kNVq, kNVq * sizeof(int));
        if (out_stop) out_stop[r] = act ? 0 : 1;
        if (out_gate) {
            out_gate[2 * r] = h_gate[2 * r];
            out_gate[2 * r + 1] = h_gate[2 * r + 1];
        }
        Slot &s = slots_[size_t(sids[r])];
        if (act) {
            s.frame += 1;
            if (run_global) s.pos += 1;
        }
    }
    if (out_logits) std::memcpy(out_logits, h_logits, size_t(R) * kNVq * kCodebook * sizeof(float));
}

// n_frames consecutive frames for n streams without a host round trip between frames: the
// frame graph is replayed back to back and k_frame_commit advances positions, frame indices
// and active flags on the device.  Pages for every position the call can write are
// reserved up front.  out_codes [n_frames][n][16] (-1 after a stream stopped);
// out_frames_done [n] = frames each stream produced.
void Engine::step_frames(const int32_t *sids, int n, const SampleParamsC &p, int n_frames, int32_t *out_codes,
                         int32_t *out_frames_done) {
    if (n <= 0 || n_frames <= 0) return;
    if (n > max_streams_) throw std::runtime_error("batch larger than max_streams");
    if (n_frames > kMaxFramesPerCall) throw std::runtime_error("n_frames above the per-call limit");
    std::vector<int> upd;
    std::vector<char> seen(size_t(max_streams_), 0);
    for (int r = 0; r < n; ++r) {
        const int sid = sids[r];
        check_slot(sid);
        if (seen[size_t(sid)]) throw std::runtime_error("stream listed twice in one step");
        seen[size_t(sid)] = 1;
        ensure_pages(sid, slots_[size_t(sid)].pos, slots_[size_t(sid)].pos + n_frames - 1, upd);
    }
    upload_page_updates(upd);
    const int R = n;
    for (int r = 0; r < R; ++r) {
        const Slot &s = slots_[size_t(sids[r])];
        h_ctl_[off_slot() + r] = sids[r];
        h_ctl_[off_pos() + r] = s.pos;
        h_ctl_[off_frame() + r] = s.frame;
        h_ctl_[off_active_in() + r] = 1;
    }
    h_ctl_[off_pages()] = 0;
    h_ctl_[off_fslot()] = 0;
    FrameCtl *fc = reinterpret_cast<FrameCtl *>(h_ctl_ + off_fctl());
    fc->min_frames = p.min_frames;
    fc->greedy_frames = p.greedy_frames;
    fc->rep_penalty = p.repetition_penalty;
    fc->end_greedy = p.end_greedy;
    fc->greedy = p.greedy;
    fc->temperature = p.temperature;
    fc->top_k = p.top_k;
    fc->top_p = p.top_p;
    fc->has_forced = 0;
    CK(cudaMemcpyAsync(d_ctl_, h_ctl_, size_t(ctl_ints_) * sizeof(int), cudaMemcpyHostToDevice, stream_));
    int total_launches = 0;
    frame_fused_ = fused_ok(p);
    for (int f = 0; f < n_frames; ++f) {
        run_captured((uint64_t(1) << 40) | (uint64_t(frame_fused_) << 36) | (uint64_t(1) << 32) | uint64_t(R),
                     [&] { issue_frame(R, true); });
        total_launches += launches_;
        if (timing_ && f + 1 < n_frames) {
            CK(cudaStreamSynchronize(stream_));
            accumulate_timing();
        }
    }
    int *h_frames = reinterpret_cast<int *>(h_out_);
    CK(cudaMemcpyAsync(h_frames, d_ctl_ + off_frame(), size_t(R) * sizeof(int), cudaMemcpyDeviceToHost, stream_));
    if (out_codes)
        CK(cudaMemcpyAsync(out_codes, codes_hist_, size_t(n_frames) * R * kNVq * sizeof(int), cudaMemcpyDeviceToHost,
                           stream_));
    CK(cudaMemcpyAsync(h_err_, dev_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    check_device_error();
    accumulate_timing();
    launches_ = total_launches;
    for (int r = 0; r < R; ++r) {
        Slot &s = slots_[size_t(sids[r])];
        const int done = h_frames[r] - s.frame;
        s.frame += done;
        s.pos += done;
        if (out_frames_done) out_frames_done[r] = done;
    }
}

void Engine::global_step_embed(const int32_t *sids, int n, const float *x, float *hidden_out) {
    if (n <= 0) return;
    if (n > max_streams_) throw std::runtime_error("batch larger than max_streams");
    launches_ = 0;
    std::vector<int> upd;
    for (int r = 0; r < n; ++r) {
        check_slot(sids[r]);
        ensure_pages(sids[r], slots_[size_t(sids[r])].pos, slots_[size_t(sids[r])].pos, upd);
    }
    upload_page_updates(upd);
    int *slot = h_ctl_, *pos = h_ctl_ + r_max_;
    for (int r = 0; r < n; ++r) {
        slot[r] = sids[r];
        pos[r] = slots_[size_t(sids[r])].pos;
    }
    CK(cudaMemcpyAsync(d_ctl_, h_ctl_, size_t(2 * r_max_) * sizeof(int), cudaMemcpyHostToDevice, stream_));
    std::memcpy(h_x_, x, size_t(n) * kHidden * sizeof(float));
    CK(cudaMemcpyAsync(x_, h_x_, size_t(n) * kHidden * sizeof(float), cudaMemcpyHostToDevice, stream_));
    run_captured((uint64_t(2) << 40) | uint64_t(n), [&] { issue_global_embed(n); });
    float *h = reinterpret_cast<float *>(h_out_);
    if (hidden_out) {
        launch_k(false, k_gather_rows, dim3(n), dim3(256), 0, stream_, hidden_, d_ctl_, n, q_);
        CK(cudaMemcpyAsync(h, q_, size_t(n) * kHidden * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    }
    CK(cudaMemcpyAsync(h_err_, dev_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    check_device_error();
    if (hidden_out) std::memcpy(hidden_out, h, size_t(n) * kHidden * sizeof(float));
    accumulate_timing();
    for (int r = 0; r < n; ++r) slots_[size_t(sids[r])].pos += 1;
}

// The launch sequence of one frame for R rows (llm.cpp:643-712); all per-call data comes
// from the control block already copied to d_ctl_, so the sequence is graph-capturable.
void Engine::issue_frame(int R, bool run_global) {
    const int *d_slot = d_ctl_ + off_slot(), *d_pos = d_ctl_ + off_pos(), *d_frame = d_ctl_ + off_frame();
    const int *d_forced = d_ctl_ + off_forced();
    const FrameCtl *d_fc = reinterpret_cast<const FrameCtl *>(d_ctl_ + off_fctl());
    // builder state carried between launches of one frame only (an exception in an earlier
    // frame's issue must not leave it set)
    ln1_prebuilt_ = false;
    pending_resid_ = nullptr;
    k_page_updates<<<unsigned((R + 127) / 128), 128, 0, stream_>>>(d_ctl_ + off_pages(), page_table_, pages_per_stream_);
    mark(KK_PAGES);
    // ---- local decoder: 17 steps (llm.cpp:648-698)
    if (frame_fused_) {  // greedy frames: step 0, the end gate, steps 1..16 with heads and codes
        launch_local_fused(R, 0, 1);
        launch_k(pdl_, k_gate, dim3(R), dim3(256), 0, stream_, lx_, R, llnf_w_, llnf_b_, qm(wte_), d_frame, d_fc,
                 d_ctl_ + off_active_in(), active_, gate_, d_slot, rng_);
        mark(KK_GATE);
        launch_local_fused(R, 1, kLocalLen);
    } else {
    launch_k(pdl_, k_gather_rows, dim3(R), dim3(256), 0, stream_, hidden_, d_slot, R, lx_);
    mark(KK_GATHER);
    for (int ls = 0; ls < kLocalLen; ++ls) {
        if (ls == 1) {
            launch_k(pdl_, k_lookup_rows, dim3(R), dim3(256), 0, stream_, qm(wte_), kSlotToken, R, lx_);
            mark(KK_LOOKUP);
        }
        block(local_, 0, true, R, d_slot, nullptr, ls, lx_);
        if (ls == 0) {
            launch_k(pdl_, k_gate, dim3(R), dim3(256), 0, stream_, lx_, R, llnf_w_, llnf_b_, qm(wte_), d_frame, d_fc,
                     d_ctl_ + off_active_in(), active_, gate_, d_slot, rng_);
            mark(KK_GATE);
        } else {
            const int ch = ls - 1;
            if (use_tc(R)) {
                heads_tc(ch, R);
            } else {
                GemvArgs h{};
                h.nrows = R;
                h.w = qm(aemb_[ch]);
                h.x = lx_;
                h.ldx = kHidden;
                h.ln_w = llnf_w_;
                h.ln_b = llnf_b_;
                h.out = logits_ + size_t(ch) * kCodebook;
                h.ldo = kNVq * kCodebook;
                launch_gemv<PRO_LN, EPI_STORE>(h, stream_, pdl_);
                mark(KK_HEADS);
            }
            // on the tensor-core path the sampler also writes the next step's LN1 image
            NextImage img;
            if (use_tc(R) && ch + 1 < kNVq) {
                img.ln_w = local_.ln1_w;
                img.ln_b = local_.ln1_b;
                img.bimg = bimg_a_;
                img.N = (R + 15) / 16 * 16;
                img.parts = tc_parts(gemm_path_ == 3 ? TC_F16 : TC_F16X3);
                ln1_prebuilt_ = true;
            }
            launch_k(pdl_, k_sample, dim3(R), dim3(256), 0, stream_, logits_ + size_t(ch) * kCodebook, kNVq * kCodebook,
                     ch, d_slot, R, counts_, d_fc, d_forced, active_, codes_, used_, qm(aemb_[ch]),
                     ch + 1 < kNVq ? lx_ : nullptr, d_frame, rng_, img);
            mark(KK_SAMPLE);
        }
    }
    }
    // ---- global step on [9, used codes] (llm.cpp:703-708)
    if (run_global) {
        launch_k(pdl_, k_embed_frame, dim3(R), dim3(256), 0, stream_, tables(), used_, R, x_);
        mark(KK_EMBED);
        global_layers(R, d_slot, d_pos);
        launch_k(pdl_, k_layernorm_rows, dim3(R), dim3(256), 0, stream_, x_, R, lnf_w_, lnf_b_, hidden_, d_slot, active_,
                 lnf_xfix_);
        mark(KK_LNF);
    }
    launch_k(pdl_, k_frame_commit, dim3(1), dim3(256), 0, stream_, codes_, active_, R, run_global ? 1 : 0, d_ctl_ + off_pos(),
                                           d_ctl_ + off_frame(), d_ctl_ + off_active_in(), d_ctl_ + off_fslot(),
                                           kMaxFramesPerCall, codes_hist_);
    mark(KK_COMMIT);
}

// 12 global layers + ln_f on embeddings already in x_ (llm.cpp:248-255).
void Engine::issue_global_embed(int R) {
    global_layers(R, d_ctl_ + off_slot(), d_ctl_ + off_pos());
    launch_k(pdl_, k_layernorm_rows, dim3(R), dim3(256), 0, stream_, x_, R, lnf_w_, lnf_b_, hidden_, d_ctl_ + off_slot(),
             static_cast<const int *>(nullptr), lnf_xfix_);
    mark(KK_LNF);
}

// ------------------------------------------------------------------ graphs and timing

const char *kernel_kind_name(int kind) {
    static const char *names[KK_COUNT] = {
        "page_updates", "gather_hidden", "lookup_slot_row", "embed_frame", "attn_plan",
        "qkv_global", "attn_decode_paged", "proj_global", "fc_in_global", "fc_out_global", "ln_f",
        "qkv_local", "attn_local", "proj_local", "fc_in_local", "fc_out_local", "gate_w8a8",
        "audio_heads", "sample", "frame_commit", "build_activation_image", "attn_combine", "attn_prefill", "qkv_rope",
        "local_decoder_fused", "small_layer_attn", "small_layer_mlp"};
    return (kind >= 0 && kind < KK_COUNT) ? names[kind] : "?";
}

void Engine::mark(int kind) {
    ++launches_;
    if (capturing_ && timing_) {
        cudaEvent_t ev;
        CK(cudaEventCreate(&ev));
        CK(cudaEventRecordWithFlags(ev, stream_, cudaEventRecordExternal));  // a timed node of the graph
        capturing_->events.push_back(ev);
        capturing_->kinds.push_back(kind);
    }
}

template <class F>
void Engine::run_captured(uint64_t key, F &&issue) {
    launches_ = 0;
    last_graph_ = nullptr;
    if (!use_graphs_) {
        issue();
        CK(cudaGetLastError());
        return;
    }
    key |= (uint64_t(timing_) << 48) | (uint64_t(gemm_path_) << 50);  // both change what is captured
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
        CapturedGraph g;
        capturing_ = &g;
        cudaGraph_t graph = nullptr;
        CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        if (timing_) {
            cudaEvent_t ev;
            CK(cudaEventCreate(&ev));
            CK(cudaEventRecordWithFlags(ev, stream_, cudaEventRecordExternal));  // a timed node of the graph
            g.events.push_back(ev);
        }
        try {
            issue();
        } catch (...) {
            cudaStreamEndCapture(stream_, &graph);
            if (graph) cudaGraphDestroy(graph);
            capturing_ = nullptr;
            throw;
        }
        capturing_ = nullptr;
        CK(cudaStreamEndCapture(stream_, &graph));
        CK(cudaGraphInstantiate(&g.exec, graph, 0));
        CK(cudaGraphDestroy(graph));
        g.launches = launches_;
        it = graphs_.emplace(key, std::move(g)).first;
    }
    CK(cudaGraphLaunch(it->second.exec, stream_));
    launches_ = it->second.launches;
    last_graph_ = timing_ ? &it->second : nullptr;
}

void Engine::accumulate_timing() {
    if (!timing_ || !last_graph_) return;
    const CapturedGraph &g = *last_graph_;
    for (size_t i = 0; i + 1 < g.events.size(); ++i) {
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, g.events[i], g.events[i + 1]));
        prof_ms_[g.kinds[i]] += ms;
        prof_n_[g.kinds[i]] += 1;
    }
    last_graph_ = nullptr;
}

void Engine::set_kernel_timing(bool on) {
    timing_ = on;
    for (int k = 0; k < KK_COUNT; ++k) {
        prof_ms_[k] = 0.0;
        prof_n_[k] = 0;
    }
}

void Engine::read_kernel_timing(float *total_ms, int *launches, int max_kinds, int *n_kinds) const {
    const int n = std::min(max_kinds, int(KK_COUNT));
    for (int k = 0; k < n; ++k) {
        if (total_ms) total_ms[k] = float(prof_ms_[k]);
        if (launches) launches[k] = prof_n_[k];
    }
    if (n_kinds) *n_kinds = KK_COUNT;
}

// ------------------------------------------------------------------ state access

namespace {

__global__ void k_kv_scatter(const float *__restrict__ src, int n, int p0, const int *__restrict__ pages,
                             __half *__restrict__ kv, int n_pages, int kvsel) {
    // src [12][n][768] fp32 -> pages of this stream
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = (long long)kLayers * n * kHidden;
    if (t >= total) return;
    const int c = int(t % kHidden);
    const int p = int((t / kHidden) % n) + p0;
    const int l = int(t / ((long long)kHidden * n));
    const int page = pages[p / kPage];
    kv[(size_t)l * n_pages * kPageHalfs + (size_t)page * kPageHalfs +
       ((kvsel * kHeads + c / kHeadDim) * kPage + p % kPage) * kHeadDim + c % kHeadDim] = __float2half_rn(src[t]);
}

__global__ void k_kv_gather(const __half *__restrict__ kv, int n_pages, int layer, int p0, int n,
                            const int *__restrict__ pages, int kvsel, float *__restrict__ dst) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)n * kHidden) return;
    const int c = int(t % kHidden);
    const int p = int(t / kHidden) + p0;
    const int page = pages[p / kPage];
    dst[t] = __half2float(kv[(size_t)layer * n_pages * kPageHalfs + (size_t)page * kPageHalfs +
                             ((kvsel * kHeads + c / kHeadDim) * kPage + p % kPage) * kHeadDim + c % kHeadDim]);
}

}  // namespace

void Engine::set_state(int sid, const float *k, const float *v, int n_pos, const float *hidden) {
    check_slot(sid);
    if (n_pos <= 0 || n_pos > max_ctx_) throw std::runtime_error("bad state length");
    Slot &s = slots_[size_t(sid)];
    std::vector<int> upd;
    ensure_pages(sid, 0, n_pos - 1, upd);
    upload_page_updates(upd);
    const size_t nel = size_t(kLayers) * n_pos * kHidden;
    float *d = nullptr;
    int *dp = nullptr;
    CK(cudaMalloc(&d, nel * sizeof(float)));
    CK(cudaMalloc(&dp, s.pages.size() * sizeof(int)));
    // every copy goes through the engine's stream: a blocking cudaMemcpy from pageable memory
    // may return before its DMA lands and is not ordered with a non-blocking stream
    CK(cudaMemcpyAsync(dp, s.pages.data(), s.pages.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
    for (int kvsel = 0; kvsel < 2; ++kvsel) {
        CK(cudaMemcpyAsync(d, kvsel ? v : k, nel * sizeof(float), cudaMemcpyHostToDevice, stream_));
        k_kv_scatter<<<unsigned((nel + 255) / 256), 256, 0, stream_>>>(d, n_pos, 0, dp, kv_, n_pages_, kvsel);
        CK(cudaStreamSynchronize(stream_));
    }
    if (hidden)
        CK(cudaMemcpyAsync(hidden_ + size_t(sid) * kHidden, hidden, kHidden * sizeof(float), cudaMemcpyHostToDevice,
                           stream_));
    CK(cudaStreamSynchronize(stream_));
    CK(cudaFree(d));
    CK(cudaFree(dp));
    s.pos = n_pos;
}

void Engine::get_kv(int sid, int layer, int p0, int n, float *k, float *v) {
    check_slot(sid);
    const Slot &s = slots_[size_t(sid)];
    if (layer < 0 || layer >= kLayers || p0 < 0 || n <= 0 || (p0 + n - 1) / kPage >= int(s.pages.size()))
        throw std::runtime_error("get_kv range outside the stream's pages");
    float *d = nullptr;
    int *dp = nullptr;
    CK(cudaMalloc(&d, size_t(n) * kHidden * sizeof(float)));
    CK(cudaMalloc(&dp, s.pages.size() * sizeof(int)));
    CK(cudaMemcpyAsync(dp, s.pages.data(), s.pages.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
    for (int kvsel = 0; kvsel < 2; ++kvsel) {
        float *out = kvsel ? v : k;
        if (!out) continue;
        k_kv_gather<<<unsigned((size_t(n) * kHidden + 255) / 256), 256, 0, stream_>>>(kv_, n_pages_, layer, p0, n, dp,
                                                                                       kvsel, d);
        CK(cudaMemcpyAsync(out, d, size_t(n) * kHidden * sizeof(float), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
    }
    CK(cudaFree(d));
    CK(cudaFree(dp));
}

void Engine::get_hidden(int sid, float *out) {
    check_slot(sid);
    CK(cudaMemcpyAsync(out, hidden_ + size_t(sid) * kHidden, kHidden * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
}

void Engine::debug_matrix_bytes(const std::string &name, uint8_t *out, size_t out_bytes) {
    auto it = mats_.find(name);
    if (it == mats_.end()) throw std::runtime_error("no matrix named " + name);
    const DevMat &m = it->second;
    const size_t nblocks = size_t(m.rows / 4) * (m.cols / 32);
    if (out_bytes < nblocks * 136) throw std::runtime_error("output buffer too small");
    std::vector<int8_t> qs(nblocks * 128);
    std::vector<uint16_t> sc(nblocks * 4);
    CK(cudaStreamSynchronize(stream_));
    CK(cudaMemcpy(qs.data(), m.qs, qs.size(), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(sc.data(), m.sc, sc.size() * 2, cudaMemcpyDeviceToHost));
    for (size_t b = 0; b < nblocks; ++b) {
        std::memcpy(out + b * 136, sc.data() + b * 4, 8);
        std::memcpy(out + b * 136 + 8, qs.data() + b * 128, 128);
    }
}

// The tensor-core tile copy of a matrix turned back into Q8_0_4X4 file bytes (inverse of
// k_repack_tiles), to prove that layout is a byte permutation of the file too.
void Engine::debug_matrix_tile_bytes(const std::string &name, uint8_t *out, size_t out_bytes) {
    auto it = mats_.find(name);
    if (it == mats_.end()) throw std::runtime_error("no matrix named " + name);
    const DevMat &m = it->second;
    if (!m.qt) throw std::runtime_error("matrix has no tensor-core tile layout: " + name);
    const int nb = m.cols / 32, nch = m.cols / kTcK;
    if (out_bytes < size_t(m.rows / 4) * nb * 136) throw std::runtime_error("output buffer too small");
    std::vector<int8_t> qt(size_t(m.rows) * m.cols);
    std::vector<uint16_t> st(size_t(m.rows) * nb);
    CK(cudaMemcpyAsync(qt.data(), m.qt, qt.size(), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(st.data(), m.st, st.size() * 2, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    for (int row = 0; row < m.rows; ++row) {
        const int tile = row / kTcM, mm = row % kTcM, k4 = row & 3;
        for (int c = 0; c < nch; ++c) {
            const size_t base = (size_t(tile) * nch + c) * kTcM + mm;
            for (int j = 0; j < 4; ++j) {
                const int b = 2 * c + (j >> 1);
                uint8_t *blk = out + (size_t(row >> 2) * nb + b) * 136;
                std::memcpy(blk + 8 + k4 * 32 + (j & 1) * 16, qt.data() + base * 64 + ((j ^ ((mm >> 1) & 3)) << 4), 16);
                if ((j & 1) == 0) std::memcpy(blk + k4 * 2, st.data() + base * 2 + (j >> 1), 2);
            }
        }
    }
}

void Engine::set_cuda_stream(void *s) {
    CK(cudaStreamSynchronize(stream_));
    stream_ = s ? static_cast<cudaStream_t>(s) : own_stream_;
}

namespace {

// N(0,1) from a counter-based hash (splitmix64) and the Box-Muller transform.
__device__ __forceinline__ float hashed_normal(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float u1 = (float((z >> 40) & 0xFFFFFF) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = float(z & 0xFFFFFF) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void k_fill_state_normal(__half *__restrict__ kv, int n_pages, const int *__restrict__ pages, int n_pos,
                                    uint64_t seed, float *__restrict__ hidden) {
    const long long total = 2LL * kLayers * n_pos * kHidden;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int c = int(t % kHidden);
        const int p = int((t / kHidden) % n_pos);
        const int kvsel = int((t / ((long long)kHidden * n_pos)) & 1);
        const int l = int(t / (2LL * kHidden * n_pos));
        kv[(size_t)l * n_pages * kPageHalfs + (size_t)pages[p / kPage] * kPageHalfs +
           ((kvsel * kHeads + c / kHeadDim) * kPage + p % kPage) * kHeadDim + c % kHeadDim] =
            __float2half_rn(hashed_normal(seed, uint64_t(t)));
    }
    if (blockIdx.x == 0)
        for (int c = threadIdx.x; c < kHidden; c += blockDim.x) hidden[c] = hashed_normal(~seed, uint64_t(c));
}

}  // namespace

// Synthetic prefilled state for benchmarks and tests: K, V ~ N(0,1) rounded to fp16 for
// positions 0..n_pos-1 of every layer, hidden ~ N(0,1); deterministic for a seed.
void Engine::debug_inject_wait_timeout(bool on) {
    const int v = on ? 1 : 0;
    CK(cudaMemcpyAsync(dev_err_ + 1, &v, sizeof(int), cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));
}

void Engine::fill_state_random(int sid, int n_pos, uint64_t seed) {
    check_slot(sid);
    if (n_pos <= 0 || n_pos > max_ctx_) throw std::runtime_error("bad state length");
    Slot &s = slots_[size_t(sid)];
    std::vector<int> upd;
    ensure_pages(sid, 0, n_pos - 1, upd);
    upload_page_updates(upd);
    k_fill_state_normal<<<148 * 8, 256, 0, stream_>>>(kv_, n_pages_, page_table_ + size_t(sid) * pages_per_stream_,
                                                      n_pos, seed, hidden_ + size_t(sid) * kHidden);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(stream_));
    s.pos = n_pos;
}

}  // namespace mossgpu
