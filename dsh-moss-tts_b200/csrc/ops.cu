// ops.cu -- standalone kernel-level C entry points over caller-owned device buffers.
//
// mossgpu_attention_decode_paged: the engine's paged fp16 flash-decode (one layer) for
// callers that keep their own KV pages, e.g. a host framework that manages the cache and
// only wants the attention kernel.  Every pointer is a device pointer; the caller also
// provides the scratch workspace (plan, chunk descriptors and counter, split-K partials).
#include "../../include/mossgpu.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "kernels.cuh"

namespace {

thread_local std::string g_op_error;

int op_fail(const std::string &msg) {
    g_op_error = msg;
    return 1;
}

constexpr size_t kAlign = 256;

// Device status of the standalone ops: a kernel whose bounded barrier wait ran out records its
// code here (7: a consumer warp waited for a page, 8: the producer waited for a free stage),
// so that the failure is not silent; mossgpu_op_device_status() reads and clears it.
static __device__ int g_op_status;

// The decode-attention kernel uses 205 KB of dynamic shared memory (its page ring), above the
// 48 KB a launch gets without opting in; the opt-in is per device.
constexpr int kMaxDevices = 64;
std::mutex g_attr_mu;
bool g_attr_set[kMaxDevices] = {};

int *g_status_ptr[kMaxDevices] = {};

// Per-device set-up, once per device with that device current: the shared-memory opt-in and
// the device address of g_op_status (in host code the symbol is only a handle).
int device_setup(int *dev_out, const char *who) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return op_fail(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return op_fail(std::string(who) + ": device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (!g_attr_set[dev]) {
        e = cudaFuncSetAttribute(mossgpu::k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 mossgpu::kAttnSmem);
        if (e != cudaSuccess) return op_fail(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_op_status);
        if (e != cudaSuccess || !p) return op_fail(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_status_ptr[dev] = static_cast<int *>(p);
        g_attr_set[dev] = true;
    }
    *dev_out = dev;
    return 0;
}

// plan -> decode -> combine on `st` over caller-provided scratch.
int run_attention(mossgpu::AttnArgs t, int *work, int4 *desc, int max_items, cudaStream_t st, const char *who) {
    using namespace mossgpu;
    int dev = -1;
    if (device_setup(&dev, who) != 0) return 1;
    cudaError_t e;
    t.err = g_status_ptr[dev];
    k_attn_plan<<<1, kPlanThreads, 0, st>>>(t.row_pos, t.row_slot, t.pages_per_stream, t.R, max_items, const_cast<int *>(t.plan),
                                  desc, work, 1);
    t.desc = desc;
    t.work = work;
    k_attn_decode<<<148, kAttnThreads, kAttnSmem, st>>>(t);
    k_attn_combine<<<(t.R * kHeads + 7) / 8, 256, 0, st>>>(t);
    e = cudaGetLastError();
    if (e != cudaSuccess) return op_fail(std::string(who) + " launch: " + cudaGetErrorString(e));
    return 0;
}

// q rows are read as float4 and the pages are fetched with 16-byte bulk copies
int check_alignment(const float *q, const void *kv_layer, const char *who) {
    if (reinterpret_cast<uintptr_t>(q) % 16 != 0 || reinterpret_cast<uintptr_t>(kv_layer) % 16 != 0)
        return op_fail(std::string(who) + ": q and kv_layer must be 16-byte aligned");
    return 0;
}

size_t round_up(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

// Workspace layout for R rows: [plan: 2 + R + 1 ints][chunk counter][chunk descriptors:
// G int4][partials: G * 12 * kPartStride floats], G = chunks the plan may cut (>= R).
constexpr size_t kGroupBytes = sizeof(float) * mossgpu::kPartStride * mossgpu::kHeads;  // partials of one chunk
struct Layout {
    size_t plan, work, desc, part;
    int groups;
};

Layout layout_for(int R, size_t bytes) {
    Layout l{};
    l.plan = 0;
    l.work = round_up(sizeof(int) * (size_t(R) + 3));
    l.desc = l.work + kAlign;
    const size_t avail = bytes > l.desc ? bytes - l.desc : 0;
    size_t g = avail / (kGroupBytes + sizeof(int4));
    while (g > 0 && round_up(g * sizeof(int4)) + g * kGroupBytes > avail) --g;
    l.groups = int(std::min<size_t>(g, 1u << 26));
    l.part = l.desc + round_up(size_t(l.groups) * sizeof(int4));
    return l;
}

}  // namespace

extern "C" {

const char *mossgpu_op_last_error(void) { return g_op_error.c_str(); }

int mossgpu_op_device_status(int *code) {
    if (!code) return op_fail("op_device_status: code is NULL");
    int dev = -1;
    if (device_setup(&dev, "op_device_status") != 0) return 1;
    int v = 0;
    cudaError_t e = cudaMemcpy(&v, g_status_ptr[dev], sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v != 0) {
        const int zero = 0;
        e = cudaMemcpy(g_status_ptr[dev], &zero, sizeof(int), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return op_fail(std::string("op_device_status: ") + cudaGetErrorString(e));
    *code = v;
    return 0;
}

size_t mossgpu_attention_workspace_bytes(int R) {
    if (R <= 0) return 0;
    // room for 8 split-K chunks per row on average; the plan widens chunks to fit any length
    const Layout l = layout_for(R, 0);
    const size_t g = size_t(R) * 8;
    return l.desc + round_up(g * sizeof(int4)) + g * kGroupBytes;
}

int mossgpu_attention_decode_paged(const float *q, const void *kv_layer, const int32_t *page_table,
                                   int pages_per_stream, const int32_t *row_slot, const int32_t *row_pos, int R,
                                   float *out, void *workspace, size_t workspace_bytes, void *cuda_stream) {
    using namespace mossgpu;
    if (R <= 0) return 0;
    if (!q || !kv_layer || !page_table || !row_slot || !row_pos || !out || !workspace)
        return op_fail("attention_decode_paged: a required pointer is NULL");
    if (pages_per_stream <= 0) return op_fail("attention_decode_paged: pages_per_stream must be positive");
    const Layout l = layout_for(R, workspace_bytes);
    if (l.groups < R)
        return op_fail("attention_decode_paged: workspace too small (need mossgpu_attention_workspace_bytes(R))");
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
        return op_fail("attention_decode_paged: workspace must be 16-byte aligned");
    if (check_alignment(q, kv_layer, "attention_decode_paged") != 0) return 1;
    char *ws = static_cast<char *>(workspace);
    AttnArgs t{};
    t.q = q;
    t.kv = static_cast<const __half *>(kv_layer);
    t.page_table = page_table;
    t.pages_per_stream = pages_per_stream;
    t.row_slot = row_slot;
    t.row_pos = row_pos;
    t.plan = reinterpret_cast<int *>(ws + l.plan);
    t.R = R;
    t.part = reinterpret_cast<float *>(ws + l.part);
    t.out = out;
    return run_attention(t, reinterpret_cast<int *>(ws + l.work), reinterpret_cast<int4 *>(ws + l.desc),
                         l.groups * kHeads, static_cast<cudaStream_t>(cuda_stream), "attention_decode_paged");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free variant of mossgpu_attention_decode_paged.
//
// Some callers cannot allocate device memory at the moment they need attention: a real-time
// audio callback in a plugin host (cudaMalloc and cudaFree can block for milliseconds, and
// cudaFree synchronises the whole device), or a host program whose device memory is owned by
// another allocator that it may not go around.  For them the scratch this kernel needs (the
// split-K plan, the chunk counter and descriptors, the partial results) lives in the fixed array below,
// which the CUDA runtime creates on every GPU that loads this library and keeps until the
// process exits.
namespace {

constexpr int kNoAllocMaxRows = 256;     // rows per call
constexpr int kNoAllocMaxGroups = 341;   // split-K chunks (12 partials each); chunks widen to fit
constexpr size_t kNoAllocPlanBytes = 2048;                                    // 2 + R + 1 ints
constexpr size_t kNoAllocWorkBytes = 256;                                     // chunk counter
constexpr size_t kNoAllocDescBytes = 5632;                                    // chunk descriptors
constexpr size_t kNoAllocPartBytes = kGroupBytes * kNoAllocMaxGroups;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocPlanBytes + kNoAllocWorkBytes + kNoAllocDescBytes + kNoAllocPartBytes;  // ~1.07 MiB
static_assert(kNoAllocPlanBytes >= sizeof(int) * (kNoAllocMaxRows + 3), "plan area too small");
static_assert(kNoAllocDescBytes >= sizeof(int4) * kNoAllocMaxGroups, "descriptor area too small");
static_assert(kNoAllocMaxGroups >= kNoAllocMaxRows, "every row needs at least one chunk");

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array, looked up once per device (with that device current).  In host
// code the array's name is only a host-side handle, never a device address.
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return op_fail(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return op_fail("attention_decode_paged_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess || !p) return op_fail(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}

}  // namespace

extern "C" int mossgpu_attention_decode_paged_noalloc(const float *q, const void *kv_layer, const int32_t *page_table,
                                                      int pages_per_stream, const int32_t *row_slot,
                                                      const int32_t *row_pos, int R, float *out, void *cuda_stream) {
    using namespace mossgpu;
    if (R <= 0) return 0;
    if (R > kNoAllocMaxRows)
        return op_fail("attention_decode_paged_noalloc: R = " + std::to_string(R) + " rows exceeds the limit of " +
                       std::to_string(kNoAllocMaxRows) + " (use mossgpu_attention_decode_paged with a workspace)");
    if (!q || !kv_layer || !page_table || !row_slot || !row_pos || !out)
        return op_fail("attention_decode_paged_noalloc: a required pointer is NULL");
    if (pages_per_stream <= 0) return op_fail("attention_decode_paged_noalloc: pages_per_stream must be positive");
    if (check_alignment(q, kv_layer, "attention_decode_paged_noalloc") != 0) return 1;
    void *scratch = nullptr;
    if (noalloc_scratch(&scratch) != 0) return 1;
    char *base = static_cast<char *>(scratch);
    // every part of the array is rewritten before it is read: the plan kernel writes the plan
    // and descriptors and zeroes the chunk counter; partials are written before k_attn_combine
    AttnArgs t{};
    t.q = q;
    t.kv = static_cast<const __half *>(kv_layer);
    t.page_table = page_table;
    t.pages_per_stream = pages_per_stream;
    t.row_slot = row_slot;
    t.row_pos = row_pos;
    t.plan = reinterpret_cast<int *>(base);
    t.R = R;
    t.part = reinterpret_cast<float *>(base + kNoAllocPlanBytes + kNoAllocWorkBytes + kNoAllocDescBytes);
    t.out = out;
    return run_attention(t, reinterpret_cast<int *>(base + kNoAllocPlanBytes),
                         reinterpret_cast<int4 *>(base + kNoAllocPlanBytes + kNoAllocWorkBytes),
                         kNoAllocMaxGroups * kHeads, static_cast<cudaStream_t>(cuda_stream),
                         "attention_decode_paged_noalloc");
}
