// ops.cu -- standalone kernel-level C entry points over caller-owned device buffers.
//
// mossgpu_attention_decode_paged: the engine's paged fp16 flash-decode (one layer) for
// callers that keep their own KV pages, e.g. a host framework that manages the cache and
// only wants the attention kernel.  Every pointer is a device pointer; the caller also
// provides the scratch workspace (plan, split-K partials, arrival counters).
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

// The decode-attention kernel uses 205 KB of dynamic shared memory (its page ring), above the
// 48 KB a launch gets without opting in; the opt-in is per device.
constexpr int kMaxDevices = 64;
std::mutex g_attr_mu;
bool g_attr_set[kMaxDevices] = {};

int launch_decode(const mossgpu::AttnArgs &t, cudaStream_t st, const char *who) {
    using namespace mossgpu;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return op_fail(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return op_fail(std::string(who) + ": device ordinal out of range");
    {
        std::lock_guard<std::mutex> lock(g_attr_mu);
        if (!g_attr_set[dev]) {
            e = cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
            if (e != cudaSuccess) return op_fail(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
            g_attr_set[dev] = true;
        }
    }
    k_attn_decode<<<148, kAttnThreads, kAttnSmem, st>>>(t);
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

// Workspace layout for R rows: [plan: 2 + R + 1 ints][counters: R * 12 ints, chunk counter]
// [partials]
struct Layout {
    size_t plan, counters, part, total;
    int items;
};

Layout layout_for(int R, size_t bytes) {
    Layout l{};
    l.plan = 0;
    l.counters = round_up(sizeof(int) * (size_t(R) + 3));
    l.part = l.counters + round_up(sizeof(int) * (size_t(R) * mossgpu::kHeads + 1));
    const size_t part_bytes = bytes > l.part ? bytes - l.part : 0;
    l.items = int(std::min<size_t>(part_bytes / (sizeof(float) * mossgpu::kPartStride), 1u << 30));
    l.total = bytes;
    return l;
}

}  // namespace

extern "C" {

const char *mossgpu_op_last_error(void) { return g_op_error.c_str(); }

size_t mossgpu_attention_workspace_bytes(int R) {
    if (R <= 0) return 0;
    // room for 8 split-K chunks per (row, head); the plan widens chunks to fit any length
    const Layout l = layout_for(R, 0);
    return l.part + sizeof(float) * mossgpu::kPartStride * size_t(R) * mossgpu::kHeads * 8;
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
    if (l.items < R * kHeads)
        return op_fail("attention_decode_paged: workspace too small (need mossgpu_attention_workspace_bytes(R))");
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
        return op_fail("attention_decode_paged: workspace must be 16-byte aligned");
    if (check_alignment(q, kv_layer, "attention_decode_paged") != 0) return 1;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    char *ws = static_cast<char *>(workspace);
    int *plan = reinterpret_cast<int *>(ws + l.plan);
    int *counter = reinterpret_cast<int *>(ws + l.counters);
    float *part = reinterpret_cast<float *>(ws + l.part);
    // arrival counters must start at zero (the workspace's contents are unspecified)
    cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(int) * size_t(R) * kHeads, st);
    if (e != cudaSuccess) return op_fail(std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    k_attn_plan<<<1, 32, 0, st>>>(row_pos, R, l.items, plan, counter + R * kHeads, 1);
    AttnArgs t{};
    t.q = q;
    t.kv = static_cast<const __half *>(kv_layer);
    t.page_table = page_table;
    t.pages_per_stream = pages_per_stream;
    t.row_slot = row_slot;
    t.row_pos = row_pos;
    t.plan = plan;
    t.R = R;
    t.part = part;
    t.counter = counter;
    t.work = counter + R * kHeads;
    t.out = out;
    return launch_decode(t, st, "attention_decode_paged");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free variant of mossgpu_attention_decode_paged.
//
// Some callers cannot allocate device memory at the moment they need attention: a real-time
// audio callback in a plugin host (cudaMalloc and cudaFree can block for milliseconds, and
// cudaFree synchronises the whole device), or a host program whose device memory is owned by
// another allocator that it may not go around.  For them the scratch this kernel needs (the
// split-K plan, the arrival counters and the partial results) lives in the fixed array below,
// which the CUDA runtime creates on every GPU that loads this library and keeps until the
// process exits.
namespace {

constexpr int kNoAllocMaxRows = 256;    // rows per call
constexpr int kNoAllocMaxItems = 4096;  // split-K (chunk, head) partials; chunks widen to fit
constexpr size_t kNoAllocPlanBytes = 2048;                                   // 2 + R + 1 ints
constexpr size_t kNoAllocCounterBytes = sizeof(int) * kNoAllocMaxRows * mossgpu::kHeads + 256;  // + chunk counter
constexpr size_t kNoAllocPartBytes = sizeof(float) * mossgpu::kPartStride * kNoAllocMaxItems;
constexpr size_t kNoAllocScratchBytes = kNoAllocPlanBytes + kNoAllocCounterBytes + kNoAllocPartBytes;  // ~1.08 MiB
static_assert(kNoAllocPlanBytes >= sizeof(int) * (kNoAllocMaxRows + 3), "plan area too small");

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
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    char *base = static_cast<char *>(scratch);
    int *plan = reinterpret_cast<int *>(base);
    int *counter = reinterpret_cast<int *>(base + kNoAllocPlanBytes);
    float *part = reinterpret_cast<float *>(base + kNoAllocPlanBytes + kNoAllocCounterBytes);
    // the array keeps whatever the previous call left: the arrival counters must start at zero
    // (the plan is rewritten and the partials are written before they are read)
    cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(int) * size_t(R) * kHeads, st);
    if (e != cudaSuccess) return op_fail(std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    int *work = counter + kNoAllocMaxRows * kHeads;  // zeroed by the plan kernel
    k_attn_plan<<<1, 32, 0, st>>>(row_pos, R, kNoAllocMaxItems, plan, work, 1);
    AttnArgs t{};
    t.q = q;
    t.kv = static_cast<const __half *>(kv_layer);
    t.page_table = page_table;
    t.pages_per_stream = pages_per_stream;
    t.row_slot = row_slot;
    t.row_pos = row_pos;
    t.plan = plan;
    t.R = R;
    t.part = part;
    t.counter = counter;
    t.work = work;
    t.out = out;
    return launch_decode(t, st, "attention_decode_paged_noalloc");
}
