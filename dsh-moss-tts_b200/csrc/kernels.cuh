// kernels.cuh -- sm_100a kernels for the MOSS-TTS-Nano per-frame LLM step.
//
// Work is expressed over a "row batch": R rows, row r = (stream slot, position).  A decode
// step is one row per stream; a prefill is one row per prompt position.  Every kernel reads
// its per-row data (slot, position, frame index, forced codes) from device memory, so the
// whole frame can be captured once per batch size and replayed as a CUDA graph.
//
// Data layout in HBM (see engine.cu for allocation):
//   weights  Q8_0_4X4 split into two planes per matrix (engine.cu: repack kernel):
//              qs [R/4][K/32][4][32] int8   (the file's 128 quant bytes of each block)
//              sc [R/4][K/32][4]     fp16   (the file's 8 scale bytes of each block)
//   KV       fp16 pages of 16 positions: [layer][page][k|v][head][16][64]
//   local KV fp32 [slot][k|v][17][768]
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "types.h"

namespace mossgpu {
// Internal linkage: every translation unit that launches these kernels (engine.cu, ops.cu)
// compiles its own copy, so no host stub is defined twice.
namespace {

// --------------------------------------------------------------------------- helpers

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Residual accumulators of the small-batch layers (layer_small.cuh): int64 in units of 2^-32,
// summed with integer atomics so that the result does not depend on the order of the adds.
__device__ __forceinline__ long long float_to_fixed(float v) { return __double2ll_rn((double)v * 4294967296.0); }
__device__ __forceinline__ float fixed_to_float(long long s) { return (float)((double)s * (1.0 / 4294967296.0)); }

__device__ __forceinline__ int4 ldg_stream(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch.  Kernels of a frame are launched so that each may start
// while its predecessor is still running: work that only touches weights goes before
// pdl_wait(); pdl_wait() returns once the predecessor grid has completed and its writes are
// visible; pdl_trigger() then lets the successor grid start its own prologue.  Launched
// without the attribute, both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
    pdl_wait();
    pdl_trigger();
}

// ---- shared-memory barriers and bulk copies (cp.async.bulk, no tensor map, no multicast)

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done)
                 : "r"(addr), "r"(parity)
                 : "memory");
    return done != 0;
}

// Bounded wait for the phase with the given parity: try_wait (which suspends the thread in
// hardware for a while) in a tight loop, then 1 us sleeps until about a second has passed.
// Returns false, and records `code` in *err when err is not null, on time-out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    const uint32_t addr = smem_u32(bar);
    for (int it = 0; it < 4096; ++it)
        if (mbar_try(addr, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try(addr, parity)) return true;
        if (global_ns() - t0 > 1000000000ull) break;
        __nanosleep(1000);
    }
    if (err) atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// xoshiro128** step and uniform draw of the reference sampler (sampler.h:25-48), on a
// stream's state in global memory; one thread per stream draws.
__device__ __forceinline__ uint32_t rng_rotl(uint32_t x, int k) { return (x << k) | (x >> (32 - k)); }
__device__ __forceinline__ float rng_uniform(uint32_t *st) {
    uint32_t s0 = st[0], s1 = st[1], s2 = st[2], s3 = st[3];
    const uint32_t result = rng_rotl(s1 * 5u, 7) * 9u;
    const uint32_t t = s1 << 9;
    s2 ^= s0;
    s3 ^= s1;
    s1 ^= s2;
    s0 ^= s3;
    s2 ^= t;
    s3 = rng_rotl(s3, 11);
    st[0] = s0;
    st[1] = s1;
    st[2] = s2;
    st[3] = s3;
    return (float)(result >> 8) * (1.0f / 16777216.0f);
}

// gelu_new (llm.cpp:22-25), same operation order
__device__ __forceinline__ float gelu_new(float v) {
    const float k = 0.7978845608028654f;
    const float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(__fmul_rn(k, __fadd_rn(v, c)))));
}

// 16 int8 -> 16 floats, exact, without integer-to-float conversions (a slow pipe): byte b with
// its sign bit flipped is b + 128 as an unsigned byte; placed as the low mantissa byte of 2^23
// (0x4B000000) it reads as 8388608 + (b + 128), and subtracting 8388736 leaves b.
__device__ __forceinline__ void unpack16(const int4 q, float *w) {
    const uint32_t words[4] = {(uint32_t)q.x ^ 0x80808080u, (uint32_t)q.y ^ 0x80808080u, (uint32_t)q.z ^ 0x80808080u,
                               (uint32_t)q.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[4 * i + j] = __uint_as_float(__byte_perm(words[i], 0x4B000000u, 0x7540u | j)) - 8388736.0f;
    }
}

// LayerNorm of one 768-vector held in shared memory, in place, by one warp (llm.cpp:159-171).
__device__ __forceinline__ void warp_layernorm(float *x, const float *w, const float *b) {
    const int lane = threadIdx.x & 31;
    float s = 0.f;
    for (int i = lane; i < kHidden; i += 32) s += x[i];
    const float mean = __fdiv_rn(warp_sum(s), (float)kHidden);
    float v = 0.f;
    for (int i = lane; i < kHidden; i += 32) {
        const float d = x[i] - mean;
        v = fmaf(d, d, v);
    }
    const float var = __fdiv_rn(warp_sum(v), (float)kHidden);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(var + 1e-5f));
    __syncwarp();
    for (int i = lane; i < kHidden; i += 32)
        x[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[i], mean), inv), w[i]), b[i]);
}

// --------------------------------------------------------------------------- weights repack

// Split Q8_0_4X4 file bytes (136-byte blocks: 8 scale bytes + 128 quant bytes) into the
// 16-byte-aligned quant plane and the scale plane.  A pure byte permutation.
__global__ void k_repack_q8x4(const uint8_t *__restrict__ src, int8_t *__restrict__ qs, __half *__restrict__ sc,
                              long long nblocks) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8-byte word
    const long long words = nblocks * 17;
    if (t >= words) return;
    const long long blk = t / 17;
    const int w = (int)(t - blk * 17);
    const uint8_t *s = src + blk * 136 + w * 8;  // 8-byte aligned: 136 = 17 * 8
    const uint2 v = *reinterpret_cast<const uint2 *>(s);
    if (w == 0) {
        *reinterpret_cast<uint2 *>(sc + blk * 4) = v;
    } else {
        *reinterpret_cast<uint2 *>(qs + blk * 128 + (w - 1) * 8) = v;
    }
}

// --------------------------------------------------------------------------- GEMV

enum { PRO_NONE = 0, PRO_LN = 1 };
enum { EPI_STORE = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GELU = 3 };

struct GemvArgs {
    QMat w;
    const float *bias;     // [rows] or null
    const float *x;        // input rows [R][ldx]
    int ldx;
    const float *ln_w, *ln_b;
    int nrows;             // R
    int ks;                // K slices per group (warps per group)
    int gpc;               // groups per CTA
    float *out;            // EPI_STORE/GELU: [R][ldo]; EPI_RESID: residual [R][ldo] (in place)
    int ldo;
    // EPI_QKV
    float *q_out;          // [R][768]
    __half *kv;            // paged global KV for this layer (layer offset applied)
    const int *page_table; // [slots][pages_per_stream]
    int pages_per_stream;
    float *lkv;            // local KV [slots][2][17][768] (when kv == null)
    const int *row_slot;
    const int *row_pos;    // position used for RoPE and the KV write (null: fixed_pos)
    int fixed_pos;         // local decoder: the local position of every row
    const float2 *rope;    // [max_ctx][32] (cos, sin)
};

// y[r][row] = sum_k W[row][k] * x'[r][k], x' = LN(x) or x, W in Q8_0_4X4 (fp32 math, A16).
// A warp owns one (group of 4 rows, K slice); lane l always reads row (l%8)/2, half l%2 of
// each 32-column block, so a warp's loads are 512 contiguous bytes.
template <int PRO, int EPI, int MAXR>
__global__ void __launch_bounds__(512) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(16) float smem[];
    const int K = a.w.cols;
    const int nb = K >> 5;
    const int r0 = blockIdx.y * MAXR;
    const int nr = min(MAXR, a.nrows - r0);
    float *xs = smem;                      // [MAXR][K]
    float *red = smem + MAXR * K;          // [warps][4][MAXR]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    const int gl = warp / a.ks, slice = warp - gl * a.ks;
    const int g = blockIdx.x * a.gpc + gl;
    const int ngroups = a.w.rows >> 2;
    const int bps = nb / a.ks;              // blocks per slice
    const int k = (lane & 7) >> 1, h = lane & 1;
    const bool active = gl < a.gpc && g < ngroups;
    const int8_t *wq = a.w.qs + ((size_t)g * nb + (size_t)slice * bps) * 128;
    const __half *ws = a.w.sc + ((size_t)g * nb + (size_t)slice * bps) * 4;
    const int nchunks = bps * 8;

    // 0. this lane's first two weight chunks and scales: static data, fetched before waiting
    //    for the kernel that produces x, so the HBM latency overlaps it
    int4 pq0 = make_int4(0, 0, 0, 0), pq1 = make_int4(0, 0, 0, 0);
    float pd0 = 0.f, pd1 = 0.f;
    if (active && lane < nchunks) {
        pq0 = ldg_stream(wq + (size_t)lane * 16);
        pd0 = __half2float(ws[(lane >> 3) * 4 + k]);
    }
    if (active && lane + 32 < nchunks) {
        pq1 = ldg_stream(wq + (size_t)(lane + 32) * 16);
        pd1 = __half2float(ws[((lane + 32) >> 3) * 4 + k]);
    }
    pdl_enter();

    // 1. stage the input rows (and LayerNorm them) in shared memory
    for (int i = tid; i < nr * (K >> 2); i += blockDim.x) {
        const int r = i / (K >> 2), c = i - r * (K >> 2);
        reinterpret_cast<float4 *>(xs + r * K)[c] =
            reinterpret_cast<const float4 *>(a.x + (size_t)(r0 + r) * a.ldx)[c];
    }
    __syncthreads();
    if (PRO == PRO_LN) {
        for (int r = warp; r < nr; r += nwarps) warp_layernorm(xs + r * K, a.ln_w, a.ln_b);
        __syncthreads();
    }

    // 2. dot products
    float acc[MAXR];
#pragma unroll
    for (int r = 0; r < MAXR; ++r) acc[r] = 0.f;
    if (active) {
        for (int i = lane; i < nchunks; i += 64) {
            int4 q0 = pq0, q1 = pq1;
            float d0 = pd0, d1 = pd1;
            const bool two = i + 32 < nchunks;
            if (i != lane) {  // chunks beyond the prefetched pair
                q0 = ldg_stream(wq + (size_t)i * 16);
                d0 = __half2float(ws[(i >> 3) * 4 + k]);
                if (two) {
                    q1 = ldg_stream(wq + (size_t)(i + 32) * 16);
                    d1 = __half2float(ws[((i + 32) >> 3) * 4 + k]);
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                if (u == 1 && !two) break;
                const int ii = i + 32 * u;
                const int b = ii >> 3;
                const float d = u ? d1 : d0;
                float wf[16];
                unpack16(u ? q1 : q0, wf);
                const int xoff = (slice * bps + b) * 32 + h * 16;
#pragma unroll
                for (int r = 0; r < MAXR; ++r) {
                    if (r < nr) {
                        const float4 *xv = reinterpret_cast<const float4 *>(xs + r * K + xoff);
                        float s = 0.f;
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float4 xx = xv[t];
                            s = fmaf(wf[4 * t + 0], xx.x, s);
                            s = fmaf(wf[4 * t + 1], xx.y, s);
                            s = fmaf(wf[4 * t + 2], xx.z, s);
                            s = fmaf(wf[4 * t + 3], xx.w, s);
                        }
                        acc[r] = fmaf(s, d, acc[r]);
                    }
                }
            }
        }
    }
    // reduce the 8 lanes that share row k (xor over h and lane/8)
#pragma unroll
    for (int r = 0; r < MAXR; ++r) {
        float v = acc[r];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        acc[r] = v;
    }
    if (lane < 8 && (lane & 1) == 0) {
#pragma unroll
        for (int r = 0; r < MAXR; ++r) red[(warp * 4 + (lane >> 1)) * MAXR + r] = acc[r];
    }
    __syncthreads();

    // 3. epilogue: thread (gl, k, r) sums the K slices of its output
    float *fin = red + nwarps * 4 * MAXR;   // [gpc][4][MAXR]
    for (int t = tid; t < a.gpc * 4 * MAXR; t += blockDim.x) {
        const int egl = t / (4 * MAXR);
        const int ek = (t / MAXR) & 3;
        const int er = t % MAXR;
        float v = 0.f;
        for (int s = 0; s < a.ks; ++s) v += red[((egl * a.ks + s) * 4 + ek) * MAXR + er];
        fin[t] = v;
    }
    __syncthreads();
    for (int t = tid; t < a.gpc * 4 * MAXR; t += blockDim.x) {
        const int egl = t / (4 * MAXR);
        const int ek = (t / MAXR) & 3;
        const int er = t % MAXR;
        const int eg = blockIdx.x * a.gpc + egl;
        if (er >= nr || eg >= ngroups) continue;
        const int row = eg * 4 + ek;
        const int rr = r0 + er;
        float v = fin[t];
        if (EPI == EPI_STORE) {
            if (a.bias) v = __fadd_rn(v, a.bias[row]);
            a.out[(size_t)rr * a.ldo + row] = v;
        } else if (EPI == EPI_GELU) {
            a.out[(size_t)rr * a.ldo + row] = gelu_new(__fadd_rn(v, a.bias[row]));
        } else if (EPI == EPI_RESID) {
            float *o = a.out + (size_t)rr * a.ldo + row;
            *o = __fadd_rn(*o, __fadd_rn(v, a.bias[row]));
        } else {  // EPI_QKV: bias, RoPE on q and k (pairs 2i,2i+1 share a 4-row group), KV append
            if (ek & 1) continue;  // the even row of each pair writes both rows
            const float v0 = __fadd_rn(v, a.bias[row]);
            const float v1 = __fadd_rn(fin[t + MAXR], a.bias[row + 1]);
            const int pos = a.row_pos ? a.row_pos[rr] : a.fixed_pos;
            float o0 = v0, o1 = v1;
            if (row < 2 * kHidden) {
                const int i = (row % kHeadDim) >> 1;
                const float2 cs = a.rope[(size_t)pos * (kHeadDim / 2) + i];
                o0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
                o1 = __fadd_rn(__fmul_rn(v1, cs.x), __fmul_rn(v0, cs.y));
            }
            if (row < kHidden) {
                a.q_out[(size_t)rr * kHidden + row] = o0;
                a.q_out[(size_t)rr * kHidden + row + 1] = o1;
            } else {
                const int kvsel = row < 2 * kHidden ? 0 : 1;
                const int c = row - kHidden * (1 + kvsel);
                const int slot = a.row_slot[rr];
                if (a.kv) {
                    const int page = a.page_table[(size_t)slot * a.pages_per_stream + pos / kPage];
                    __half *dst = a.kv + (size_t)page * kPageHalfs +
                                  ((kvsel * kHeads + c / kHeadDim) * kPage + pos % kPage) * kHeadDim + (c % kHeadDim);
                    *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(o0, o1);
                } else {
                    float *dst = a.lkv + (((size_t)slot * 2 + kvsel) * kLocalLen + pos) * kHidden + c;
                    dst[0] = o0;
                    dst[1] = o1;
                }
            }
        }
    }
}

// --------------------------------------------------------------------------- attention

// Split-K plan over the row batch: row r attends to n_r = pos_r + 1 positions, cut into
// chunks of `chunk` positions (whole pages).  plan[0] = chunk, plan[1] = total chunks,
// plan[2 + r] = first chunk of row r (R + 1 entries).  The chunk is the smallest power-of-two
// multiple of kAttnChunk keeping chunks * heads within `max_items` (the partial-result
// capacity).  desc[g] describes chunk g for the decode kernel: {row | split << 30, first
// position, end position, page-table offset of the first page}, split = the row has more
// than one chunk.  One CTA of kPlanThreads threads; it also zeroes the decode kernel's work
// counters.
__global__ void __launch_bounds__(kPlanThreads) k_attn_plan(const int *__restrict__ row_pos, const int *__restrict__ row_slot,
                                                        int pages_per_stream, int R, int max_items, int *__restrict__ plan,
                                                        int4 *__restrict__ desc, int *__restrict__ work, int nwork) {
    pdl_enter();
    __shared__ long long red_t[kPlanThreads / 32];
    __shared__ int red_i[kPlanThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    constexpr int NW = kPlanThreads / 32;
    for (int i = tid; i < nwork; i += kPlanThreads) work[i] = 0;
    // chunk length: kAttnChunk doubled until all rows' chunks x 12 heads fit max_items
    int chunk = kAttnChunk;
    for (;;) {
        long long t = 0;
        for (int r = tid; r < R; r += kPlanThreads) t += max(0, row_pos[r] + chunk) / chunk;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0) red_t[wid] = t;
        __syncthreads();
        long long tot = 0;
#pragma unroll
        for (int w = 0; w < NW; ++w) tot += red_t[w];
        __syncthreads();  // red_t is rewritten by the next iteration
        if (tot * kHeads <= max_items || chunk >= (1 << 20)) break;
        chunk *= 2;
    }
    // rows in tiles of kPlanThreads: exclusive prefix sum of the chunk counts (warp scans, then
    // the warp totals), one thread writes its row's chunk descriptors
    int acc = 0;
    for (int b = 0; b < R; b += kPlanThreads) {
        const int r = b + tid;
        const int n = r < R ? row_pos[r] + 1 : 0;
        const int v = max(0, n - 1 + chunk) / chunk;  // rows with pos < 0 have no chunk
        int inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) red_i[wid] = inc;
        __syncthreads();
        int before = 0, total = 0;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const int x = red_i[w];
            before += w < wid ? x : 0;
            total += x;
        }
        __syncthreads();  // red_i is rewritten by the next tile
        const int g0 = acc + before + inc - v;
        if (r < R) {
            plan[2 + r] = g0;
            const int base = row_slot[r] * pages_per_stream;
            for (int c = 0; c < v; ++c) {
                const int p0 = c * chunk;
                desc[g0 + c] = make_int4(r | ((v > 1) << 30), p0, min(n, p0 + chunk), base + p0 / kPage);
            }
        }
        acc += total;
    }
    if (tid == 0) {
        plan[0] = chunk;
        plan[1] = acc;
        plan[2 + R] = acc;
    }
}

struct AttnArgs {
    const float *q;         // [R][768], 16-byte aligned
    const __half *kv;       // layer base of the paged KV, 16-byte aligned
    const int *page_table;
    int pages_per_stream;
    const int *row_slot, *row_pos;
    const int *plan;        // from k_attn_plan
    const int4 *desc;       // chunk descriptors from k_attn_plan
    int R;
    float *part;            // [chunks * 12][kPartStride] partials: m, l, pad, pad, o[64]
    int *work;              // next chunk to hand out; zeroed by k_attn_plan
    float *out;             // [R][768]
    // tensor-core path: write the output straight into the next GEMM's fp16 activation image
    // (bimg_parts = 1: fp16; 2: fp16 and fp16 remainder) instead of `out`
    uint8_t *bimg;
    int bimg_N, bimg_parts;
    int *err;               // bounded-wait time-out flag (may be null)
    // Fault injection for the time-out test (may be null; 0 = off): when *inject != 0 the
    // producer leaves the first ring stage it fills unfilled -- no copy issued, no arrival --
    // so the consumers' bounded wait on it runs out.  Nothing is in flight on that stage.
    const int *inject;
};

// byte offset of element (n, k) in a tensor-core activation image with N rows: the
// SWIZZLE_128B K-major layout [k/64][n][128 B], 16-byte unit (k%64)/8 stored at unit ^ (n%8)
__device__ __forceinline__ size_t bimg_off(int n, int k, int N) {
    return ((size_t)(k >> 6) * N + n) * 128 + ((((k & 63) >> 3) ^ (n & 7)) << 4) + ((k & 7) << 1);
}

// One row n of an activation image, written by one warp: lane l holds the 8-element units l,
// l + 32, l + 64 of the row in v; optional LayerNorm (llm.cpp:159-171: warp-reduced mean and
// variance), then the fp16 value and (parts = 2) the fp16 of its remainder per element.
constexpr int kBimgRowUnits = kHidden / 256;
__device__ __forceinline__ void bimg_row_write(float (&v)[kBimgRowUnits][8], int lane, int n, int N,
                                               const float *__restrict__ ln_w, const float *__restrict__ ln_b,
                                               int parts, uint8_t *__restrict__ bimg) {
    if (ln_w) {
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < kBimgRowUnits; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) sum += v[j][e];
        const float mean = __fdiv_rn(warp_sum(sum), (float)kHidden);
        float var = 0.f;
#pragma unroll
        for (int j = 0; j < kBimgRowUnits; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float d = v[j][e] - mean;
                var = fmaf(d, d, var);
            }
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(warp_sum(var), (float)kHidden) + 1e-5f));
#pragma unroll
        for (int j = 0; j < kBimgRowUnits; ++j) {
            const int k0 = 8 * (lane + 32 * j);
            const float4 w0 = *reinterpret_cast<const float4 *>(ln_w + k0), w1 = *reinterpret_cast<const float4 *>(ln_w + k0 + 4);
            const float4 c0 = *reinterpret_cast<const float4 *>(ln_b + k0), c1 = *reinterpret_cast<const float4 *>(ln_b + k0 + 4);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            const float bv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e)
                v[j][e] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j][e], mean), inv), wv[e]), bv[e]);
        }
    }
    const size_t part = (size_t)kHidden * N * 2;
#pragma unroll
    for (int j = 0; j < kBimgRowUnits; ++j) {
        __align__(16) __half h[8];
        __align__(16) __half l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            h[e] = __float2half_rn(v[j][e]);
            l[e] = __float2half_rn(v[j][e] - __half2float(h[e]));
        }
        const size_t off = bimg_off(n, 8 * (lane + 32 * j), N);
        *reinterpret_cast<int4 *>(bimg + off) = *reinterpret_cast<const int4 *>(h);
        if (parts == 2) *reinterpret_cast<int4 *>(bimg + part + off) = *reinterpret_cast<const int4 *>(l);
    }
}

// Store 8 consecutive output dims (one lane's share of a head) of row r.
__device__ __forceinline__ void attn_store8(const AttnArgs &a, int r, int k0, const float *y) {
    if (a.bimg) {  // 8 dims = one 16-byte unit of the activation image
        __align__(16) __half h[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            h[j] = __float2half_rn(y[j]);
            lo[j] = __float2half_rn(y[j] - __half2float(h[j]));
        }
        const size_t off = bimg_off(r, k0, a.bimg_N);
        *reinterpret_cast<int4 *>(a.bimg + off) = *reinterpret_cast<const int4 *>(h);
        if (a.bimg_parts == 2)
            *reinterpret_cast<int4 *>(a.bimg + (size_t)kHidden * a.bimg_N * 2 + off) = *reinterpret_cast<const int4 *>(lo);
    } else {
        float *dst = a.out + (size_t)r * kHidden + k0;
        reinterpret_cast<float4 *>(dst)[0] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4 *>(dst)[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
}

// Flash-decode over fp16 pages, one CTA per SM.  A page of one layer holds K and V of all 12
// heads for 16 positions, 48 KB contiguous ([k|v][head][16][64] fp16), so the whole page
// moves with one cp.async.bulk.  A producer warp claims chunks (whole pages of one row,
// described by k_attn_plan) from an atomic counter, one chunk ahead, and streams their pages
// -- with the row's query on the chunk's first page -- into a 4-stage ring in shared memory;
// 12 consumer warps, one per head, read their head's 2 KB K and V blocks from a stage (8 lanes
// per position, 8 dims a lane, 4 positions per step, online softmax in fp32) and release it.
// At the end of a chunk a warp writes its (row, head) result, or, for a row split into several
// chunks, a partial that k_attn_combine merges.  Every barrier wait is bounded.
constexpr int kAttnConsumers = kHeads;                     // consumer warps: one per head
constexpr int kAttnThreads = (kAttnConsumers + 1) * 32;    // + the producer warp
constexpr int kAttnStages = 4;
constexpr int kAttnPageBytes = kPageHalfs * 2;             // 49152
constexpr int kAttnQBytes = kHidden * 4;                   // one query row, fp32
constexpr int kAttnSmem = kAttnStages * (kAttnPageBytes + kAttnQBytes) + 1024;  // 209,920

struct AttnStage {  // written by the producer before the stage's barrier arrive
    int r;          // row
    int pb;         // first position of the page
    int p1;         // end of the chunk (exclusive)
    int flags;      // 1: first page of a chunk (query copied), 2: last page, 4: no more work,
                    // 8: the row is split (write a partial)
    int g;          // chunk index (its partials live at g * 12 + head)
    int pad[3];
};

__global__ void __launch_bounds__(kAttnThreads, 1) k_attn_decode(const AttnArgs a) {
    extern __shared__ __align__(128) uint8_t attn_smem[];
    uint8_t *pages = attn_smem;                                          // [stage][49152]
    float *qs = reinterpret_cast<float *>(attn_smem + kAttnStages * kAttnPageBytes);  // [stage][768]
    AttnStage *meta = reinterpret_cast<AttnStage *>(attn_smem + kAttnStages * (kAttnPageBytes + kAttnQBytes));
    uint64_t *full = reinterpret_cast<uint64_t *>(meta + kAttnStages);  // [stage]
    uint64_t *empty = full + kAttnStages;                               // [stage]
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kAttnStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAttnConsumers);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_enter();
    const int total = a.plan[1];

    if (wid == kAttnConsumers) {
        // ------------------------------------------------------------------ producer warp
        int seq = 0;
        bool ok = true;
        int g = 0;
        const bool inject = a.inject != nullptr && *a.inject != 0;
        if (lane == 0) g = atomicAdd(a.work, 1);
        g = __shfl_sync(0xffffffffu, g, 0);
        int4 d = g < total ? a.desc[g] : make_int4(0, 0, 0, 0);
        for (;;) {
            const bool stop = g >= total;
            int gn = 0;
            if (!stop && lane == 0) gn = atomicAdd(a.work, 1);  // claim the next chunk now
            const int r = d.x & 0x3fffffff, split = d.x >> 30, p0 = d.y, p1 = d.z;
            const int npg = stop ? 1 : (p1 - p0 + kPage - 1) / kPage;
            for (int jb = 0; jb < npg && ok; jb += 32) {
                const int pid = (!stop && jb + lane < npg) ? a.page_table[d.w + jb + lane] : 0;
                const int jend = min(npg, jb + 32);
                for (int j = jb; j < jend; ++j) {
                    const int page = __shfl_sync(0xffffffffu, pid, j - jb);
                    if (lane == 0) {
                        const int s = seq % kAttnStages;
                        if (!mbar_wait(&empty[s], ((seq / kAttnStages) & 1) ^ 1, a.err, 8)) {
                            ok = false;
                        } else if (inject && seq == 0 && !stop) {
                            // fault injection: this stage stays unfilled (see AttnArgs::inject)
                        } else {
                            AttnStage &m = meta[s];
                            m.r = r;
                            m.pb = p0 + j * kPage;
                            m.p1 = p1;
                            m.flags = stop ? 4 : ((j == 0 ? 1 : 0) | (j == npg - 1 ? 2 : 0) | (split ? 8 : 0));
                            m.g = g;
                            if (stop) {
                                mbar_arrive(&full[s]);
                            } else {
                                mbar_expect_tx(&full[s], kAttnPageBytes + (j == 0 ? kAttnQBytes : 0));
                                bulk_g2s(pages + (size_t)s * kAttnPageBytes, a.kv + (size_t)page * kPageHalfs,
                                         kAttnPageBytes, &full[s]);
                                if (j == 0)
                                    bulk_g2s(qs + s * kHidden, a.q + (size_t)r * kHidden, kAttnQBytes, &full[s]);
                            }
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    ++seq;
                    if (!ok) break;
                }
            }
            if (stop || !ok) break;
            g = __shfl_sync(0xffffffffu, gn, 0);
            d = g < total ? a.desc[g] : make_int4(0, 0, 0, 0);
        }
        if ((!ok || inject) && lane == 0) {
            // the consumers may have stopped waiting (a time-out): let every copy this warp
            // issued land before the CTA exits.  The stage that failed its wait (when !ok)
            // and the injected unfilled stage issued nothing and are skipped.
            const int issued = ok ? seq : seq - 1;
            for (int k = max(0, issued - kAttnStages); k < issued; ++k)
                if (!(inject && k == 0)) mbar_wait(&full[k % kAttnStages], (k / kAttnStages) & 1, nullptr, 0);
        }
        return;
    }

    // ---------------------------------------------------------------------- consumer warps
    const int hd = wid;
    const int ps = lane >> 3, ds = lane & 7;
    float qv[8];
    float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.f;
    for (int seq = 0;; ++seq) {
        const int s = seq % kAttnStages;
        if (!mbar_wait(&full[s], (seq / kAttnStages) & 1, a.err, 7)) return;
        const AttnStage st = meta[s];
        if (st.flags & 4) break;
        if (st.flags & 1) {
            const float4 *qp = reinterpret_cast<const float4 *>(qs + s * kHidden + hd * kHeadDim + ds * 8);
            const float4 x0 = qp[0], x1 = qp[1];
            qv[0] = x0.x * 0.125f; qv[1] = x0.y * 0.125f; qv[2] = x0.z * 0.125f; qv[3] = x0.w * 0.125f;
            qv[4] = x1.x * 0.125f; qv[5] = x1.y * 0.125f; qv[6] = x1.z * 0.125f; qv[7] = x1.w * 0.125f;
        }
        const uint8_t *kb = pages + (size_t)s * kAttnPageBytes + hd * (kPage * kHeadDim * 2) + ds * 16;
        const uint8_t *vb = kb + kHeads * kPage * kHeadDim * 2;
        float sc[4];
        int4 vr[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int pp = ps + 4 * u;  // position within the page
            const int4 kr = *reinterpret_cast<const int4 *>(kb + pp * 128);
            vr[u] = *reinterpret_cast<const int4 *>(vb + pp * 128);
            if (st.pb + pp >= st.p1) vr[u] = make_int4(0, 0, 0, 0);  // past the end: stale bits
            const __half2 *kh = reinterpret_cast<const __half2 *>(&kr);
            float dd = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(kh[e]);
                dd = fmaf(qv[2 * e], kf.x, dd);
                dd = fmaf(qv[2 * e + 1], kf.y, dd);
            }
            sc[u] = dd;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // the stage's data is in registers now
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 1);
            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 2);
            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 4);
            if (st.pb + ps + 4 * u >= st.p1) sc[u] = -INFINITY;
        }
        const float mn = fmaxf(fmaxf(m, fmaxf(sc[0], sc[1])), fmaxf(sc[2], sc[3]));
        if (mn != -INFINITY) {  // else: no valid position for this lane group yet
            const float corr = __expf(m - mn);
            float pw[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) pw[u] = __expf(sc[u] - mn);  // 0 for -inf scores
            l = l * corr + ((pw[0] + pw[1]) + (pw[2] + pw[3]));
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] *= corr;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const __half2 *vh = reinterpret_cast<const __half2 *>(&vr[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 vf = __half22float2(vh[e]);
                    o[2 * e] = fmaf(pw[u], vf.x, o[2 * e]);
                    o[2 * e + 1] = fmaf(pw[u], vf.y, o[2 * e + 1]);
                }
            }
            m = mn;
        }
        if (!(st.flags & 2)) continue;

        // ---- end of the chunk: merge the 4 position groups (lanes ds, ds+8, ds+16, ds+24)
#pragma unroll
        for (int off = 8; off <= 16; off <<= 1) {
            const float mo = __shfl_xor_sync(0xffffffffu, m, off);
            const float lo2 = __shfl_xor_sync(0xffffffffu, l, off);
            const float mx = fmaxf(m, mo);
            const float c1 = (m == -INFINITY) ? 0.f : __expf(m - mx);
            const float c2 = (mo == -INFINITY) ? 0.f : __expf(mo - mx);
            l = l * c1 + lo2 * c2;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float oo = __shfl_xor_sync(0xffffffffu, o[j], off);
                o[j] = o[j] * c1 + oo * c2;
            }
            m = mx;
        }
        if (lane < 8) {
            if (st.flags & 8) {  // split row: partial (m, l, unnormalised o) for k_attn_combine
                float *pp = a.part + ((size_t)st.g * kHeads + hd) * kPartStride;
                reinterpret_cast<float4 *>(pp + 4 + ds * 8)[0] = make_float4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<float4 *>(pp + 4 + ds * 8)[1] = make_float4(o[4], o[5], o[6], o[7]);
                if (lane == 0) *reinterpret_cast<float2 *>(pp) = make_float2(m, l);
            } else {
                const float inv = 1.f / l;
                float y[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) y[j] = o[j] * inv;
                attn_store8(a, st.r, hd * kHeadDim + ds * 8, y);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = 0.f;
        m = -INFINITY;
        l = 0.f;
    }
}

// Merge the split-K partials of every (row, head) whose row was split into several chunks:
// out = sum_c exp(m_c - M) o_c / sum_c exp(m_c - M) l_c.  One warp per (row, head); lane i
// owns dims 8 (i % 8) .. +7 of chunks i / 8, i / 8 + 4, ...
__global__ void __launch_bounds__(256) k_attn_combine(const AttnArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (w >= a.R * kHeads) return;
    const int r = w / kHeads, hd = w - r * kHeads;
    const int g0 = a.plan[2 + r], nch = a.plan[3 + r] - g0;
    if (nch <= 1) return;
    const float *base = a.part + ((size_t)g0 * kHeads + hd) * kPartStride;
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, __ldcg(base + (size_t)c * kHeads * kPartStride));
    M = warp_max(M);
    const int cg = lane >> 3, ds = lane & 7;
    float L = 0.f, y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = 0.f;
    for (int c = cg; c < nch; c += 4) {
        const float *q = base + (size_t)c * kHeads * kPartStride;
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(q));
        const float4 o0 = __ldcg(reinterpret_cast<const float4 *>(q + 4 + ds * 8));
        const float4 o1 = __ldcg(reinterpret_cast<const float4 *>(q + 4 + ds * 8) + 1);
        const float wgt = ml.x == -INFINITY ? 0.f : __expf(ml.x - M);
        L = fmaf(ml.y, wgt, L);
        y[0] = fmaf(o0.x, wgt, y[0]); y[1] = fmaf(o0.y, wgt, y[1]);
        y[2] = fmaf(o0.z, wgt, y[2]); y[3] = fmaf(o0.w, wgt, y[3]);
        y[4] = fmaf(o1.x, wgt, y[4]); y[5] = fmaf(o1.y, wgt, y[5]);
        y[6] = fmaf(o1.z, wgt, y[6]); y[7] = fmaf(o1.w, wgt, y[7]);
    }
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {
        L += __shfl_xor_sync(0xffffffffu, L, off);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] += __shfl_xor_sync(0xffffffffu, y[j], off);
    }
    if (lane < 8) {
        const float inv = 1.f / L;
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] *= inv;
        attn_store8(a, r, hd * kHeadDim + ds * 8, y);
    }
}

// Decode attention for small batches (the CUDA-core path, <= 8 rows): one CTA per (row, head),
// its 16 warps taking the row's pages round-robin (warp w: pages w, w + 16, ...), each with
// the lane layout and online softmax of k_attn_decode (8 lanes per position, 8 dims a lane, 4
// positions a step); the warps' partial (max, sum, output) merge in shared memory.  One launch
// per layer and no plan: the split-K path needs three (plan, decode, combine), which at one
// row is latency, not bandwidth.
constexpr int kArWarps = 16;
__global__ void __launch_bounds__(kArWarps * 32) k_attn_rows(const float *__restrict__ q, const __half *__restrict__ kv,
                                                            const int *__restrict__ page_table, int pages_per_stream,
                                                            const int *__restrict__ row_slot, const int *__restrict__ row_pos,
                                                            float *__restrict__ out, uint8_t *__restrict__ bimg, int bimg_N,
                                                            int bimg_parts) {
    __shared__ float sm_m[kArWarps], sm_l[kArWarps];
    __shared__ __align__(16) float sm_o[kArWarps][kHeadDim];
    pdl_enter();
    const int r = blockIdx.x / kHeads, hd = blockIdx.x % kHeads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ps = lane >> 3, ds = lane & 7;
    const int n = row_pos[r] + 1;  // positions 0 .. pos
    const int npg = (n + kPage - 1) / kPage;
    const int slot = row_slot[r];
    float qv[8];
    {
        const float4 *qp = reinterpret_cast<const float4 *>(q + (size_t)r * kHidden + hd * kHeadDim + ds * 8);
        const float4 x0 = qp[0], x1 = qp[1];
        qv[0] = x0.x * 0.125f; qv[1] = x0.y * 0.125f; qv[2] = x0.z * 0.125f; qv[3] = x0.w * 0.125f;
        qv[4] = x1.x * 0.125f; qv[5] = x1.y * 0.125f; qv[6] = x1.z * 0.125f; qv[7] = x1.w * 0.125f;
    }
    float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.f;
    // the page-table entry of a warp's next page is fetched one iteration ahead, so that each
    // iteration waits on one memory round trip (the K/V loads) instead of two
    const int *pt = page_table + (size_t)slot * pages_per_stream;
    int page_next = warp < npg ? pt[warp] : 0;
    for (int pg = warp; pg < npg; pg += kArWarps) {
        const int page = page_next;
        if (pg + kArWarps < npg) page_next = pt[pg + kArWarps];
        const __half *kb = kv + (size_t)page * kPageHalfs + (size_t)hd * kPage * kHeadDim + ds * 8;
        const __half *vb = kb + (size_t)kHeads * kPage * kHeadDim;
        const int pb = pg * kPage;
        int4 kr[4], vr[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int pp = ps + 4 * u;
            kr[u] = *reinterpret_cast<const int4 *>(kb + pp * kHeadDim);
            vr[u] = *reinterpret_cast<const int4 *>(vb + pp * kHeadDim);
            if (pb + pp >= n) vr[u] = make_int4(0, 0, 0, 0);  // past the row's end: stale bits
        }
        float sc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const __half2 *kh = reinterpret_cast<const __half2 *>(&kr[u]);
            float dd = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(kh[e]);
                dd = fmaf(qv[2 * e], kf.x, dd);
                dd = fmaf(qv[2 * e + 1], kf.y, dd);
            }
            sc[u] = dd;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 1);
            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 2);
            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 4);
            if (pb + ps + 4 * u >= n) sc[u] = -INFINITY;
        }
        const float mn = fmaxf(fmaxf(m, fmaxf(sc[0], sc[1])), fmaxf(sc[2], sc[3]));
        if (mn != -INFINITY) {
            const float corr = __expf(m - mn);
            float pw[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) pw[u] = __expf(sc[u] - mn);
            l = l * corr + ((pw[0] + pw[1]) + (pw[2] + pw[3]));
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] *= corr;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const __half2 *vh = reinterpret_cast<const __half2 *>(&vr[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 vf = __half22float2(vh[e]);
                    o[2 * e] = fmaf(pw[u], vf.x, o[2 * e]);
                    o[2 * e + 1] = fmaf(pw[u], vf.y, o[2 * e + 1]);
                }
            }
            m = mn;
        }
    }
    // merge the 4 position groups of the warp (lanes ds, ds + 8, ds + 16, ds + 24)
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, off);
        const float lo2 = __shfl_xor_sync(0xffffffffu, l, off);
        const float mx = fmaxf(m, mo);
        const float c1 = (m == -INFINITY) ? 0.f : __expf(m - mx);
        const float c2 = (mo == -INFINITY) ? 0.f : __expf(mo - mx);
        l = l * c1 + lo2 * c2;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float oo = __shfl_xor_sync(0xffffffffu, o[j], off);
            o[j] = o[j] * c1 + oo * c2;
        }
        m = mx;
    }
    if (lane < 8) {
        if (lane == 0) {
            sm_m[warp] = m;
            sm_l[warp] = l;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) sm_o[warp][ds * 8 + j] = o[j];
    }
    __syncthreads();
    // merge the warps (a warp without pages has m = -inf and weighs nothing)
    if (threadIdx.x < kHeadDim) {
        const int d = threadIdx.x;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kArWarps; ++w) M = fmaxf(M, sm_m[w]);
        float L = 0.f, y = 0.f;
#pragma unroll
        for (int w = 0; w < kArWarps; ++w) {
            const float wgt = sm_m[w] == -INFINITY ? 0.f : __expf(sm_m[w] - M);
            L = fmaf(sm_l[w], wgt, L);
            y = fmaf(sm_o[w][d], wgt, y);
        }
        const float res = y / L;
        if (bimg) {  // the tensor-core path: straight into the proj GEMM's activation image
            const __half h = __float2half_rn(res);
            const size_t off = bimg_off(r, hd * kHeadDim + d, bimg_N);
            *reinterpret_cast<__half *>(bimg + off) = h;
            if (bimg_parts == 2)
                *reinterpret_cast<__half *>(bimg + (size_t)kHidden * bimg_N * 2 + off) = __float2half_rn(res - __half2float(h));
        } else {
            out[(size_t)r * kHidden + hd * kHeadDim + d] = res;
        }
    }
}

// Local decoder attention: n = lpos + 1 <= 17 positions of fp32 local KV.
// One warp per (row, head); scores in llm.cpp:189-217 order per position.  With bimg set the
// output goes straight into the next tensor-core GEMM's activation image (N rows, parts).
__global__ void __launch_bounds__(384) k_attn_local(const float *__restrict__ q, const float *__restrict__ lkv,
                                                    const int *__restrict__ row_slot, int lpos, int R,
                                                    float *__restrict__ out, uint8_t *__restrict__ bimg, int bimg_N,
                                                    int bimg_parts) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (w >= R * kHeads) return;
    const int r = w / kHeads, hd = w - r * kHeads;
    const int slot = row_slot[r];
    const int n = lpos + 1;
    const float *kb = lkv + ((size_t)slot * 2 + 0) * kLocalLen * kHidden + hd * kHeadDim;
    const float *vb = lkv + ((size_t)slot * 2 + 1) * kLocalLen * kHidden + hd * kHeadDim;
    const float *qh = q + (size_t)r * kHidden + hd * kHeadDim;
    float s = -INFINITY;
    if (lane < n) {
        float dot = 0.f;
        const float4 *kp = reinterpret_cast<const float4 *>(kb + (size_t)lane * kHidden);
        const float4 *qp = reinterpret_cast<const float4 *>(qh);
#pragma unroll
        for (int d = 0; d < kHeadDim / 4; ++d) {
            const float4 kk = kp[d], qq = qp[d];
            dot = fmaf(qq.x, kk.x, dot);
            dot = fmaf(qq.y, kk.y, dot);
            dot = fmaf(qq.z, kk.z, dot);
            dot = fmaf(qq.w, kk.w, dot);
        }
        s = dot * 0.125f;
    }
    const float mx = warp_max(s);
    const float e = lane < n ? expf(s - mx) : 0.f;
    const float sum = warp_sum(e);
    const float wgt = e * (1.0f / sum);
    float o0 = 0.f, o1 = 0.f;
    for (int p = 0; p < n; ++p) {
        const float wp = __shfl_sync(0xffffffffu, wgt, p);
        const float2 vv = reinterpret_cast<const float2 *>(vb + (size_t)p * kHidden)[lane];
        o0 = fmaf(wp, vv.x, o0);
        o1 = fmaf(wp, vv.y, o1);
    }
    if (bimg) {
        const __half2 hv = __floats2half2_rn(o0, o1);
        const size_t off = bimg_off(r, hd * kHeadDim + 2 * lane, bimg_N);
        *reinterpret_cast<__half2 *>(bimg + off) = hv;
        if (bimg_parts == 2)
            *reinterpret_cast<__half2 *>(bimg + (size_t)kHidden * bimg_N * 2 + off) =
                __floats2half2_rn(o0 - __low2float(hv), o1 - __high2float(hv));
    } else {
        reinterpret_cast<float2 *>(out + (size_t)r * kHidden + hd * kHeadDim)[lane] = make_float2(o0, o1);
    }
}

// --------------------------------------------------------------------------- embeddings

__device__ __forceinline__ float deq_elem(const QMat &m, int row, int col) {
    const int nb = m.cols >> 5;
    const size_t blk = (size_t)(row >> 2) * nb + (col >> 5);
    const float d = __half2float(m.sc[blk * 4 + (row & 3)]);
    return d * (float)m.qs[blk * 128 + (row & 3) * 32 + (col & 31)];
}



// x[r] = deq(wte[row[0]]) + sum_ch deq(aemb[ch][row[ch+1]]) over valid codes (llm.cpp:148-157)
__global__ void k_embed_rows(const EmbedTables t, const int *__restrict__ rows17, int R, float *__restrict__ x) {
    pdl_enter();
    const int r = blockIdx.x;
    if (r >= R) return;
    const int *row = rows17 + (size_t)r * (kNVq + 1);
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) {
        float v = deq_elem(t.wte, row[0], c);
        for (int ch = 0; ch < kNVq; ++ch) {
            const int code = row[ch + 1];
            if (code == kAudioPad || code < 0 || code >= kCodebook) continue;
            v = __fadd_rn(v, deq_elem(t.aemb[ch], code, c));
        }
        x[(size_t)r * kHidden + c] = v;
    }
}

// Global-step input from the codes the local decoder used: row = [9, used codes...]
__global__ void k_embed_frame(const EmbedTables t, const int *__restrict__ used, int R, float *__restrict__ x) {
    pdl_enter();
    const int r = blockIdx.x;
    if (r >= R) return;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) {
        float v = deq_elem(t.wte, kSlotToken, c);
        for (int ch = 0; ch < kNVq; ++ch) {
            const int code = used[r * kNVq + ch];
            if (code == kAudioPad || code < 0 || code >= kCodebook) continue;
            v = __fadd_rn(v, deq_elem(t.aemb[ch], code, c));
        }
        x[(size_t)r * kHidden + c] = v;
    }
}

// lx[r] = deq(wte[row]) (local step 1 input: the slot token row, llm.cpp:682)
__global__ void k_lookup_rows(const QMat m, int row, int R, float *__restrict__ x) {
    pdl_enter();
    const int r = blockIdx.x;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) x[(size_t)r * kHidden + c] = deq_elem(m, row, c);
}

// --------------------------------------------------------------------------- LayerNorm / commit

// out[r] = LN(x[r]) for rows whose commit flag is set (all rows when commit is null);
// also copies the result to out2[r] when given.
// xfix (nullable): the rows come from the int64 residual accumulators of the small-batch
// layers (2^-32 units) instead of x
__global__ void k_layernorm_rows(const float *__restrict__ x, int R, const float *__restrict__ w,
                                 const float *__restrict__ b, float *__restrict__ out, const int *__restrict__ out_index,
                                 const int *__restrict__ commit, const long long *__restrict__ xfix) {
    __shared__ float xs[kHidden];
    pdl_enter();
    const int r = blockIdx.x;
    if (r >= R) return;
    if (commit && !commit[r]) return;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x)
        xs[c] = xfix ? fixed_to_float(xfix[(size_t)r * kHidden + c]) : x[(size_t)r * kHidden + c];
    __syncthreads();
    if (threadIdx.x < 32) warp_layernorm(xs, w, b);
    __syncthreads();
    const int dst = out_index ? out_index[r] : r;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) out[(size_t)dst * kHidden + c] = xs[c];
}

// out[dst[i]] = LayerNorm(x[src[i]]) for i < n: the ln_f of the rows that end their streams
// in a prefill pass, in one launch (llm.cpp:395-399)
__global__ void k_layernorm_pick(const float *__restrict__ x, const int *__restrict__ src, const int *__restrict__ dst,
                                 int n, const float *__restrict__ w, const float *__restrict__ b, float *__restrict__ out) {
    __shared__ float xs[kHidden];
    pdl_enter();
    const int i = blockIdx.x;
    if (i >= n) return;
    const float *row = x + (size_t)src[i] * kHidden;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) xs[c] = row[c];
    __syncthreads();
    if (threadIdx.x < 32) warp_layernorm(xs, w, b);
    __syncthreads();
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) out[(size_t)dst[i] * kHidden + c] = xs[c];
}

// gather rows: dst[r] = src[index[r]]
__global__ void k_gather_rows(const float *__restrict__ src, const int *__restrict__ index, int R, float *__restrict__ dst) {
    pdl_enter();
    const int r = blockIdx.x;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) dst[(size_t)r * kHidden + c] = src[(size_t)index[r] * kHidden + c];
}

// --------------------------------------------------------------------------- end gate



// AVX2 horizontal sum tree of the reference (gemv_avx2.cpp:24-31)
__device__ __forceinline__ float hsum8(const float *v) {
    const float s0 = __fadd_rn(v[0], v[4]), s1 = __fadd_rn(v[1], v[5]);
    const float s2 = __fadd_rn(v[2], v[6]), s3 = __fadd_rn(v[3], v[7]);
    return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}

// W8A8 two-row gate on LN(lx) (llm.cpp:274-315, quant.cpp:28-54, gemv_avx2.cpp:105-121), in
// the reference's exact arithmetic order; sets active[r] = 0 when generation ends.
__global__ void __launch_bounds__(256) k_gate(const float *__restrict__ lx, int R, const float *__restrict__ ln_w,
                                              const float *__restrict__ ln_b, const QMat wte,
                                              const int *__restrict__ frame_idx, const FrameCtl *__restrict__ ctl,
                                              const int *__restrict__ active_in, int *__restrict__ active,
                                              float *__restrict__ gate_out, const int *__restrict__ row_slot,
                                              uint32_t *__restrict__ rng) {
    __shared__ float xs[kHidden];
    __shared__ int8_t qa[kHidden];
    __shared__ float as[kHidden / 32];
    __shared__ float pair[2];
    pdl_enter();
    const int r = blockIdx.x;
    for (int c = threadIdx.x; c < kHidden; c += blockDim.x) xs[c] = lx[(size_t)r * kHidden + c];
    __syncthreads();
    if (threadIdx.x < 32) warp_layernorm(xs, ln_w, ln_b);
    __syncthreads();
    if (threadIdx.x < kHidden / 32) {
        const int b = threadIdx.x;
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) {
            const float v = fabsf(xs[b * 32 + i]);
            amax = (amax < v) ? v : amax;
        }
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
        as[b] = d;
        for (int i = 0; i < 32; ++i) {
            int q = __float2int_rn(__fmul_rn(xs[b * 32 + i], id));
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            qa[b * 32 + i] = (int8_t)q;
        }
    }
    __syncthreads();
    if (threadIdx.x < 2) {
        const int row = threadIdx.x == 0 ? kEndToken : kSlotToken;
        const int nb = kHidden / 32;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int b = 0; b < nb; ++b) {
            const size_t blk = (size_t)(row >> 2) * nb + b;
            const float dw = __half2float(wte.sc[blk * 4 + (row & 3)]);
            const int8_t *qs = wte.qs + blk * 128 + (row & 3) * 32;
            const float s = __fmul_rn(dw, as[b]);
            for (int j = 0; j < 8; ++j) {
                int p = 0;
                for (int i = 4 * j; i < 4 * j + 4; ++i) p += (int)qs[i] * (int)qa[b * 32 + i];
                acc[j] = fmaf((float)p, s, acc[j]);
            }
        }
        pair[threadIdx.x] = hsum8(acc);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float l_end = pair[0], l_slot = pair[1];
        if (gate_out) {
            gate_out[2 * r] = l_end;
            gate_out[2 * r + 1] = l_slot;
        }
        // end_reached (llm.cpp:30-35): greedy compare, or one draw against p(slot) =
        // 1 / (1 + e^(l_end - l_slot)) computed in double with the difference clamped to +-80
        bool stop = false;
        if (active_in[r] && frame_idx[r] >= ctl->min_frames) {
            if (ctl->end_greedy) {
                stop = l_end > l_slot;
            } else {
                double d = (double)l_end - (double)l_slot;
                d = d < -80.0 ? -80.0 : (d > 80.0 ? 80.0 : d);
                const float p_slot = (float)(1.0 / (1.0 + exp(d)));
                stop = rng_uniform(rng + (size_t)row_slot[r] * 4) >= p_slot;
            }
        }
        active[r] = (active_in[r] && !stop) ? 1 : 0;  // a stream that stopped stays stopped
    }
}

// End of a frame: record this frame's codes (-1 for streams that are not active), then
// advance each active stream's position and frame index and carry its active flag to the
// next frame of the same call.  One CTA, so the frame counter moves after every read of it.
__global__ void __launch_bounds__(256) k_frame_commit(const int *__restrict__ codes, const int *__restrict__ active,
                                                      int R, int run_global, int *__restrict__ pos,
                                                      int *__restrict__ frame_idx, int *__restrict__ active_in,
                                                      int *__restrict__ fslot, int max_frames,
                                                      int *__restrict__ codes_hist) {
    pdl_enter();
    const int f = *fslot;
    if (f < max_frames) {
        for (int i = threadIdx.x; i < R * kNVq; i += blockDim.x)
            codes_hist[((size_t)f * R) * kNVq + i] = active[i / kNVq] ? codes[i] : -1;
    }
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        const int a = active[r];
        if (a) {
            frame_idx[r] += 1;
            if (run_global) pos[r] += 1;
        }
        active_in[r] = a;
    }
    if (threadIdx.x == 0) *fslot = f + 1;
}

// --------------------------------------------------------------------------- sampler

// Greedy code choice with the reference's repetition penalty (sampler.cpp:9-28): the penalty
// is applied once per earlier occurrence of the code on this channel, then the first index
// of the maximum wins.  Then records the used code (forced or predicted), counts it, and
// writes the next local-decoder input deq(aemb[ch][used]) (llm.cpp:686-698).
// sample_token (sampler.cpp:9-77) for channel ch of every row, one CTA per row: the
// repetition penalty once per earlier occurrence (counts), then either the first maximum
// (greedy, top_k == 1, or frame < greedy_frames), or temperature, a sort by (value desc,
// index asc), top-k, exp / sum in that order, the top-p cut and one xoshiro128** draw walked
// down the sorted list.  Writes the prediction, the code used (forced or predicted), the
// counts update and the next local input row aemb[ch][used]; with img != null also that row's
// LayerNorm activation image (the next local step's LN1, as k_build_bimg writes it), so that
// the next step starts at its QKV GEMM.
struct NextImage {
    const float *ln_w = nullptr, *ln_b = nullptr;
    uint8_t *bimg = nullptr;
    int N = 0, parts = 0;
};
__global__ void __launch_bounds__(256) k_sample(const float *__restrict__ logits, int ld_logits, int ch,
                                                const int *__restrict__ row_slot, int R,
                                                uint16_t *__restrict__ counts, const FrameCtl *__restrict__ ctl,
                                                const int *__restrict__ forced, const int *__restrict__ active,
                                                int *__restrict__ codes_out, int *__restrict__ used_out,
                                                const QMat aemb, float *__restrict__ next_x,
                                                const int *__restrict__ frame_idx, uint32_t *__restrict__ rng,
                                                NextImage img) {
    __shared__ float sv[kCodebook];
    __shared__ int si[kCodebook];
    __shared__ float bv[8];
    __shared__ int bi[8];
    __shared__ int s_pred, s_used;
    pdl_enter();
    const int r = blockIdx.x;
    const int slot = row_slot[r];
    const float *lg = logits + (size_t)r * ld_logits;
    uint16_t *cnt = counts + ((size_t)slot * kNVq + ch) * kCodebook;
    const float p = ctl->rep_penalty;
    const bool greedy = ctl->greedy || ctl->top_k == 1 || frame_idx[r] < ctl->greedy_frames;
    for (int t = threadIdx.x; t < kCodebook; t += blockDim.x) {
        float v = lg[t];
        if (p != 1.0f) {
            const int c = cnt[t];
            for (int j = 0; j < c; ++j) v = v < 0.f ? __fmul_rn(v, p) : __fdiv_rn(v, p);
        }
        sv[t] = v;
        si[t] = t;
    }
    if (greedy) {
        float best = -INFINITY;
        int besti = 0x7fffffff;
        for (int t = threadIdx.x; t < kCodebook; t += blockDim.x) {
            const float v = sv[t];
            if (v > best || (v == best && t < besti)) { best = v; besti = t; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
            if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
        }
        const int warp = threadIdx.x >> 5;
        if ((threadIdx.x & 31) == 0) { bv[warp] = best; bi[warp] = besti; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
                if (bv[w] > best || (bv[w] == best && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
            // all-NaN logits compare false everywhere: code 0, as the reference's first-max
            // scan (best index starts at 0) returns
            s_pred = besti < kCodebook ? besti : 0;
        }
    } else {
        const float temp = ctl->temperature;
        if (temp > 0.0f && temp != 1.0f) {
            const float inv = __fdiv_rn(1.0f, temp);
            for (int t = threadIdx.x; t < kCodebook; t += blockDim.x) sv[t] = __fmul_rn(sv[t], inv);
        }
        __syncthreads();
        // bitonic sort of (value, index): "before" = larger value, or equal value and lower index
        for (int k = 2; k <= kCodebook; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int i = threadIdx.x; i < kCodebook; i += blockDim.x) {
                    const int ixj = i ^ j;
                    if (ixj > i) {
                        const float va = sv[i], vb = sv[ixj];
                        const int ia = si[i], ib = si[ixj];
                        const bool a_first = va > vb || (va == vb && ia < ib);
                        if (((i & k) == 0) ? !a_first : a_first) {
                            sv[i] = vb;
                            sv[ixj] = va;
                            si[i] = ib;
                            si[ixj] = ia;
                        }
                    }
                }
                __syncthreads();
            }
        }
        if (threadIdx.x == 0) {  // the reference's sequential sums, in sorted order
            const int kk = ctl->top_k > 0 ? (ctl->top_k < kCodebook ? ctl->top_k : kCodebook) : kCodebook;
            int size = kk;
            const float maxv = sv[0];
            float sum = 0.0f;
            for (int j = 0; j < size; ++j) {
                const float e = expf(sv[j] - maxv);
                sv[j] = e;
                sum += e;
            }
            if (ctl->top_p < 1.0f) {
                float cum = 0.0f;
                int keep = 0;
                for (; keep < size; ++keep) {
                    cum += sv[keep] / sum;
                    if (cum >= ctl->top_p) {
                        ++keep;
                        break;
                    }
                }
                size = keep > 1 ? keep : 1;
                sum = 0.0f;
                for (int j = 0; j < size; ++j) sum += sv[j];
            }
            int out = si[size - 1];
            if (active[r]) {  // a stream that stopped draws nothing more
                float rr = rng_uniform(rng + (size_t)slot * 4) * sum;
                for (int j = 0; j < size; ++j) {
                    rr -= sv[j];
                    if (rr <= 0.0f) {
                        out = si[j];
                        break;
                    }
                }
            }
            s_pred = out;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int pred = s_pred;
        const int used = ctl->has_forced ? forced[r * kNVq + ch] : pred;
        codes_out[r * kNVq + ch] = pred;
        used_out[r * kNVq + ch] = used;
        if (active[r] && used >= 0 && used < kCodebook) cnt[used] = (uint16_t)(cnt[used] + 1);
        s_used = used;
    }
    __syncthreads();
    if (next_x && img.bimg) {
        // warp 0: the row in k_build_bimg's lane layout (units l, l + 32, l + 64), to x and image
        if (threadIdx.x < 32) {
            const int used = s_used, lane = threadIdx.x;
            const bool ok = used >= 0 && used < kCodebook;
            float v[kBimgRowUnits][8];
#pragma unroll
            for (int j = 0; j < kBimgRowUnits; ++j) {
                const int k0 = 8 * (lane + 32 * j);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[j][e] = ok ? deq_elem(aemb, used, k0 + e) : 0.f;
                float4 *xp = reinterpret_cast<float4 *>(next_x + (size_t)r * kHidden + k0);
                xp[0] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
                xp[1] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
            }
            bimg_row_write(v, lane, r, img.N, img.ln_w, img.ln_b, img.parts, img.bimg);
        }
    } else if (next_x) {
        const int used = s_used;
        for (int c = threadIdx.x; c < kHidden; c += blockDim.x)
            next_x[(size_t)r * kHidden + c] = (used >= 0 && used < kCodebook) ? deq_elem(aemb, used, c) : 0.f;
    }
}

// scatter page-table updates: upd = [count][slot, index, page] x count;
// table[slot * pps + index] = page
__global__ void k_page_updates(const int *__restrict__ upd, int *__restrict__ table, int pps) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < upd[0]) table[(size_t)upd[1 + 3 * i] * pps + upd[2 + 3 * i]] = upd[3 + 3 * i];
}

}  // namespace
}  // namespace mossgpu
