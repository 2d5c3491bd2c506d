// step_small.cuh -- the 12 global layers for a small row batch (R <= 8) as ONE persistent
// kernel (llm.cpp:230-246 per layer, llm.cpp:248-255 for the step).
//
// At a handful of rows every kernel of the layer-by-layer path is latency bound (a launch,
// one round of loads, a short dot product), so the step is ~75 dependent launches of a few
// microseconds each.  Here one cooperative launch of 148 CTAs (one per SM) walks all 12
// layers; the dependencies become counters in global memory that CTAs wait on (bounded):
//
//   phase A (per layer; 12 teams of 12 CTAs, team h = attention head h)
//     A1  x (the input, or the previous layer's residual sum) -> LN1, in shared memory
//     A2  the 192 QKV rows of head h (its q, k and v features): bias, RoPE, q to scratch,
//         k and v appended to the fp16 KV page                          -> team sync 1
//     A3  decode attention of head h, one warp per (row, chunk of pages) -> team sync 2
//     A4  merge the chunks; the head's share of proj: W_proj[:, 64h..64h+63] . attn_h,
//         added into the residual accumulator (team 0 also adds x and the bias)
//                                                                        -> grid sync
//   phase B (96 CTAs: CTA b owns fc_in features 32b..32b+31)
//     B1  residual sum -> x -> LN2
//     B2  fc_in rows of the CTA: bias, GELU
//     B3  its share of fc_out: W_fc_out[:, 32b..32b+31] . gelu, added into the next
//         residual accumulator (CTA 0 also adds x and the bias)           -> grid sync
//
// Data written inside the launch (q, the new KV position, partials, accumulators) is read
// with L2-only loads after the counter that publishes it.
// Residual accumulators are fixed point (int64, 2^-32 units): partial sums from many CTAs add
// exactly and in any order, so the result does not depend on timing.  All weights are
// prefetched into L2 at the start (85 MB of the 126 MB L2), so every phase after the first
// reads them from L2.  Waits spin on acquire loads with a ~1 s bound; on time-out the kernel
// records a code in err and every CTA returns.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "kernels.cuh"
#include "types.h"

namespace mossgpu {
namespace {

constexpr int kSmallMaxR = 8;         // rows per launch
constexpr int kStepCtas = 148;        // one per SM (cooperative launch)
constexpr int kStepThreads = 512;     // 16 warps
constexpr int kTeamCtas = 12;         // phase A CTAs per head
constexpr int kFcCtas = kFF / 32;     // 96 phase B CTAs
constexpr int kStepMaxChunks = 16;    // attention chunks per (row, head)
constexpr int kStepSyncs = 1 + kLayers * kHeads * 2;  // grid counter + team counters

struct StepLayer {
    const int8_t *attn_qs, *proj_qs, *fcin_qs, *fcout_qs;
    const __half *attn_sc, *proj_sc, *fcin_sc, *fcout_sc;
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    const float *attn_b, *proj_b, *fcin_b, *fcout_b;
};

struct StepArgs {
    const StepLayer *layers;      // [12], device memory
    __half *kv;                   // paged KV, layer 0
    size_t layer_halfs;           // halfs per layer of the KV pool
    const int *page_table;
    int pages_per_stream;
    const int *row_slot, *row_pos;
    int R;
    const float2 *rope;           // [max_ctx][32]
    float *x;                     // [R][768]: input embeddings in, final residual stream out
    float *q;                     // [R][768] scratch
    float *apart;                 // [12][R][16][kPartStride] attention partials
    unsigned long long *acc;      // [12][2][R][768] residual accumulators, zero at launch
    unsigned *sync;               // [kStepSyncs], zero at launch
    int *err;
    size_t weight_bytes[4 * 2];   // per layer: qs and sc bytes of attn, proj, fc_in, fc_out
};

__device__ __forceinline__ long long to_fix(float v) { return __float2ll_rn(v * 4294967296.0f); }
__device__ __forceinline__ float from_fix(unsigned long long v) {
    return __ll2float_rn((long long)v) * 2.3283064365386963e-10f;  // 2^-32
}
__device__ __forceinline__ void add_fix(unsigned long long *p, float v) {
    atomicAdd(p, (unsigned long long)to_fix(v));
}

// CTA-wide: every thread's writes are published, one count is added to *ctr, and the CTA
// waits until *ctr >= target.  Returns false on time-out (error code recorded).
__device__ bool step_sync(unsigned *ctr, unsigned target, int *err, int code) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
        int ok = 1;
        const uint64_t t0 = global_ns();
        for (int it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
            if (v >= target) break;
            if ((it & 15) == 15 && global_ns() - t0 > 1000000000ull) {
                atomicCAS(err, 0, code);
                ok = 0;
                break;
            }
        }
        __threadfence();
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    // the slice [p, p + bytes) of a weight buffer; p and bytes multiples of 16
    const char *c = static_cast<const char *>(p);
    while (bytes > 0) {
        const uint32_t n = bytes > 65536 ? 65536u : (uint32_t)bytes;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
        c += n;
        bytes -= n;
    }
}

// this CTA's 1/148 share of a buffer, in 16-byte units
__device__ __forceinline__ void prefetch_share(const void *p, size_t bytes) {
    const size_t units = bytes >> 4;
    const size_t u0 = units * blockIdx.x / kStepCtas, u1 = units * (blockIdx.x + 1) / kStepCtas;
    if (u1 > u0) prefetch_l2(static_cast<const char *>(p) + (u0 << 4), (u1 - u0) << 4);
}

// One warp: partial dot products of a 4-row group of a Q8_0_4X4 plane matrix with nr rows of
// xs ([r][K] in shared memory), over the K blocks [b0, b0 + nbk).  Lane l reads 16 bytes of
// row (l % 8) / 2, half l % 2 of each 32-column block (the engine's GEMV lane layout).  On
// return lanes 0, 2, 4, 6 hold the sums of rows 0..3 in acc[r].
__device__ __forceinline__ void warp_group_dot(const int8_t *qs, const __half *sc, int nb, int g, int b0, int nbk,
                                               const float *xs, int K, int nr, float acc[kSmallMaxR]) {
    const int lane = threadIdx.x & 31;
    const int k = (lane & 7) >> 1, h = lane & 1;
    const int8_t *wq = qs + ((size_t)g * nb + b0) * 128;
    const __half *ws = sc + ((size_t)g * nb + b0) * 4;
#pragma unroll
    for (int r = 0; r < kSmallMaxR; ++r) acc[r] = 0.f;
    const int nchunks = nbk * 8;
    for (int i = lane; i < nchunks; i += 32) {
        const int4 q = ldg_stream(wq + (size_t)i * 16);
        const float d = __half2float(ws[(i >> 3) * 4 + k]);
        float wf[16];
        unpack16(q, wf);
        const int xoff = (b0 + (i >> 3)) * 32 + h * 16;
#pragma unroll
        for (int r = 0; r < kSmallMaxR; ++r) {
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
#pragma unroll
    for (int r = 0; r < kSmallMaxR; ++r) {
        float v = acc[r];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        acc[r] = v;
    }
}

// x rows from the input (layer 0) or from a residual accumulator, then LayerNorm into xl
__device__ void step_load_ln(const StepArgs &a, const unsigned long long *acc, const float *ln_w, const float *ln_b,
                             float *xraw, float *xl) {
    const int R = a.R;
    for (int i = threadIdx.x; i < R * kHidden; i += blockDim.x) {
        const float v = acc ? from_fix(__ldcg(acc + i)) : a.x[i];  // written in this launch: L2 only
        xraw[i] = v;
        xl[i] = v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    if (warp < R) warp_layernorm(xl + warp * kHidden, ln_w, ln_b);
    __syncthreads();
}

__global__ void __launch_bounds__(kStepThreads, 1) k_global_step_small(const StepArgs a) {
    extern __shared__ __align__(16) float sm[];
    float *xraw = sm;                                 // [R][768]
    float *xl = xraw + kSmallMaxR * kHidden;          // [R][768] LayerNormed
    float *red = xl + kSmallMaxR * kHidden;           // [16 warps][4][R]
    float *attn = red + 16 * 4 * kSmallMaxR;          // [R][64]
    float *gel = attn + kSmallMaxR * kHeadDim;        // [R][32]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int R = a.R;
    const int cta = blockIdx.x;
    const bool in_a = cta < kHeads * kTeamCtas;
    const int team = cta / kTeamCtas, tc = cta % kTeamCtas;  // phase A: head and rank in the team
    const bool in_b = cta < kFcCtas;
    const size_t racc = (size_t)R * kHidden;          // one accumulator

    // every CTA streams its share of all weights into L2, layer by layer
    if (tid == 0) {
        for (int l = 0; l < kLayers; ++l) {
            const StepLayer &L = a.layers[l];
            prefetch_share(L.attn_qs, a.weight_bytes[0]);
            prefetch_share(L.attn_sc, a.weight_bytes[1]);
            prefetch_share(L.proj_qs, a.weight_bytes[2]);
            prefetch_share(L.proj_sc, a.weight_bytes[3]);
            prefetch_share(L.fcin_qs, a.weight_bytes[4]);
            prefetch_share(L.fcin_sc, a.weight_bytes[5]);
            prefetch_share(L.fcout_qs, a.weight_bytes[6]);
            prefetch_share(L.fcout_sc, a.weight_bytes[7]);
        }
    }
    unsigned grid_target = 0;

    for (int l = 0; l < kLayers; ++l) {
        const StepLayer &L = a.layers[l];
        unsigned long long *acc_p = a.acc + (size_t)l * 2 * racc;  // after proj
        unsigned long long *acc_f = acc_p + racc;                   // after fc_out
        const unsigned long long *acc_in = l ? a.acc + ((size_t)(l - 1) * 2 + 1) * racc : nullptr;
        __half *kvl = a.kv + (size_t)l * a.layer_halfs;

        // ============================== phase A
        if (in_a) {
            const int h = team;
            step_load_ln(a, acc_in, L.ln1_w, L.ln1_b, xraw, xl);
            // A2: team-group tg = 4 tc + warp / 4 (q, k, v blocks of 16 groups), K slice warp % 4
            {
                const int tg = 4 * tc + (warp >> 2), slice = warp & 3;
                const int g = (tg / 16) * (kHidden / 4) + 16 * h + (tg % 16);
                float acc[kSmallMaxR];
                warp_group_dot(L.attn_qs, L.attn_sc, kHidden / 32, g, slice * 6, 6, xl, kHidden, R, acc);
                if (lane < 8 && (lane & 1) == 0)
#pragma unroll
                    for (int r = 0; r < kSmallMaxR; ++r) red[(warp * 4 + (lane >> 1)) * kSmallMaxR + r] = acc[r];
                __syncthreads();
                // 4 groups x 2 row pairs x R rows: bias, RoPE, q out / KV append
                for (int t = tid; t < 4 * 2 * R; t += blockDim.x) {
                    const int gl = t / (2 * R), pr = (t / R) & 1, r = t % R;
                    float y[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float v = 0.f;
                        for (int s = 0; s < 4; ++s) v += red[((gl * 4 + s) * 4 + 2 * pr + e) * kSmallMaxR + r];
                        y[e] = v;
                    }
                    const int tgl = 4 * tc + gl;
                    const int gg = (tgl / 16) * (kHidden / 4) + 16 * h + (tgl % 16);
                    const int gm = gg * 4 + 2 * pr;  // even row of the pair
                    const float yb = __fadd_rn(y[0], L.attn_b[gm]), other = __fadd_rn(y[1], L.attn_b[gm + 1]);
                    const int pos = a.row_pos[r];
                    float o0 = yb, o1 = other;
                    if (gm < 2 * kHidden) {
                        const float2 cs = a.rope[(size_t)pos * (kHeadDim / 2) + ((gm % kHeadDim) >> 1)];
                        o0 = __fsub_rn(__fmul_rn(yb, cs.x), __fmul_rn(other, cs.y));
                        o1 = __fadd_rn(__fmul_rn(other, cs.x), __fmul_rn(yb, cs.y));
                    }
                    if (gm < kHidden) {
                        *reinterpret_cast<float2 *>(a.q + (size_t)r * kHidden + gm) = make_float2(o0, o1);
                    } else {
                        const int kvsel = gm < 2 * kHidden ? 0 : 1;
                        const int c = gm - kHidden * (1 + kvsel);
                        const int page = a.page_table[(size_t)a.row_slot[r] * a.pages_per_stream + pos / kPage];
                        __half *dst = kvl + (size_t)page * kPageHalfs +
                                      ((kvsel * kHeads + c / kHeadDim) * kPage + pos % kPage) * kHeadDim + (c % kHeadDim);
                        *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(o0, o1);
                    }
                }
            }
            unsigned *ts = a.sync + 1 + (l * kHeads + h) * 2;
            if (!step_sync(ts, kTeamCtas, a.err, 11)) return;

            // A3: one warp per (row, chunk); <= 16 chunks of whole pages per row
            {
                const int tw = tc * 16 + warp;
                int item = tw, r = 0, npg = 0, pc = 1, nch = 0;
                for (r = 0; r < R; ++r) {
                    npg = (a.row_pos[r] + kPage) / kPage;
                    pc = (npg + kStepMaxChunks - 1) / kStepMaxChunks;
                    nch = (npg + pc - 1) / pc;
                    if (item < nch) break;
                    item -= nch;
                }
                if (r < R) {
                    const int n = a.row_pos[r] + 1;
                    const int pg0 = item * pc, pg1 = min(npg, pg0 + pc);
                    const int ps = lane >> 3, ds = lane & 7;
                    const float4 *qp = reinterpret_cast<const float4 *>(a.q + (size_t)r * kHidden + h * kHeadDim + ds * 8);
                    const float4 x0 = __ldcg(qp), x1 = __ldcg(qp + 1);
                    const float qv[8] = {x0.x * 0.125f, x0.y * 0.125f, x0.z * 0.125f, x0.w * 0.125f,
                                         x1.x * 0.125f, x1.y * 0.125f, x1.z * 0.125f, x1.w * 0.125f};
                    const int *pt = a.page_table + (size_t)a.row_slot[r] * a.pages_per_stream;
                    float m = -INFINITY, lsum = 0.f, o[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) o[j] = 0.f;
                    for (int pg = pg0; pg < pg1; ++pg) {
                        const __half *kb = kvl + (size_t)pt[pg] * kPageHalfs + h * kPage * kHeadDim + ds * 8;
                        const __half *vb = kb + kHeads * kPage * kHeadDim;
                        float sc[4];
                        int4 vr[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int pp = ps + 4 * u;
                            // L2 loads: the newest position was written in this launch
                            const int4 kr = __ldcg(reinterpret_cast<const int4 *>(kb + pp * kHeadDim));
                            vr[u] = __ldcg(reinterpret_cast<const int4 *>(vb + pp * kHeadDim));
                            if (pg * kPage + pp >= n) vr[u] = make_int4(0, 0, 0, 0);
                            const __half2 *kh = reinterpret_cast<const __half2 *>(&kr);
                            float d = 0.f;
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 kf = __half22float2(kh[e]);
                                d = fmaf(qv[2 * e], kf.x, d);
                                d = fmaf(qv[2 * e + 1], kf.y, d);
                            }
                            sc[u] = d;
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 1);
                            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 2);
                            sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], 4);
                            if (pg * kPage + ps + 4 * u >= n) sc[u] = -INFINITY;
                        }
                        const float mn = fmaxf(fmaxf(m, fmaxf(sc[0], sc[1])), fmaxf(sc[2], sc[3]));
                        if (mn == -INFINITY) continue;
                        const float corr = __expf(m - mn);
                        float pw[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) pw[u] = __expf(sc[u] - mn);
                        lsum = lsum * corr + ((pw[0] + pw[1]) + (pw[2] + pw[3]));
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
#pragma unroll
                    for (int off = 8; off <= 16; off <<= 1) {
                        const float mo = __shfl_xor_sync(0xffffffffu, m, off);
                        const float lo2 = __shfl_xor_sync(0xffffffffu, lsum, off);
                        const float mx = fmaxf(m, mo);
                        const float c1 = (m == -INFINITY) ? 0.f : __expf(m - mx);
                        const float c2 = (mo == -INFINITY) ? 0.f : __expf(mo - mx);
                        lsum = lsum * c1 + lo2 * c2;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float oo = __shfl_xor_sync(0xffffffffu, o[j], off);
                            o[j] = o[j] * c1 + oo * c2;
                        }
                        m = mx;
                    }
                    float *pp = a.apart + (((size_t)h * R + r) * kStepMaxChunks + item) * kPartStride;
                    if (lane < 8) {
                        reinterpret_cast<float4 *>(pp + 4 + ds * 8)[0] = make_float4(o[0], o[1], o[2], o[3]);
                        reinterpret_cast<float4 *>(pp + 4 + ds * 8)[1] = make_float4(o[4], o[5], o[6], o[7]);
                        if (lane == 0) *reinterpret_cast<float2 *>(pp) = make_float2(m, lsum);
                    }
                }
            }
            if (!step_sync(ts + 1, kTeamCtas, a.err, 12)) return;

            // A4: merge the chunks of head h for every row (warp r), then the proj share
            if (warp < R) {
                const int r = warp;
                const int npg = (a.row_pos[r] + kPage) / kPage;
                const int pc = (npg + kStepMaxChunks - 1) / kStepMaxChunks;
                const int nch = (npg + pc - 1) / pc;
                const float *base = a.apart + ((size_t)h * R + r) * kStepMaxChunks * kPartStride;
                float M = -INFINITY;
                for (int c = 0; c < nch; ++c) M = fmaxf(M, __ldcg(base + (size_t)c * kPartStride));
                float Ls = 0.f, y0 = 0.f, y1 = 0.f;
                for (int c = 0; c < nch; ++c) {
                    const float *q = base + (size_t)c * kPartStride;
                    const float w = __expf(__ldcg(q) - M);
                    Ls = fmaf(__ldcg(q + 1), w, Ls);
                    const float2 ov = __ldcg(reinterpret_cast<const float2 *>(q + 4) + lane);
                    y0 = fmaf(ov.x, w, y0);
                    y1 = fmaf(ov.y, w, y1);
                }
                const float inv = 1.f / Ls;
                attn[r * kHeadDim + 2 * lane] = y0 * inv;
                attn[r * kHeadDim + 2 * lane + 1] = y1 * inv;
            }
            __syncthreads();
            {
                // proj rows 4 g .. 4 g + 3, K blocks 2h, 2h+1: team warp tw = group g (192 groups)
                const int g = tc * 16 + warp;
                const int k = (lane & 7) >> 1, hh = lane & 1, blk = (lane >> 3) & 1;
                float acc[kSmallMaxR];
#pragma unroll
                for (int r = 0; r < kSmallMaxR; ++r) acc[r] = 0.f;
                if (lane < 16) {
                    const int b = 2 * h + blk;
                    const int4 q = ldg_stream(L.proj_qs + (((size_t)g * (kHidden / 32) + b) * 8 + (lane & 7)) * 16);
                    const float d = __half2float(L.proj_sc[((size_t)g * (kHidden / 32) + b) * 4 + k]);
                    float wf[16];
                    unpack16(q, wf);
#pragma unroll
                    for (int r = 0; r < kSmallMaxR; ++r) {
                        if (r < R) {
                            const float *xv = attn + r * kHeadDim + blk * 32 + hh * 16;
                            float s = 0.f;
#pragma unroll
                            for (int t = 0; t < 16; ++t) s = fmaf(wf[t], xv[t], s);
                            acc[r] = s * d;
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < kSmallMaxR; ++r) {
                    float v = acc[r];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 8);
                    acc[r] = v;
                }
                if (lane < 8 && (lane & 1) == 0) {
                    const int j = g * 4 + k;
                    for (int r = 0; r < R; ++r) {
                        add_fix(acc_p + (size_t)r * kHidden + j, acc[r]);
                        if (h == 0) {  // the residual input and the bias, once
                            add_fix(acc_p + (size_t)r * kHidden + j, xraw[r * kHidden + j]);
                            add_fix(acc_p + (size_t)r * kHidden + j, L.proj_b[j]);
                        }
                    }
                }
            }
        }
        grid_target += kStepCtas;
        if (!step_sync(a.sync, grid_target, a.err, 13)) return;

        // ============================== phase B
        if (in_b) {
            const int b = cta;
            step_load_ln(a, acc_p, L.ln2_w, L.ln2_b, xraw, xl);
            // B2: fc_in groups 8b + warp / 2, K slice warp % 2 (12 blocks each)
            {
                const int gl = warp >> 1, slice = warp & 1;
                float acc[kSmallMaxR];
                warp_group_dot(L.fcin_qs, L.fcin_sc, kHidden / 32, 8 * b + gl, slice * 12, 12, xl, kHidden, R, acc);
                if (lane < 8 && (lane & 1) == 0)
#pragma unroll
                    for (int r = 0; r < kSmallMaxR; ++r) red[(warp * 4 + (lane >> 1)) * kSmallMaxR + r] = acc[r];
                __syncthreads();
                for (int t = tid; t < 32 * R; t += blockDim.x) {
                    const int f = t % 32, r = t / 32;  // feature 32 b + f = row 4 (8 b + f / 4) + f % 4
                    const int gl2 = f >> 2, k = f & 3;
                    const float v = red[((2 * gl2) * 4 + k) * kSmallMaxR + r] + red[((2 * gl2 + 1) * 4 + k) * kSmallMaxR + r];
                    gel[r * 32 + f] = gelu_new(__fadd_rn(v, L.fcin_b[32 * b + f]));
                }
                __syncthreads();
            }
            // B3: fc_out rows (192 groups, 12 per warp), K block b: lanes 8 i .. 8 i + 7 take group
            // 12 warp + 3 it + i's 8 chunks
            for (int it = 0; it < 3; ++it) {
                const int g = warp * 12 + it * 4 + (lane >> 3);
                const int k = (lane & 7) >> 1, hh = lane & 1;
                const int4 q = ldg_stream(L.fcout_qs + (((size_t)g * (kFF / 32) + b) * 8 + (lane & 7)) * 16);
                const float d = __half2float(L.fcout_sc[((size_t)g * (kFF / 32) + b) * 4 + k]);
                float wf[16];
                unpack16(q, wf);
                float acc[kSmallMaxR];
#pragma unroll
                for (int r = 0; r < kSmallMaxR; ++r) {
                    acc[r] = 0.f;
                    if (r < R) {
                        const float *xv = gel + r * 32 + hh * 16;
                        float s = 0.f;
#pragma unroll
                        for (int t = 0; t < 16; ++t) s = fmaf(wf[t], xv[t], s);
                        acc[r] = s * d;
                    }
                    acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
                }
                if ((lane & 1) == 0) {
                    const int j = g * 4 + k;
                    for (int r = 0; r < R; ++r) add_fix(acc_f + (size_t)r * kHidden + j, acc[r]);
                }
            }
            if (b == 0) {  // the residual input and the bias, once
                for (int t = tid; t < R * kHidden; t += blockDim.x) {
                    add_fix(acc_f + t, xraw[t]);
                    add_fix(acc_f + t, L.fcout_b[t % kHidden]);
                }
            }
        }
        grid_target += kStepCtas;
        if (!step_sync(a.sync, grid_target, a.err, 14)) return;
    }
    // final residual stream -> x (ln_f runs after this kernel)
    if (cta == 0) {
        const unsigned long long *acc_last = a.acc + ((size_t)(kLayers - 1) * 2 + 1) * racc;
        for (int t = tid; t < R * kHidden; t += blockDim.x) a.x[t] = from_fix(acc_last[t]);
    }
}

constexpr size_t kStepSmem =
    sizeof(float) * (2 * kSmallMaxR * kHidden + 16 * 4 * kSmallMaxR + kSmallMaxR * kHeadDim + kSmallMaxR * 32);

}  // namespace
}  // namespace mossgpu
