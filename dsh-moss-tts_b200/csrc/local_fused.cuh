// local_fused.cuh -- the local codebook decoder (reference llm.cpp:648-698: 17 one-layer steps
// per frame, the 16 tied audio heads and the greedy sampler with the repetition penalty) as one
// kernel per launch instead of ~10 dependent launches per step.
//
// Work split: a thread-block cluster of C CTAs runs G = 8 batch rows through the steps.  CTA c
// owns a fixed slice of every weight matrix -- 1/C of the output rows of QKV, proj, fc_in and
// the audio head, and 1/C of the K columns of fc_out (whose input is its own fc_in slice) -- and
// streams that slice from L2 (the local weights are ~21 MB) through a ring of bulk copies that a
// producer warp fills ahead of use, across step boundaries, since weights do not depend on data.
// Activations stay in shared memory: every CTA keeps the rows' residual stream, normalises it
// itself (LayerNorm is cheap next to a cluster exchange), and the CTAs exchange their output
// slices through distributed shared memory.  Per step and CTA:
//   LN1 -> QKV slice (+bias, RoPE; q and the new K/V row to global) | cluster phase
//   attention of its (row, head) items over <= 17 positions -> every CTA's proj input | phase
//   proj slice (+bias, +residual) -> every CTA's residual stream | phase
//   LN2 -> fc_in slice (+bias, GELU) -> own fc_out input slice
//   fc_out partial over its K slice -> the owner CTA of each output row | phase
//   sum of the C partials (fixed order) +bias +residual -> every CTA's residual stream | phase
//   ln_f -> head slice -> logits (global) and the penalised first maximum of its codes -> every
//   CTA | phase; the winner over the C candidates is the code; every CTA gathers its embedding
//   as the next step's input.
// A launch runs steps [step0, step1).  Step 0 alone is one launch (its output goes to the end
// gate, k_gate); steps 1..16 are the second, after the gate has set each stream's active flag.
//
// Tensor cores: mma.sync m16n8k16 (fp16 in, fp32 accumulate) with the 8 batch rows as N.  The
// weights' int8 values are exact in fp16 and are converted in registers (no shared-memory round
// trip); the per-32-column block scales (Q8_0) vary along K, so each block's product is
// accumulated from zero and scaled into the fp32 sum in registers, as the reference's block dot
// does (sum_b d_b * sum_i q_i x_i).  Activations are split into fp16 hi + lo parts so that the
// product carries fp32-level precision (two MMAs per block and K step).  At 8 rows per tile the
// problem is latency- and L2-bound, not tensor-throughput-bound.
//
// Synchronisation: a cluster "phase" is a pair of mbarriers per CTA (even / odd phases) that
// every CTA's consumer warps complete with one remote arrive per CTA (release.cluster), and wait
// on with acquire.cluster.  The producer warp is not part of the phases.  Every wait is bounded;
// a wait that runs out records a code (31 ring data, 32 ring slot, 33 cluster phase) and sets a
// CTA-wide flag after which no wait spins again, so every thread still reaches the kernel's
// final cluster barrier (no CTA leaves while another may write its shared memory), and the
// producer lets every bulk copy it issued land first.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "types.h"

namespace mossgpu {
namespace {

constexpr int kLfG = 8;               // batch rows per cluster (the MMA N)
constexpr int kLfWarps = 8;           // consumer warps (warp n also handles row n)
constexpr int kLfThreads = (kLfWarps + 1) * 32;
constexpr int kLfUnitQ = 12288;       // int8 bytes of one ring unit (24 tile-blocks of 512 B)
constexpr int kLfUnitS = 768;         // its fp16 scales (24 x 16)
constexpr int kLfStage = kLfUnitQ + kLfUnitS;
constexpr int kLfActStride = kHidden + 32;  // halves per activation row (conflict-free 16 B loads)

// Weight matrix in the MMA fragment layout (k_repack_mma): [rows/16][nb][512] bytes and
// [rows/16][nb][16] fp16.  In the 512-byte record of (16-row tile, 32-column block), lane
// L = 4 g + t owns bytes [16 L, 16 L + 16): row g at columns 2t + (j & 1) + 8 (j >> 1) for
// j = 0..7, then row g + 8 at the same columns.  Each byte holds q + 128 (the int8 quant in
// offset binary, ready for the fp16 conversion below).  The 16 scales are ordered (row g,
// row g + 8) for g = 0..7.
struct LfMat {
    const int8_t *qm;
    const __half *sm;
    int nb;  // 32-column blocks per row
};

// GEMV planes ([rows/4][nb][4][32] int8, [rows/4][nb][4] fp16) -> the fragment layout.  One
// thread per (tile, block, lane).
__global__ void k_repack_mma(const int8_t *__restrict__ qs, const __half *__restrict__ sc, int rows, int cols,
                             int8_t *__restrict__ qm, __half *__restrict__ sm) {
    const int nb = cols / 32;
    const long long total = (long long)(rows / 16) * nb * 32;
    const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= total) return;
    const int lane = (int)(id & 31);
    const long long tb = id >> 5;  // tile * nb + block
    const int b = (int)(tb % nb);
    const int tile = (int)(tb / nb);
    const int g = lane >> 2, t = lane & 3;
    __align__(16) int8_t out[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int row = tile * 16 + g + 8 * (j >> 3);
        const int col = 2 * t + (j & 1) + 8 * ((j >> 1) & 3);
        out[j] = (int8_t)(qs[((size_t)(row >> 2) * nb + b) * 128 + (row & 3) * 32 + col] ^ 0x80);
    }
    *reinterpret_cast<int4 *>(qm + (size_t)tb * 512 + lane * 16) = *reinterpret_cast<const int4 *>(out);
    if (lane < 16) {
        const int row = tile * 16 + (lane >> 1) + 8 * (lane & 1);
        sm[(size_t)tb * 16 + lane] = sc[((size_t)(row >> 2) * nb + b) * 4 + (row & 3)];
    }
}

struct LfArgs {
    LfMat attn, proj, fc_in, fc_out, head[kNVq];
    const float *attn_b, *proj_b, *fc_in_b, *fc_out_b;
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b, *lnf_w, *lnf_b;
    const float2 *rope;        // [pos][32] (cos, sin)
    QMat wte;                  // row 9 = step 1's input
    QMat aemb[kNVq];           // next-input embeddings
    const float *hidden;       // [slot][768]: step 0's input
    const int *row_slot;
    int R;
    float *lkv;                // [slot][k|v][17][768] fp32
    float *qbuf;               // [R][768]
    float *lx_out;             // [R][768]: step 0's output (the gate's input)
    float *logits;             // [R][16][1024]
    uint16_t *counts;          // [slot][16][1024]
    const FrameCtl *ctl;
    const int *forced;         // [R][16] when ctl->has_forced
    const int *active;         // [R]
    int *codes_out, *used_out; // [R][16]
    int step0, step1;
    int *err;
};

// ---- small PTX helpers

__device__ __forceinline__ int4 lds128(const void *p) { return *reinterpret_cast<const int4 *>(p); }

// 4 offset-binary bytes (q + 128) -> two half2 of q (bytes 0,1 and bytes 2,3), exact: 0x64XX
// is 1024 + XX as fp16, and XX = q + 128, so (0x64XX - 1152) = q.
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t a = __byte_perm(w, 0x64646464u, 0x5140);
    const uint32_t b = __byte_perm(w, 0x64646464u, 0x7362);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), bias);
    const __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), bias);
    lo = *reinterpret_cast<const uint32_t *>(&ha);
    hi = *reinterpret_cast<const uint32_t *>(&hb);
}

__device__ __forceinline__ void mma16816(float &d0, float &d1, float &d2, float &d3, uint32_t a0, uint32_t a1,
                                         uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// position of column k of an activation row: within each 32-column block, the 8 halves a lane
// reads with one 16-byte load for both K steps of the block (k = 2t + e + 8 j -> 8 t + 2 j + e)
__device__ __forceinline__ int lf_bpos(int k) {
    return (k & ~31) | (((k & 7) >> 1) << 3) | (((k >> 3) & 3) << 1) | (k & 1);
}

__device__ __forceinline__ void lf_named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kLfWarps * 32) : "memory"); }

__device__ __forceinline__ uint32_t lf_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t lf_clusterid() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t lf_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void lf_st_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void lf_st_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ float lf_ld_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void lf_st_s32(uint32_t addr, int v) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void lf_remote_arrive(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ bool lf_try_cluster(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, "
        "p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on a local mbarrier phase.  cluster_scope: acquire at cluster scope (the phases
// that other CTAs complete).  Gives up at once once `failed` is set, and after about a second
// otherwise, recording `code`.
__device__ __forceinline__ bool lf_wait(uint64_t *bar, uint32_t parity, volatile int *failed, int *err, int code,
                                        bool cluster_scope) {
    const uint32_t addr = smem_u32(bar);
    for (int it = 0; it < 2048; ++it) {
        if (cluster_scope ? lf_try_cluster(addr, parity) : mbar_try(addr, parity)) return true;
        if (*failed) return false;
    }
    const uint64_t t0 = global_ns();
    for (;;) {
        if (cluster_scope ? lf_try_cluster(addr, parity) : mbar_try(addr, parity)) return true;
        if (*failed) return false;
        if (global_ns() - t0 > 1000000000ull) break;
        __nanosleep(256);
    }
    if (err) atomicCAS(err, 0, code);
    *failed = 1;
    return false;
}

// ---- the schedule of ring units: identical for the producer and the consumers

enum { LF_QKV = 0, LF_PROJ = 1, LF_FCIN = 2, LF_FCOUT = 3, LF_HEAD = 4 };

template <int MT_, int KB_>
struct LfShape {  // 16-row tiles and 32-column blocks of a ring unit (MT * KB = 24)
    static constexpr int MT = MT_, KB = KB_;
};

struct LfPhase {
    LfMat m;
    int row0;    // first weight row of unit 0
    int rstep;   // weight rows between consecutive units
    int mt;      // 16-row tiles per unit
    int kb;      // 32-column blocks per unit
    int kb0;     // first block
    int units;
};

template <int C>
__device__ __forceinline__ LfPhase lf_phase(const LfArgs &a, int ph, int ls, int c) {
    LfPhase p{};
    switch (ph) {
        case LF_QKV: p.m = a.attn; p.mt = 1; p.kb = 24; p.rstep = 16; p.row0 = c * (kQKV / C); p.units = kQKV / C / 16; break;
        case LF_PROJ: p.m = a.proj; p.mt = 1; p.kb = 24; p.rstep = 16; p.row0 = c * (kHidden / C); p.units = kHidden / C / 16; break;
        case LF_FCIN: p.m = a.fc_in; p.mt = 1; p.kb = 24; p.rstep = 16; p.row0 = c * (kFF / C); p.units = kFF / C / 16; break;
        case LF_FCOUT:
            p.m = a.fc_out;
            p.kb = kFF / 32 / C;
            p.kb0 = c * p.kb;
            p.mt = 24 / p.kb;
            p.rstep = 16 * p.mt;
            p.row0 = 0;
            p.units = kHidden / p.rstep;
            break;
        default:
            p.m = a.head[ls - 1]; p.mt = 1; p.kb = 24; p.rstep = 16; p.row0 = c * (kCodebook / C); p.units = kCodebook / C / 16;
            break;
    }
    return p;
}

// shared-memory layout (bytes)
template <int C>
struct LfSmem {
    static constexpr int kGel = kFF / C + 32;                       // halves per fc_out-input row
    static constexpr int kMo = kHidden / C;                         // fc_out rows a CTA reduces
    static constexpr int kMh = kCodebook / C;                       // head codes per CTA
    static constexpr int xres = 0;                                  // float [8][768]
    static constexpr int act_hi = xres + kLfG * kHidden * 4;        // half [8][800]
    static constexpr int act_lo = act_hi + kLfG * kLfActStride * 2;
    static constexpr int gel_hi = act_lo + kLfG * kLfActStride * 2; // half [8][kGel]
    static constexpr int gel_lo = gel_hi + kLfG * kGel * 2;
    static constexpr int part = gel_lo + kLfG * kGel * 2;           // float [8][768]: fc_out partials
    static constexpr int lnp = part + kLfG * kHidden * 4;           // float [6][768]: LN1, LN2, ln_f w and b
    static constexpr int lgt = lnp + 6 * kHidden * 4;               // float [8][kMh]
    static constexpr int cand_v = lgt + kLfG * kMh * 4;             // float [C][8]
    static constexpr int cand_i = cand_v + C * kLfG * 4;            // int [C][8]
    static constexpr int used = cand_i + C * kLfG * 4;              // int [8]
    static constexpr int hist = used + kLfG * 4;                    // int [8][16]: codes used per channel
    static constexpr int flags = hist + kLfG * kNVq * 4;            // int failed + pad
    static constexpr int bars = (flags + 16 + 7) / 8 * 8;
    static constexpr int kStages = 9;
    static constexpr int ring = (bars + (2 * kStages + 2) * 8 + 127) / 128 * 128;
    static constexpr int total = ring + kStages * kLfStage;
};
static_assert(LfSmem<8>::total <= 232448 && LfSmem<16>::total <= 232448, "fused local decoder exceeds shared memory");

// LayerNorm (llm.cpp:159-171) of row n of the residual stream into the fp16 hi/lo activation
// rows, by one warp, with k_build_bimg's arithmetic and order.
__device__ __forceinline__ void lf_layernorm(const float *xres, int n, const float *w, const float *b, __half *hi,
                                             __half *lo, int lane) {
    float v[3][8];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const float4 *xp = reinterpret_cast<const float4 *>(xres + n * kHidden + 8 * (lane + 32 * j));
        const float4 a0 = xp[0], a1 = xp[1];
        v[j][0] = a0.x; v[j][1] = a0.y; v[j][2] = a0.z; v[j][3] = a0.w;
        v[j][4] = a1.x; v[j][5] = a1.y; v[j][6] = a1.z; v[j][7] = a1.w;
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) sum += v[j][e];
    const float mean = __fdiv_rn(warp_sum(sum), (float)kHidden);
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float d = v[j][e] - mean;
            var = fmaf(d, d, var);
        }
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(warp_sum(var), (float)kHidden) + 1e-5f));
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int k0 = 8 * (lane + 32 * j);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            float y[2];
#pragma unroll
            for (int q = 0; q < 2; ++q)
                y[q] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j][e + q], mean), inv), w[k0 + e + q]), b[k0 + e + q]);
            const __half2 h = __floats2half2_rn(y[0], y[1]);
            const float2 hf = __half22float2(h);
            const __half2 l = __floats2half2_rn(y[0] - hf.x, y[1] - hf.y);
            const int p = n * kLfActStride + lf_bpos(k0 + e);
            *reinterpret_cast<__half2 *>(hi + p) = h;
            *reinterpret_cast<__half2 *>(lo + p) = l;
        }
    }
}

// One ring unit on one warp: acc[mt][4] = sum over its blocks of scale * (W x) for 16-row
// tiles x the 8 batch rows.  act_hi / act_lo: B rows [8][stride] in lf_bpos order; kbase = the
// unit's first block within those rows.
template <int MT, int KB>
__device__ __forceinline__ void lf_unit_mma(const uint8_t *stage, const __half *act_hi, const __half *act_lo,
                                            int stride, int kbase, int lane, float (&acc)[MT][4]) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    const uint8_t *qbase = stage + lane * 16;
    const uint8_t *sbase = stage + kLfUnitQ + g * 4;
    const __half *bh = act_hi + g * stride + kbase * 32 + t * 8;
    const __half *bl = act_lo + g * stride + kbase * 32 + t * 8;
    constexpr int kUnroll = MT == 1 ? 4 : 2;  // independent blocks in flight (MMA latency)
#pragma unroll kUnroll
    for (int b = 0; b < KB; ++b) {
        const int4 xh = lds128(bh + b * 32);
        const int4 xl = lds128(bl + b * 32);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int4 q = lds128(qbase + (mt * KB + b) * 512);
            const uint32_t s2 = *reinterpret_cast<const uint32_t *>(sbase + (mt * KB + b) * 32);
            uint32_t a00, a02, a01, a03, a10, a12, a11, a13;
            i8x4_to_h2x2((uint32_t)q.x, a00, a02);  // row g: K step 0 cols 2t.., 2t+8..
            i8x4_to_h2x2((uint32_t)q.z, a01, a03);  // row g+8
            i8x4_to_h2x2((uint32_t)q.y, a10, a12);  // row g: K step 1
            i8x4_to_h2x2((uint32_t)q.w, a11, a13);  // row g+8
            // two independent chains (the hi and the lo parts of x) of two K steps each
            float h0 = 0.f, h1 = 0.f, h2 = 0.f, h3 = 0.f, l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
            mma16816(h0, h1, h2, h3, a00, a01, a02, a03, (uint32_t)xh.x, (uint32_t)xh.y);
            mma16816(l0, l1, l2, l3, a00, a01, a02, a03, (uint32_t)xl.x, (uint32_t)xl.y);
            mma16816(h0, h1, h2, h3, a10, a11, a12, a13, (uint32_t)xh.z, (uint32_t)xh.w);
            mma16816(l0, l1, l2, l3, a10, a11, a12, a13, (uint32_t)xl.z, (uint32_t)xl.w);
            const float2 s = __half22float2(*reinterpret_cast<const __half2 *>(&s2));
            acc[mt][0] = fmaf(s.x, h0 + l0, acc[mt][0]);
            acc[mt][1] = fmaf(s.x, h1 + l1, acc[mt][1]);
            acc[mt][2] = fmaf(s.y, h2 + l2, acc[mt][2]);
            acc[mt][3] = fmaf(s.y, h3 + l3, acc[mt][3]);
        }
    }
}

// xres[n][:] = row codes[n] of a Q8_0_4X4 matrix with 768 columns, dequantised as deq_elem
// does (scale * q in fp32); rows whose code is outside [0, rows) become zeros.  One
// (row, 32-column block) per thread, its 32 quants and scale loaded together.
__device__ __forceinline__ void lf_gather_rows(float *xres, const QMat &m, const int *codes, int tid) {
    constexpr int nb = kHidden / 32;
    for (int item = tid; item < kLfG * nb; item += kLfWarps * 32) {
        const int n = item / nb, b = item - n * nb;
        const int code = codes[n];
        float4 *dst = reinterpret_cast<float4 *>(xres + n * kHidden + b * 32);
        if (code < 0 || code >= m.rows) {
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        const size_t blk = (size_t)(code >> 2) * nb + b;
        const int4 *qp = reinterpret_cast<const int4 *>(m.qs + blk * 128 + (code & 3) * 32);
        const int4 q0 = qp[0], q1 = qp[1];
        const float d = __half2float(m.sc[blk * 4 + (code & 3)]);
        float w[32];
        unpack16(q0, w);
        unpack16(q1, w + 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_float4(d * w[4 * j], d * w[4 * j + 1], d * w[4 * j + 2], d * w[4 * j + 3]);
    }
}

template <int C>
__global__ void __launch_bounds__(kLfThreads, 1) k_local_fused(const LfArgs a) {
    using S = LfSmem<C>;
    constexpr int NS = S::kStages;
    extern __shared__ __align__(1024) uint8_t lf_smem[];
    float *xres = reinterpret_cast<float *>(lf_smem + S::xres);
    __half *act_hi = reinterpret_cast<__half *>(lf_smem + S::act_hi);
    __half *act_lo = reinterpret_cast<__half *>(lf_smem + S::act_lo);
    __half *gel_hi = reinterpret_cast<__half *>(lf_smem + S::gel_hi);
    __half *gel_lo = reinterpret_cast<__half *>(lf_smem + S::gel_lo);
    float *part = reinterpret_cast<float *>(lf_smem + S::part);
    float *lnp = reinterpret_cast<float *>(lf_smem + S::lnp);
    int *hist = reinterpret_cast<int *>(lf_smem + S::hist);
    float *lgt = reinterpret_cast<float *>(lf_smem + S::lgt);
    float *cand_v = reinterpret_cast<float *>(lf_smem + S::cand_v);
    int *cand_i = reinterpret_cast<int *>(lf_smem + S::cand_i);
    int *used_s = reinterpret_cast<int *>(lf_smem + S::used);
    volatile int *failed = reinterpret_cast<volatile int *>(lf_smem + S::flags);
    uint64_t *full = reinterpret_cast<uint64_t *>(lf_smem + S::bars);
    uint64_t *empty = full + NS;
    uint64_t *cbar = empty + NS;
    uint8_t *ring = lf_smem + S::ring;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = (int)lf_ctarank();
    const int rbase = (int)lf_clusterid() * kLfG;
    const int nrows = min(kLfG, a.R - rbase);
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&cbar[0], C);
        mbar_init(&cbar[1], C);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster_arrive();  // every CTA's barriers exist before any remote arrive
    cluster_wait();

    if (warp == kLfWarps) {
        // ------------------------------------------------------------- producer warp
        if (lane == 0) {
            int u = 0;
            bool ok = true;
            for (int ls = a.step0; ls < a.step1 && ok; ++ls) {
                const int nph = ls == 0 ? 4 : 5;
                for (int ph = 0; ph < nph && ok; ++ph) {
                    const LfPhase p = lf_phase<C>(a, ph, ls, c);
                    for (int i = 0; i < p.units; ++i, ++u) {
                        const int s = u % NS;
                        if (!lf_wait(&empty[s], ((u / NS) & 1) ^ 1, failed, a.err, 32, false)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&full[s], kLfStage);
                        uint8_t *dst = ring + (size_t)s * kLfStage;
                        const int tile0 = (p.row0 + i * p.rstep) / 16;
                        for (int mt = 0; mt < p.mt; ++mt) {
                            const size_t rec = (size_t)(tile0 + mt) * p.m.nb + p.kb0;
                            bulk_g2s(dst + mt * p.kb * 512, p.m.qm + rec * 512, p.kb * 512, &full[s]);
                            bulk_g2s(dst + kLfUnitQ + mt * p.kb * 32, p.m.sm + rec * 16, p.kb * 32, &full[s]);
                        }
                    }
                }
            }
            // every copy issued must land before the CTA may leave (the unit that failed its
            // slot wait issued nothing)
            for (int k = max(0, u - NS); k < u; ++k) {
                const uint32_t addr = smem_u32(&full[k % NS]);
                const uint64_t t0 = global_ns();
                while (!mbar_try(addr, (k / NS) & 1) && global_ns() - t0 < 1000000000ull) __nanosleep(256);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------- consumer warps
        pdl_wait();
        pdl_trigger();
        const FrameCtl ctl = *a.ctl;
        const int g = lane >> 2, t = lane & 3;
        // remote (cluster) addresses of the exchanged buffers: base of CTA d's copy
        const uint32_t xres_s = smem_u32(xres), acth_s = smem_u32(act_hi), actl_s = smem_u32(act_lo);
        const uint32_t part_s = smem_u32(part), cv_s = smem_u32(cand_v), ci_s = smem_u32(cand_i);
        {   // LayerNorm parameters (LN1, LN2, ln_f; weight and bias) stay in shared memory
            const float *src[6] = {a.ln1_w, a.ln1_b, a.ln2_w, a.ln2_b, a.lnf_w, a.lnf_b};
#pragma unroll
            for (int v = 0; v < 6; ++v)
                for (int i = tid; i < kHidden / 4; i += kLfWarps * 32)
                    reinterpret_cast<float4 *>(lnp + v * kHidden)[i] = reinterpret_cast<const float4 *>(src[v])[i];
        }
        // initial residual stream: the global hidden state (step 0) or the slot-token row (step 1)
        if (a.step0 == 0) {
            constexpr int per = kLfG * kHidden / 4 / (kLfWarps * 32);  // float4s per thread
            float4 v[per];
#pragma unroll
            for (int j = 0; j < per; ++j) {  // all loads first, then the stores
                const int i4 = tid + j * kLfWarps * 32, n = i4 / (kHidden / 4), k4 = i4 - n * (kHidden / 4);
                v[j] = n < nrows ? reinterpret_cast<const float4 *>(a.hidden + (size_t)a.row_slot[rbase + n] * kHidden)[k4]
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < per; ++j) reinterpret_cast<float4 *>(xres)[tid + j * kLfWarps * 32] = v[j];
        } else {
            if (tid < kLfG) used_s[tid] = kSlotToken;
            lf_named_sync();
            lf_gather_rows(xres, a.wte, used_s, tid);
        }
        lf_named_sync();
        int u = 0;       // ring unit counter
        int cph = 0;     // cluster phase counter

        auto cluster_phase = [&]() {
            asm volatile("fence.acq_rel.cluster;" ::: "memory");
            lf_named_sync();
            if (tid < C) lf_remote_arrive(lf_map(smem_u32(&cbar[cph & 1]), (uint32_t)tid));  // one per CTA
            lf_wait(&cbar[cph & 1], (cph >> 1) & 1, failed, a.err, 33, true);
            ++cph;
        };
        // run the units of one phase; epi(mt, acc, i) for each unit i of this warp
        auto gemm = [&](const LfPhase &p, const __half *bh, const __half *bl, int stride, auto mtkb, auto &&epi) {
            constexpr int MT = decltype(mtkb)::MT, KB = decltype(mtkb)::KB;
            for (int i = warp; i < p.units; i += kLfWarps) {
                const int uu = u + i;
                const int s = uu % NS;
                lf_wait(&full[s], (uu / NS) & 1, failed, a.err, 31, false);
                float acc[MT][4];
                lf_unit_mma<MT, KB>(ring + (size_t)s * kLfStage, bh, bl, stride, 0, lane, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                epi(acc, i);
            }
            u += p.units;
        };
        using Full = LfShape<1, 24>;
        using Fco = LfShape<24 / (kFF / 32 / C), kFF / 32 / C>;  // fc_out: this CTA's K slice

        for (int ls = a.step0; ls < a.step1; ++ls) {
            // ---- LN1 -> QKV slice
            if (warp < kLfG) lf_layernorm(xres, warp, lnp, lnp + kHidden, act_hi, act_lo, lane);
            lf_named_sync();
            {
                const LfPhase p = lf_phase<C>(a, LF_QKV, ls, c);
                gemm(p, act_hi, act_lo, kLfActStride, Full{}, [&](float(&acc)[1][4], int i) {
                    const int f0 = p.row0 + i * 16 + g;  // rows f0 and f0 + 8
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int f = f0 + 8 * h;
                        const float bias = a.attn_b[f];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int n = 2 * t + e;
                            const float v = __fadd_rn(acc[0][2 * h + e], bias);
                            const float pv = __shfl_xor_sync(0xffffffffu, v, 4);  // the pair partner f ^ 1
                            float o = v;
                            if (f < 2 * kHidden) {
                                const float2 cs = a.rope[(size_t)ls * (kHeadDim / 2) + ((f % kHeadDim) >> 1)];
                                o = (f & 1) ? __fadd_rn(__fmul_rn(v, cs.x), __fmul_rn(pv, cs.y))
                                            : __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(pv, cs.y));
                            }
                            if (n < nrows) {
                                const int r = rbase + n;
                                if (f < kHidden) {
                                    a.qbuf[(size_t)r * kHidden + f] = o;
                                } else {
                                    const int kv = f < 2 * kHidden ? 0 : 1;
                                    a.lkv[(((size_t)a.row_slot[r] * 2 + kv) * kLocalLen + ls) * kHidden + f -
                                          kHidden * (1 + kv)] = o;
                                }
                            }
                        }
                    }
                });
            }
            cluster_phase();
            // ---- attention: items (row, head) c, c + C, ... -> every CTA's proj input
            for (int it = c + C * warp; it < kLfG * kHeads; it += C * kLfWarps) {
                const int n = it / kHeads, hd = it - n * kHeads;
                float o0 = 0.f, o1 = 0.f;
                if (n < nrows) {
                    const int r = rbase + n, slot = a.row_slot[r], np = ls + 1;
                    const float *kb = a.lkv + ((size_t)slot * 2 + 0) * kLocalLen * kHidden + hd * kHeadDim;
                    const float *vb = a.lkv + ((size_t)slot * 2 + 1) * kLocalLen * kHidden + hd * kHeadDim;
                    const float *qh = a.qbuf + (size_t)r * kHidden + hd * kHeadDim;
                    float sc = -INFINITY;
                    if (lane < np) {  // k_attn_local's arithmetic: lane = position
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
                        sc = dot * 0.125f;
                    }
                    float2 vv[kLocalLen];  // every V row the item needs, loaded before use
#pragma unroll
                    for (int pp = 0; pp < kLocalLen; ++pp)
                        vv[pp] = pp < np ? reinterpret_cast<const float2 *>(vb + (size_t)pp * kHidden)[lane]
                                         : make_float2(0.f, 0.f);
                    const float mx = warp_max(sc);
                    const float ex = lane < np ? expf(sc - mx) : 0.f;
                    const float wgt = ex * (1.0f / warp_sum(ex));
#pragma unroll
                    for (int pp = 0; pp < kLocalLen; ++pp) {
                        if (pp < np) {
                            const float wp = __shfl_sync(0xffffffffu, wgt, pp);
                            o0 = fmaf(wp, vv[pp].x, o0);
                            o1 = fmaf(wp, vv[pp].y, o1);
                        }
                    }
                }
                const __half2 h = __floats2half2_rn(o0, o1);
                const float2 hf = __half22float2(h);
                const __half2 l = __floats2half2_rn(o0 - hf.x, o1 - hf.y);
                const uint32_t off = (uint32_t)(n * kLfActStride + lf_bpos(hd * kHeadDim + 2 * lane)) * 2;
                for (int d = 0; d < C; ++d) {
                    lf_st_u32(lf_map(acth_s + off, (uint32_t)d), *reinterpret_cast<const uint32_t *>(&h));
                    lf_st_u32(lf_map(actl_s + off, (uint32_t)d), *reinterpret_cast<const uint32_t *>(&l));
                }
            }
            cluster_phase();
            // ---- proj slice + bias + residual -> every CTA's residual stream
            {
                const LfPhase p = lf_phase<C>(a, LF_PROJ, ls, c);
                gemm(p, act_hi, act_lo, kLfActStride, Full{}, [&](float(&acc)[1][4], int i) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int f = p.row0 + i * 16 + g + 8 * h;
                        const float bias = a.proj_b[f];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int n = 2 * t + e;
                            const float xn = __fadd_rn(xres[n * kHidden + f], __fadd_rn(acc[0][2 * h + e], bias));
                            const uint32_t off = (uint32_t)(n * kHidden + f) * 4;
                            for (int d = 0; d < C; ++d) lf_st_f32(lf_map(xres_s + off, (uint32_t)d), xn);
                        }
                    }
                });
            }
            cluster_phase();
            // ---- LN2 -> fc_in slice + bias + GELU -> own fc_out input
            if (warp < kLfG) lf_layernorm(xres, warp, lnp + 2 * kHidden, lnp + 3 * kHidden, act_hi, act_lo, lane);
            lf_named_sync();
            {
                const LfPhase p = lf_phase<C>(a, LF_FCIN, ls, c);
                gemm(p, act_hi, act_lo, kLfActStride, Full{}, [&](float(&acc)[1][4], int i) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int kl = i * 16 + g + 8 * h;  // column of this CTA's fc_out K slice
                        const float bias = a.fc_in_b[p.row0 + kl];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int n = 2 * t + e;
                            const float y = gelu_new(__fadd_rn(acc[0][2 * h + e], bias));
                            const __half hh = __float2half_rn(y);
                            const int pos = n * S::kGel + lf_bpos(kl);
                            gel_hi[pos] = hh;
                            gel_lo[pos] = __float2half_rn(y - __half2float(hh));
                        }
                    }
                });
            }
            lf_named_sync();
            // ---- fc_out partial over the K slice, kept here until its owner CTA pulls it
            {
                const LfPhase p = lf_phase<C>(a, LF_FCOUT, ls, c);
                gemm(p, gel_hi, gel_lo, S::kGel, Fco{}, [&](float(&acc)[Fco::MT][4], int i) {
#pragma unroll
                    for (int mt = 0; mt < Fco::MT; ++mt)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int f = i * p.rstep + mt * 16 + g + 8 * h;
#pragma unroll
                            for (int e = 0; e < 2; ++e) part[(2 * t + e) * kHidden + f] = acc[mt][2 * h + e];
                        }
                });
            }
            cluster_phase();
            // ---- this CTA's rows of fc_out: the C partials in order (read from every CTA) + bias +
            // residual -> everyone
            for (int i = tid; i < kLfG * S::kMo; i += kLfWarps * 32) {
                const int n = i / S::kMo, j = i - n * S::kMo, f = c * S::kMo + j;
                const uint32_t off = (uint32_t)(n * kHidden + f) * 4;
                float pv[C];
#pragma unroll
                for (int src = 0; src < C; ++src) pv[src] = lf_ld_f32(lf_map(part_s + off, (uint32_t)src));
                float sum = pv[0];
#pragma unroll
                for (int src = 1; src < C; ++src) sum = __fadd_rn(sum, pv[src]);
                const float xn = __fadd_rn(xres[n * kHidden + f], __fadd_rn(sum, a.fc_out_b[f]));
                for (int d = 0; d < C; ++d) lf_st_f32(lf_map(xres_s + off, (uint32_t)d), xn);  // same [8][768] layout
            }
            cluster_phase();
            if (ls == 0) {  // step 0's output: the end gate's input; step 1's input is the slot token
                if (c == 0)
                    for (int i = tid; i < nrows * kHidden; i += kLfWarps * 32) a.lx_out[(size_t)rbase * kHidden + i] = xres[i];
                if (tid < kLfG) used_s[tid] = kSlotToken;
                lf_named_sync();
                lf_gather_rows(xres, a.wte, used_s, tid);
                lf_named_sync();
                continue;
            }
            // ---- ln_f -> head slice -> logits and this CTA's candidate per row
            const int ch = ls - 1;
            if (warp < kLfG) lf_layernorm(xres, warp, lnp + 4 * kHidden, lnp + 5 * kHidden, act_hi, act_lo, lane);
            lf_named_sync();
            {
                const LfPhase p = lf_phase<C>(a, LF_HEAD, ls, c);
                gemm(p, act_hi, act_lo, kLfActStride, Full{}, [&](float(&acc)[1][4], int i) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int j = i * 16 + g + 8 * h;  // code - c * kMh
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int n = 2 * t + e;
                            lgt[n * S::kMh + j] = acc[0][2 * h + e];
                            if (n < nrows)
                                a.logits[((size_t)(rbase + n) * kNVq + ch) * kCodebook + c * S::kMh + j] = acc[0][2 * h + e];
                        }
                    }
                });
            }
            lf_named_sync();
            if (warp < kLfG) {  // warp n: repetition penalty (sampler.cpp:14-21), first maximum of this CTA's codes
                const int n = warp;
                float best = -INFINITY;
                int besti = 0x7fffffff;
                if (n < nrows) {
                    const uint16_t *cnt = a.counts + ((size_t)a.row_slot[rbase + n] * kNVq + ch) * kCodebook;
                    const float pen = ctl.rep_penalty;
                    int cc[S::kMh / 32];
#pragma unroll
                    for (int q = 0; q < S::kMh / 32; ++q) cc[q] = cnt[c * S::kMh + lane + 32 * q];  // loads first
#pragma unroll
                    for (int q = 0; q < S::kMh / 32; ++q) {
                        const int j = lane + 32 * q;
                        const int code = c * S::kMh + j;
                        float v = lgt[n * S::kMh + j];
                        if (pen != 1.0f)
                            for (int z = 0; z < cc[q]; ++z) v = v < 0.f ? __fmul_rn(v, pen) : __fdiv_rn(v, pen);
                        if (v > best || (v == best && code < besti)) {
                            best = v;
                            besti = code;
                        }
                    }
                }
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
                    if (ov > best || (ov == best && oi < besti)) {
                        best = ov;
                        besti = oi;
                    }
                }
                if (lane < C) {
                    const uint32_t off = (uint32_t)(c * kLfG + n) * 4;
                    lf_st_f32(lf_map(cv_s + off, (uint32_t)lane), best);
                    lf_st_s32(lf_map(ci_s + off, (uint32_t)lane), besti);
                }
            }
            cluster_phase();
            if (warp < kLfG) {  // the winner over the C candidates (first maximum), the code used
                const int n = warp;
                float best = lane < C ? cand_v[lane * kLfG + n] : -INFINITY;
                int besti = lane < C ? cand_i[lane * kLfG + n] : 0x7fffffff;
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
                    if (ov > best || (ov == best && oi < besti)) {
                        best = ov;
                        besti = oi;
                    }
                }
                const int pred = besti < kCodebook ? besti : 0;  // all-NaN logits: code 0
                int usedc = -1;
                if (n < nrows) {
                    const int r = rbase + n;
                    usedc = ctl.has_forced ? a.forced[r * kNVq + ch] : pred;
                    if (c == 0 && lane == 0) {
                        a.codes_out[r * kNVq + ch] = pred;
                        a.used_out[r * kNVq + ch] = usedc;
                    }
                }
                if (lane == 0) {
                    used_s[n] = usedc;
                    hist[n * kNVq + ch] = usedc;
                }
            }
            lf_named_sync();
            if (ch + 1 < kNVq) {
                lf_gather_rows(xres, a.aemb[ch], used_s, tid);
                lf_named_sync();
            }
        }
    }
    // the repetition history (sampler.cpp:14-21): a channel's counts are read only when that
    // channel samples, so the frame's increments can wait until every channel has sampled
    if (warp < kLfG && c == 0 && a.step1 > 1 && lane < kNVq) {
        const int n = warp, ch = lane;
        if (n < nrows && ch >= max(a.step0, 1) - 1 && ch < a.step1 - 1) {
            const int r = rbase + n, uc = hist[n * kNVq + ch];
            if (a.active[r] && uc >= 0 && uc < kCodebook) {
                uint16_t *cnt = a.counts + ((size_t)a.row_slot[r] * kNVq + ch) * kCodebook;
                cnt[uc] = (uint16_t)(cnt[uc] + 1);
            }
        }
    }
    __syncwarp();
    cluster_arrive();  // no CTA leaves while another may still write its shared memory
    cluster_wait();
}

}  // namespace
}  // namespace mossgpu
