// layer_small.cuh -- one global transformer layer (llm.cpp:230-246) for decode batches of at
// most 8 rows, in two launches instead of five.
//
// At this batch the layer is a chain of dependent phases, each too small to keep HBM busy, so
// its time is the hand-offs between them.  Two launches per layer keep only the hand-offs that
// need the whole layer's output (proj and fc_out read every head / every feature); the rest
// run inside a thread-block cluster, synchronised by cluster barriers and exchanging data
// through distributed shared memory (DSMEM).  Every exchange is a push: the producing threads
// store into the consuming CTAs' shared memory (st.shared::cluster), and one cluster barrier
// (release / acquire) later the consumers read their own shared memory, so no phase waits on a
// remote load's round trip; the first remote store of a CTA waits on a cluster barrier phase
// that every CTA arrives at when it starts.  Everything that does not depend on the previous
// launch -- the weights, LayerNorm parameters, biases, RoPE factors and the rows' cached K/V
// pages -- is copied into shared memory before the launch waits for its predecessor
// (programmatic dependent launch), so those HBM reads overlap the previous launch.  Global
// stores come after a CTA's last cluster barrier, so no barrier waits for them.
//
// The contractions run on the tensor cores (mma.sync m16n8k16, fp32 accumulation): weights as
// the MMA fragment records of k_repack_mma (exact int8 -> fp16), activations split into fp16
// hi + lo planes (x = hi + lo to ~2^-22), the 8 batch rows as the MMA's N; each 32-column
// block's products are scaled by its per-row scale and added in fp32.
//
// Launch A (k_small_attn), 12 clusters of 8 CTAs, cluster = attention head hd, CTA rank c:
//   x in; LN1 (every CTA, redundantly); QKV
//   rows for dims 8c..8c+7 of q, k and v of the head (24 weight rows) with bias and RoPE,
//   pushed to the head's 8 CTAs; attention over pages c, c+8, ... of each row (online
//   softmax); the CTA's partial result pushed to the 8 CTAs and merged there; proj rows
//   96c..96c+95 over the head's 64 columns added into the accumulator; the CTA's k, v dims
//   appended to the KV cache.
// Launch B (k_small_mlp), 12 clusters of 8 CTAs, CTA j = blockIdx.x (features 32j..32j+31):
//   x in; LN2; fc_in rows 32j.. + bias + gelu_new; fc_out column block j (a partial sum of
//   every output row), each warp's 96 output rows pushed to the CTA that reduces them (CTA c:
//   rows 96c..96c+95); the 8 partials summed in rank order and added into the accumulator.
//
// The residual stream between launches is an int64 accumulator per row element in units of
// 2^-32 (|x| < 2^31), to which the launches add with atomic adds.  Integer addition is
// associative, so the sum does not depend on the order of the adds and every run gives the
// same bits.  Launch p of a step (p = 2 * layer + {0: A, 1: B}) reads x from D[p % 3] (launch
// 0: from the fp32 embedding rows), adds x' = x + its output into D[(p + 1) % 3] -- the CTAs
// that add the biases (head 0, cluster 0) also add x for their rows -- and zeroes
// D[(p + 2) % 3], which launch p + 1 adds into.  After 24 launches D[0] holds the layers'
// output, which the ln_f kernel reads; D[1] is zero again for the next step.
#pragma once

#include "kernels.cuh"
#include "gemm_tc.cuh"
#include "local_fused.cuh"

namespace mossgpu {
namespace {

constexpr int kSlThreads = 256;
constexpr int kSlCluster = 8;
constexpr int kSlMaxRows = 8;
constexpr int kSlCtas = 96;     // both launches: 12 clusters of 8
static_assert(kHeads * kSlCluster == kSlCtas && kFF / 32 == kSlCtas, "layer split");

// Phase stamps (builds with -DMOSSGPU_PHASE_STAMPS only, `bench.py --phase-stamps`): thread 0 of
// every CTA records %globaltimer at each phase boundary of launch p of a step into
// g_sl_stamps[p][CTA][phase]; small_layer_stamps() in engine.cu copies them out.
constexpr int kSlStampLaunches = 2 * kLayers;
constexpr int kSlStampPhases = 12;
#ifdef MOSSGPU_PHASE_STAMPS
__device__ unsigned long long g_sl_stamps[kSlStampLaunches][kSlCtas][kSlStampPhases];
#define SL_STAMP(ph) \
    do { \
        if (threadIdx.x == 0) g_sl_stamps[a.launch][blockIdx.x][ph] = global_ns(); \
    } while (0)
#else
#define SL_STAMP(ph) \
    do { \
    } while (0)
#endif

// (row, page) K/V pairs a CTA of launch A stages in shared memory (4 KB each): as many as let
// it share an SM with a CTA of launch B (its successor's CTAs start beside it)
__host__ __device__ constexpr int sl_kv_slots(int maxr) { return maxr <= 1 ? 12 : maxr <= 2 ? 10 : maxr <= 4 ? 4 : 2; }

struct SmallArgs {
    LfMat attn, proj, fc_in, fc_out;   // fragment records: [rows/16][nb][512] int8, [rows/16][nb][16] fp16
    const float *attn_b, *proj_b, *fc_in_b, *fc_out_b;
    const float *ln_w, *ln_b;   // LN1 (launch A) or LN2 (launch B)
    const float *x0;            // launch 0: the embedding rows [R][768] (fp32)
    const long long *d_in;      // D[p % 3], [8][768] (launches 1..23)
    long long *d_out;           // D[(p + 1) % 3]
    long long *d_zero;          // D[(p + 2) % 3]
    __half *kv;                 // this layer's KV pages
    const int *page_table;
    int pages_per_stream;
    const int *row_slot, *row_pos;
    const float2 *rope;
    int R;
    int launch;                 // p = 2 * layer + half (phase stamps)
};

__device__ __forceinline__ void sl_cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void sl_cp8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void sl_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void sl_cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void sl_st_cluster2(uint32_t addr, float x, float y) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(x), "f"(y) : "memory");
}
__device__ __forceinline__ void sl_st_cluster4(uint32_t addr, float x, float y, float z, float w) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}
__device__ __forceinline__ void sl_st_cluster_h2(uint32_t addr, __half2 h) {
    asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(addr), "r"(*reinterpret_cast<const uint32_t *>(&h)) : "memory");
}
__device__ __forceinline__ void sl_add_fixed(long long *p, long long v) {
    atomicAdd(reinterpret_cast<unsigned long long *>(p), static_cast<unsigned long long>(v));
}

// x of rows < R into xs ([R][768] fp32), and, for a CTA that adds rows base..base+95 of the
// output with their bias (xfix != null), those rows of x as fixed point into xfix[r][96]
__device__ __forceinline__ void sl_residual_in(const SmallArgs &a, float *xs, long long *xfix, int base, int tid) {
    const int R = a.R;
    for (int i = tid; i < R * (kHidden / 4); i += kSlThreads) {
        const int r = i / (kHidden / 4), q4 = i - r * (kHidden / 4);
        const bool mine = xfix && (unsigned)(4 * q4 - base) < 96u;
        long long *f = xfix + r * 96 + 4 * q4 - base;
        float4 v;
        if (a.d_in) {
            const longlong2 *dp = reinterpret_cast<const longlong2 *>(a.d_in + (size_t)r * kHidden) + 2 * q4;
            const longlong2 d0 = dp[0], d1 = dp[1];
            v = make_float4(fixed_to_float(d0.x), fixed_to_float(d0.y), fixed_to_float(d1.x), fixed_to_float(d1.y));
            if (mine) {  // the accumulator's own value, exactly
                f[0] = d0.x;
                f[1] = d0.y;
                f[2] = d1.x;
                f[3] = d1.y;
            }
        } else {
            v = reinterpret_cast<const float4 *>(a.x0 + (size_t)r * kHidden)[q4];
            if (mine) {
                f[0] = float_to_fixed(v.x);
                f[1] = float_to_fixed(v.y);
                f[2] = float_to_fixed(v.z);
                f[3] = float_to_fixed(v.w);
            }
        }
        *reinterpret_cast<float4 *>(xs + r * kHidden + 4 * q4) = v;
    }
}

// column k of activation row r -> its place in an MMA B-operand plane ([8][stride] fp16):
// lf_bpos order, so that a lane's 16-byte load covers both K steps of a 32-column block
__device__ __forceinline__ void sl_act(__half *hi, __half *lo, int stride, int r, int k, float v) {
    const __half h = __float2half_rn(v);
    const int p = r * stride + lf_bpos(k);
    hi[p] = h;
    lo[p] = __float2half_rn(v - __half2float(h));
}

// LayerNorm of rows < R of xs (llm.cpp:159-171) into the hi / lo planes ([8][768]): TPR =
// 256 / MAXR threads a row, each with E = 768 / TPR columns; two reductions (sum, then squared
// deviations) over the thread's columns, the warp and the row's warps (red: 16 floats, the
// sums in the first 8 and the squared deviations in the last 8, so two CTA barriers).  Every
// thread of the CTA calls it.  Plane rows >= R are left as they are: each MMA output column
// depends on its own B column only, and those columns are never read.
template <int MAXR>
__device__ __forceinline__ void sl_layernorm(const float *xs, int R, const float *w, const float *b, float *red,
                                             __half *hi, __half *lo, int tid) {
    constexpr int TPR = kSlThreads / MAXR, WPR = TPR / 32, E = kHidden / TPR;
    const int r = tid / TPR, j = tid - r * TPR, lane = tid & 31, wr = j >> 5;
    const bool on = r < R;
    const float *row = xs + r * kHidden;
    float v[E];
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        v[e] = on ? row[j + e * TPR] : 0.f;
        s += v[e];
    }
    s = warp_sum(s);
    if (WPR > 1) {
        if (lane == 0) red[r * WPR + wr] = s;
        __syncthreads();
        s = 0.f;
#pragma unroll
        for (int q = 0; q < WPR; ++q) s += red[r * WPR + q];
    }
    const float mean = __fdiv_rn(s, (float)kHidden);
    float d2 = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const float d = v[e] - mean;
        d2 = fmaf(d, d, d2);
    }
    d2 = warp_sum(d2);
    if (WPR > 1) {
        if (lane == 0) red[8 + r * WPR + wr] = d2;
        __syncthreads();
        d2 = 0.f;
#pragma unroll
        for (int q = 0; q < WPR; ++q) d2 += red[8 + r * WPR + q];
    }
    const float var = __fdiv_rn(d2, (float)kHidden);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(var + 1e-5f));
    if (on) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int col = j + e * TPR;
            sl_act(hi, lo, kHidden, r, col, __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[e], mean), inv), w[col]), b[col]));
        }
    }
}

// acc[mt][.] = sum over blocks b0 <= b < b1 of scale * (W x) for MT 16-row weight tiles whose
// fragment records are in shared memory (quants rec[mt][nblk][512], scales srec[mt][nblk][16])
// and the 8 activation rows of the hi / lo planes ([8][stride], block b at column 32 b).
// Lane (g, t) = (lane / 4, lane % 4) gets acc[mt] = {(row g, col 2t), (g, 2t + 1), (g + 8, 2t),
// (g + 8, 2t + 1)} of the tile's 16 x 8 result.  Per block, the hi and the lo products of its
// two K steps form two MMA chains from zero, added and scaled in fp32.
template <int MT>
__device__ __forceinline__ void sl_mma(const uint8_t *rec, const __half *srec, int nblk, int b0, int b1,
                                       const __half *act_hi, const __half *act_lo, int stride, int lane,
                                       float (&acc)[MT][4]) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    const __half *bh = act_hi + g * stride + t * 8;
    const __half *bl = act_lo + g * stride + t * 8;
#pragma unroll 2
    for (int b = b0; b < b1; ++b) {
        const int4 xh = lds128(bh + b * 32);
        const int4 xl = lds128(bl + b * 32);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int4 q = lds128(rec + (mt * nblk + b) * 512 + lane * 16);
            const uint32_t s2 = *reinterpret_cast<const uint32_t *>(srec + (mt * nblk + b) * 16 + 2 * g);
            uint32_t a00, a02, a01, a03, a10, a12, a11, a13;
            i8x4_to_h2x2((uint32_t)q.x, a00, a02);  // row g: K step 0 cols 2t.., 2t+8..
            i8x4_to_h2x2((uint32_t)q.z, a01, a03);  // row g+8
            i8x4_to_h2x2((uint32_t)q.y, a10, a12);  // row g: K step 1
            i8x4_to_h2x2((uint32_t)q.w, a11, a13);  // row g+8
            float h0 = 0.f, h1 = 0.f, h2 = 0.f, h3 = 0.f, l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
            mma16816(h0, h1, h2, h3, a00, a01, a02, a03, (uint32_t)xh.x, (uint32_t)xh.y);
            mma16816(l0, l1, l2, l3, a00, a01, a02, a03, (uint32_t)xl.x, (uint32_t)xl.y);
            mma16816(h0, h1, h2, h3, a10, a11, a12, a13, (uint32_t)xh.z, (uint32_t)xh.w);
            mma16816(l0, l1, l2, l3, a10, a11, a12, a13, (uint32_t)xl.z, (uint32_t)xl.w);
            const float2 sc = __half22float2(*reinterpret_cast<const __half2 *>(&s2));
            acc[mt][0] = fmaf(sc.x, h0 + l0, acc[mt][0]);
            acc[mt][1] = fmaf(sc.x, h1 + l1, acc[mt][1]);
            acc[mt][2] = fmaf(sc.y, h2 + l2, acc[mt][2]);
            acc[mt][3] = fmaf(sc.y, h3 + l3, acc[mt][3]);
        }
    }
}

// copy n 16-byte chunks from src to dst (shared), thread-strided
__device__ __forceinline__ void sl_copy(uint8_t *dst, const void *src, int n, int tid) {
    for (int i = tid; i < n; i += kSlThreads) sl_cp16(dst + i * 16, reinterpret_cast<const uint8_t *>(src) + i * 16);
}

// ------------------------------------------------------------------ launch A: attention half

template <int MAXR>
struct SlAttnSmem {
    static constexpr int kSlots = sl_kv_slots(MAXR);
    static constexpr int wq = 0;                               // records [3 tiles: q, k, v][24 blocks][512]
    static constexpr int wqs = wq + 3 * 24 * 512;              // half [3][24][16]
    static constexpr int wp = wqs + 3 * 24 * 32;               // records [6 tiles][2 blocks][512] (proj)
    static constexpr int wps = wp + 6 * 2 * 512;               // half [6][2][16]
    static constexpr int lnw = wps + 6 * 2 * 32;               // float [768] LN1 weight, bias
    static constexpr int lnb = lnw + kHidden * 4;
    static constexpr int bq = lnb + kHidden * 4;               // float [24] QKV bias of the CTA's dims (q, k, v)
    static constexpr int bp = bq + 24 * 4;                     // float [96] proj bias of its rows
    static constexpr int rs = bp + 96 * 4;                     // float2 [8][4] RoPE (cos, sin)
    static constexpr int meta = rs + kSlMaxRows * 4 * 8;       // int [5][8]: pos, slot, pages, first item, page of pos
    static constexpr int red = meta + 5 * kSlMaxRows * 4;      // float [16] LayerNorm partial sums
    static constexpr int xs = red + 16 * 4;                    // float [MAXR][768] x
    static constexpr int xfix = xs + MAXR * kHidden * 4;       // int64 [MAXR][96] x of the proj rows (head 0)
    static constexpr int act = xfix + MAXR * 96 * 8;           // half [2][8][768] LN1(x) hi, lo; then QKV
                                                               // partials; then [8 CTAs][MAXR][68] attention partials
    static constexpr int own = act + 2 * 8 * kHidden * 2;      // float [MAXR][24] q, k, v dims 8c..8c+7
    static constexpr int full = own + MAXR * 24 * 4;           // float [MAXR][192] the head's q | k | v
    static constexpr int newkv = full + MAXR * 192 * 4;        // half [MAXR][2][64] k, v of the new position
    static constexpr int wst = newkv + MAXR * 256;             // float [8 warps][68] m, l, -, -, o[64]
    static constexpr int ohp = wst + 8 * kPartStride * 4;      // half [2][8][64] attention output hi, lo
    static constexpr int kvs = ohp + 2 * 8 * kHeadDim * 2;     // half [slots][k|v][16][64]
    static constexpr int total = kvs + kSlots * 4096;
    static_assert(rs % 16 == 0 && xs % 16 == 0 && xfix % 16 == 0 && act % 16 == 0 && own % 16 == 0 && full % 16 == 0 &&
                      newkv % 16 == 0 && ohp % 16 == 0 && kvs % 16 == 0,
                  "16-byte aligned regions");
    static_assert(8 * 3 * 128 * 4 <= 2 * 8 * kHidden * 2 && kSlCluster * MAXR * kPartStride * 4 <= 2 * 8 * kHidden * 2,
                  "QKV partials and the cluster's attention partials fit the activation planes");
};

template <int MAXR>
__global__ void __launch_bounds__(kSlThreads) k_small_attn(const SmallArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    using S = SlAttnSmem<MAXR>;
    uint8_t *sm = smem_raw;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = (int)cluster_rank();
    const int hd = blockIdx.x / kSlCluster;
    const int R = a.R;
    int *m_pos = reinterpret_cast<int *>(sm + S::meta);
    int *m_slot = m_pos + kSlMaxRows, *m_cnt = m_pos + 2 * kSlMaxRows, *m_first = m_pos + 3 * kSlMaxRows;
    int *m_page = m_pos + 4 * kSlMaxRows;
    float *xs = reinterpret_cast<float *>(sm + S::xs);
    long long *xfix = reinterpret_cast<long long *>(sm + S::xfix);
    __half *act_hi = reinterpret_cast<__half *>(sm + S::act), *act_lo = act_hi + 8 * kHidden;
    float *qred = reinterpret_cast<float *>(sm + S::act);  // [8 warps][3][128], after the QKV MMAs
    float *precv = reinterpret_cast<float *>(sm + S::act);  // [8 CTAs][MAXR][68], after cluster barrier 1
    float *own = reinterpret_cast<float *>(sm + S::own);
    float *full = reinterpret_cast<float *>(sm + S::full);
    __half *newkv = reinterpret_cast<__half *>(sm + S::newkv);
    float *wst = reinterpret_cast<float *>(sm + S::wst);
    __half *oh_hi = reinterpret_cast<__half *>(sm + S::ohp), *oh_lo = oh_hi + 8 * kHeadDim;
    const float *bq = reinterpret_cast<const float *>(sm + S::bq);
    const float *bp = reinterpret_cast<const float *>(sm + S::bp);
    const float2 *rs = reinterpret_cast<const float2 *>(sm + S::rs);
    SL_STAMP(0);
    cluster_arrive_relaxed();  // this CTA runs: matched by the wait before its first remote store

    // ---- 0. before the wait: everything that does not depend on the previous launch.  The
    //      per-row control (slot, position, page table) was written by the host or by a kernel
    //      at least two launches back, so it is visible here as the weights are.
    if (tid < kSlMaxRows) {
        int pos = 0, slot = 0, cnt = 0, page = 0;
        if (tid < R) {
            pos = a.row_pos[tid];
            slot = a.row_slot[tid];
            const int last = pos / kPage;
            cnt = c <= last ? (last - c) / kSlCluster + 1 : 0;  // pages c, c + 8, ... <= last
            page = a.page_table[(size_t)slot * a.pages_per_stream + last];
        }
        m_pos[tid] = pos;
        m_slot[tid] = slot;
        m_cnt[tid] = cnt;
        m_page[tid] = page;
    }
    // QKV: the 16-row tiles holding q, k and v dims 8c..8c+7 of the head (rows 8 (c & 1) ..
    // of tile 4 hd + c / 2, + 48, + 96), all 24 blocks of each (contiguous records)
    const int tq = 4 * hd + (c >> 1);
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        const size_t tile = (size_t)(tq + 48 * m);
        sl_copy(sm + S::wq + m * 24 * 512, a.attn.qm + tile * 24 * 512, 24 * 32, tid);
        sl_copy(sm + S::wqs + m * 24 * 32, a.attn.sm + tile * 24 * 16, 48, tid);
    }
    // proj: tiles 6c..6c+5 (rows 96c..96c+95), blocks 2hd, 2hd + 1 (the head's 64 columns)
    for (int i = tid; i < 6 * 64; i += kSlThreads) {
        const int m = i >> 6, ch = i & 63;
        const size_t rec = (size_t)(6 * c + m) * (kHidden / 32) + 2 * hd;
        sl_cp16(sm + S::wp + m * 1024 + ch * 16, a.proj.qm + rec * 512 + ch * 16);
    }
    if (tid < 24) {
        const size_t rec = (size_t)(6 * c + (tid >> 2)) * (kHidden / 32) + 2 * hd;
        sl_cp16(sm + S::wps + tid * 16, reinterpret_cast<const uint8_t *>(a.proj.sm + rec * 16) + (tid & 3) * 16);
    }
    sl_copy(sm + S::lnw, a.ln_w, kHidden / 4, tid);
    sl_copy(sm + S::lnb, a.ln_b, kHidden / 4, tid);
    if (tid < 6) {  // QKV bias: rows part * 768 + hd * 64 + 8c + 4 (tid & 1) ..
        const int off = (tid >> 1) * kHidden + hd * kHeadDim + 8 * c + 4 * (tid & 1);
        sl_cp16(sm + S::bq + tid * 16, a.attn_b + off);
    } else if (tid < 30) {
        sl_cp16(sm + S::bp + (tid - 6) * 16, a.proj_b + 96 * c + 4 * (tid - 6));
    }
    __syncthreads();  // m_* written
    if (tid < MAXR * 4) {  // RoPE factors of the CTA's 4 q/k pairs (pair index 4c..4c+3)
        const int r = tid >> 2;
        if (r < R) sl_cp8(sm + S::rs + tid * 8, a.rope + (size_t)m_pos[r] * (kHeadDim / 2) + 4 * c + (tid & 3));
    }
    if (tid == 0) {
        int first = 0;
        for (int r = 0; r < kSlMaxRows; ++r) {
            m_first[r] = first;
            first += m_cnt[r];
        }
    }
    // the rows' cached K/V pages of this CTA (item t = (row, page c + 8i), row-major): the
    // head's 2 KB of k and 2 KB of v per page; the page holding the new position is stale
    // at that position, which is never read from here
    {
        int t = 0;
        for (int r = 0; r < R && t < S::kSlots; ++r) {
            const int cnt = m_cnt[r];
            for (int i = 0; i < cnt && t < S::kSlots; ++i, ++t) {
                const int page = a.page_table[(size_t)m_slot[r] * a.pages_per_stream + c + kSlCluster * i];
                const __half *src = a.kv + (size_t)page * kPageHalfs + (size_t)((tid >> 7) * kHeads + hd) * kPage * kHeadDim;
                sl_cp16(sm + S::kvs + t * 4096 + tid * 16, reinterpret_cast<const uint8_t *>(src) + (tid & 127) * 16);
            }
        }
    }
    sl_cp_commit();
    SL_STAMP(1);

    pdl_wait();
    pdl_trigger();
    SL_STAMP(2);

    // ---- 1. x in (head 0 keeps its proj rows of x for the accumulator), LN1 into the planes
    sl_residual_in(a, xs, hd == 0 ? xfix : nullptr, 96 * c, tid);
    sl_cp_wait_all();
    __syncthreads();
    sl_layernorm<MAXR>(xs, R, reinterpret_cast<const float *>(sm + S::lnw), reinterpret_cast<const float *>(sm + S::lnb),
                       reinterpret_cast<float *>(sm + S::red), act_hi, act_lo, tid);
    __syncthreads();
    SL_STAMP(3);

    // ---- 2. QKV: warp w takes blocks 3w..3w+2 of the three tiles; the 8 partial sums are
    //      added in warp order, then bias and RoPE (pairs 2i, 2i+1 of q and k; EPI_QKV order)
    {
        float acc[3][4];
        sl_mma<3>(sm + S::wq, reinterpret_cast<const __half *>(sm + S::wqs), 24, 3 * warp, 3 * warp + 3, act_hi, act_lo,
                  kHidden, lane, acc);
        __syncthreads();  // every warp is done with the planes, which now take the partials
#pragma unroll
        for (int m = 0; m < 3; ++m)
            *reinterpret_cast<float4 *>(qred + (warp * 3 + m) * 128 + lane * 4) =
                make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
    }
    __syncthreads();
    cluster_wait();  // every CTA of the cluster runs: its shared memory may be written
    // item (row r, part m, dim pair i0) for destination CTA d: the 8 warps' partial sums added in
    // warp order, bias, RoPE; then pushed into CTA d (each destination's thread recomputes it)
    for (int it = tid; it < kSlCluster * 12 * R; it += kSlThreads) {
        const int d = it & (kSlCluster - 1), k = it >> 3;
        const int r = k / 12, e = k - r * 12;
        const int m = e >> 2, i0 = (e & 3) * 2;   // tile (q, k, v), first dim of the pair
        const int j = 2 * (c & 1) + (r & 1);      // fragment slot: row half, column parity
        float v0 = 0.f, v1 = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            v0 += qred[(w * 3 + m) * 128 + (4 * i0 + (r >> 1)) * 4 + j];
            v1 += qred[(w * 3 + m) * 128 + (4 * (i0 + 1) + (r >> 1)) * 4 + j];
        }
        v0 = __fadd_rn(v0, bq[m * 8 + i0]);
        v1 = __fadd_rn(v1, bq[m * 8 + i0 + 1]);
        float o0 = v0, o1 = v1;
        if (m < 2) {
            const float2 cs = rs[r * 4 + (i0 >> 1)];
            o0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
            o1 = __fadd_rn(__fmul_rn(v1, cs.x), __fmul_rn(v0, cs.y));
        }
        if (d == c) {
            own[r * 24 + m * 8 + i0] = o0;
            own[r * 24 + m * 8 + i0 + 1] = o1;
        }
        // ---- 3. q, k, v dims 8c + i0, 8c + i0 + 1 of row r into CTA d, and the new position's
        //      k, v as the cache holds them (fp16)
        sl_st_cluster2(cluster_map(smem_u32(full + r * 192 + m * kHeadDim + c * 8 + i0), (uint32_t)d), o0, o1);
        if (m > 0)
            sl_st_cluster_h2(cluster_map(smem_u32(newkv + r * 128 + (m - 1) * kHeadDim + c * 8 + i0), (uint32_t)d),
                             __floats2half2_rn(o0, o1));
    }
    SL_STAMP(4);
    cluster_arrive();  // release: this thread's pushes
    cluster_wait();    // acquire: every CTA's pushes are visible
    SL_STAMP(5);
    // ---- 4. attention over this CTA's pages: warp w takes row w / WPR, items sub, sub + WPR,
    //      ...; lanes as in k_attn_rows (8 lanes a position, 8 dims a lane, 4 positions a step)
    constexpr int WPR = 8 / MAXR;
    {
        const int r = warp / WPR, sub = warp - r * WPR;
        const int ps = lane >> 3, ds = lane & 7;
        float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = 0.f;
        if (r < R) {
            const int pos = m_pos[r];
            float qv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) qv[j] = full[r * 192 + ds * 8 + j] * 0.125f;
            const int4 nk = *reinterpret_cast<const int4 *>(newkv + r * 128 + ds * 8);
            const int4 nv = *reinterpret_cast<const int4 *>(newkv + r * 128 + kHeadDim + ds * 8);
            const __half *kvs = reinterpret_cast<const __half *>(sm + S::kvs);
            for (int i = sub; i < m_cnt[r]; i += WPR) {
                const int pg = c + kSlCluster * i;
                const int t = m_first[r] + i;
                const __half *kb, *vb;
                if (t < S::kSlots) {
                    kb = kvs + (size_t)t * 2048;
                    vb = kb + kPage * kHeadDim;
                } else {
                    const int page = a.page_table[(size_t)m_slot[r] * a.pages_per_stream + pg];
                    kb = a.kv + (size_t)page * kPageHalfs + (size_t)hd * kPage * kHeadDim;
                    vb = kb + (size_t)kHeads * kPage * kHeadDim;
                }
                kb += ds * 8;
                vb += ds * 8;
                const int pb = pg * kPage;
                int4 kr[4], vr[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int p = pb + ps + 4 * u;
                    if (p < pos) {
                        kr[u] = *reinterpret_cast<const int4 *>(kb + (ps + 4 * u) * kHeadDim);
                        vr[u] = *reinterpret_cast<const int4 *>(vb + (ps + 4 * u) * kHeadDim);
                    } else if (p == pos) {
                        kr[u] = nk;
                        vr[u] = nv;
                    } else {
                        kr[u] = make_int4(0, 0, 0, 0);
                        vr[u] = make_int4(0, 0, 0, 0);
                    }
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
                    if (pb + ps + 4 * u > pos) sc[u] = -INFINITY;
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
        }
        // merge the warp's 4 position groups (lanes ds, ds + 8, ds + 16, ds + 24)
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
            float *w = wst + warp * kPartStride;
            if (lane == 0) {
                w[0] = m;
                w[1] = l;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) w[4 + ds * 8 + j] = o[j];
        }
    }
    __syncthreads();
    // the CTA's partial of each row: its WPR warps merged (a warp with no page: m = -inf), pushed
    // into slot c of every CTA's partials (the activation planes are free in every CTA once it
    // passed cluster barrier 1)
    for (int i = tid; i < R * kHeadDim; i += kSlThreads) {
        const int r = i / kHeadDim, d = i - r * kHeadDim;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < WPR; ++w) M = fmaxf(M, wst[(r * WPR + w) * kPartStride]);
        float L = 0.f, y = 0.f;
#pragma unroll
        for (int w = 0; w < WPR; ++w) {
            const float *ws = wst + (r * WPR + w) * kPartStride;
            const float wgt = ws[0] == -INFINITY ? 0.f : __expf(ws[0] - M);
            L = fmaf(ws[1], wgt, L);
            y = fmaf(ws[4 + d], wgt, y);
        }
        const uint32_t pa = smem_u32(precv + (c * MAXR + r) * kPartStride);
#pragma unroll
        for (int dst = 0; dst < kSlCluster; ++dst) {
            const uint32_t ra = cluster_map(pa, (uint32_t)dst);
            if (d == 0) sl_st_cluster2(ra, M, L);
            st_cluster_f32(ra + 16 + 4 * d, y);
        }
    }
    SL_STAMP(6);
    cluster_arrive();  // release: this thread's pushes
    cluster_wait();    // acquire: the 8 partials of every row are here
    SL_STAMP(7);

    // ---- 5. the 8 CTAs' partials merged (every CTA, for its proj rows) into the planes
    for (int i = tid; i < R * kHeadDim; i += kSlThreads) {
        const int r = i / kHeadDim, d = i - r * kHeadDim;
        float pm[kSlCluster], pl[kSlCluster], po[kSlCluster];
        float M = -INFINITY;
#pragma unroll
        for (int s = 0; s < kSlCluster; ++s) {
            const float *ps = precv + (s * MAXR + r) * kPartStride;
            pm[s] = ps[0];
            pl[s] = ps[1];
            po[s] = ps[4 + d];
            M = fmaxf(M, pm[s]);
        }
        float L = 0.f, y = 0.f;
#pragma unroll
        for (int s = 0; s < kSlCluster; ++s) {
            const float wgt = pm[s] == -INFINITY ? 0.f : __expf(pm[s] - M);
            L = fmaf(pl[s], wgt, L);
            y = fmaf(po[s], wgt, y);
        }
        sl_act(oh_hi, oh_lo, kHeadDim, r, d, y / L);
    }
    __syncthreads();
    SL_STAMP(8);

    // ---- 6. proj rows 96c..96c+95 over the head's 64 columns (warp w: tile 6c + w) into the
    //      accumulator (head 0 adds x and the bias); then this CTA's global stores: its k, v
    //      dims of the new position into the KV cache, its 8 columns of D[(p + 2) % 3]
    if (warp < 6) {
        float acc[1][4];
        sl_mma<1>(sm + S::wp + warp * 1024, reinterpret_cast<const __half *>(sm + S::wps) + warp * 32, 2, 0, 2, oh_hi,
                  oh_lo, kHeadDim, lane, acc);
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = 2 * t + (j & 1), ol = 16 * warp + g + 8 * (j >> 1);
            if (n < R) {
                long long f = float_to_fixed(acc[0][j]);
                if (hd == 0) f += float_to_fixed(bp[ol]) + xfix[n * 96 + ol];
                sl_add_fixed(a.d_out + (size_t)n * kHidden + 96 * c + ol, f);
            }
        }
    } else if (tid < 192 + 2 * R) {
        const int r = (tid - 192) >> 1, kvsel = tid & 1;
        const float *v = own + r * 24 + (1 + kvsel) * 8;
        __half2 h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
        __half *dst = a.kv + (size_t)m_page[r] * kPageHalfs +
                      ((size_t)(kvsel * kHeads + hd) * kPage + m_pos[r] % kPage) * kHeadDim + 8 * c;
        *reinterpret_cast<int4 *>(dst) = *reinterpret_cast<const int4 *>(h);
    } else if (tid >= 224 && tid < 224 + R * 8 / 2) {
        const int i = tid - 224;  // 2 columns a thread
        long long *z = a.d_zero + (size_t)(i >> 2) * kHidden + blockIdx.x * 8 + 2 * (i & 3);
        z[0] = 0;
        z[1] = 0;
    }
    SL_STAMP(9);
    SL_STAMP(10);
}

// ------------------------------------------------------------------ launch B: MLP half

template <int MAXR>
struct SlMlpSmem {
    static constexpr int wi = 0;                          // records [2 tiles][24 blocks][512]: fc_in rows 32j..
    static constexpr int wis = wi + 2 * 24 * 512;         // half [2][24][16]
    static constexpr int wo = wis + 2 * 24 * 32;          // records [48 tiles][512]: fc_out block j
    static constexpr int wos = wo + 48 * 512;             // half [48][16]
    static constexpr int lnw = wos + 48 * 32;             // float [768] LN2 weight, bias
    static constexpr int lnb = lnw + kHidden * 4;
    static constexpr int bi = lnb + kHidden * 4;          // float [32] fc_in bias of the CTA's features
    static constexpr int bo = bi + 32 * 4;                // float [96] fc_out bias of its reduce rows
    static constexpr int red = bo + 96 * 4;               // float [16] LayerNorm partial sums
    static constexpr int xs = red + 16 * 4;               // float [MAXR][768] x
    static constexpr int xfix = xs + MAXR * kHidden * 4;  // int64 [MAXR][96] x of the reduce rows (cluster 0)
    static constexpr int act = xfix + MAXR * 96 * 8;      // half [2][8][768] LN2(x) hi, lo; then fc_in partials
                                                          // [8 warps][2][128] float
    static constexpr int hpl = act + 2 * 8 * kHidden * 2; // half [2][8][32] gelu(fc_in) hi, lo
    static constexpr int orecv = hpl + 2 * 8 * 32 * 2;    // float [8 CTAs][MAXR][8 g][12 (m, h)]: fc_out
                                                          // partials of the CTA's reduce row 16 m + g + 8 h,
                                                          // pushed by the cluster's CTAs
    static constexpr int total = orecv + kSlCluster * MAXR * 96 * 4;
    static_assert(xs % 16 == 0 && xfix % 16 == 0 && act % 16 == 0 && hpl % 16 == 0 && orecv % 16 == 0 && bi % 16 == 0 && bo % 16 == 0,
                  "16-byte aligned regions");
};

template <int MAXR>
__global__ void __launch_bounds__(kSlThreads) k_small_mlp(const SmallArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    using S = SlMlpSmem<MAXR>;
    constexpr int RPT = (MAXR * 96 + kSlThreads - 1) / kSlThreads;  // reduce outputs a thread
    uint8_t *sm = smem_raw;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = (int)cluster_rank();
    const int j = blockIdx.x;  // feature block: fc_in rows 32j..32j+31, fc_out columns 32j..
    const bool first_cluster = blockIdx.x < kSlCluster;  // adds x and the bias of its reduce rows
    const int R = a.R;
    float *xs = reinterpret_cast<float *>(sm + S::xs);
    long long *xfix = reinterpret_cast<long long *>(sm + S::xfix);
    __half *act_hi = reinterpret_cast<__half *>(sm + S::act), *act_lo = act_hi + 8 * kHidden;
    float *fred = reinterpret_cast<float *>(sm + S::act);   // [8 warps][2][128], after the fc_in MMAs
    float *orecv = reinterpret_cast<float *>(sm + S::orecv);
    __half *h_hi = reinterpret_cast<__half *>(sm + S::hpl), *h_lo = h_hi + 8 * 32;
    SL_STAMP(0);
    cluster_arrive_relaxed();  // this CTA runs: matched by the wait before its first remote store

    // ---- 0. before the wait: weights, LN2, biases
    sl_copy(sm + S::wi, a.fc_in.qm + (size_t)2 * j * 24 * 512, 2 * 24 * 32, tid);  // tiles 2j, 2j + 1: contiguous
    sl_copy(sm + S::wis, a.fc_in.sm + (size_t)2 * j * 24 * 16, 2 * 24 * 2, tid);
    for (int i = tid; i < 48 * 32; i += kSlThreads) {  // block j of every fc_out tile
        const int m = i >> 5, ch = i & 31;
        sl_cp16(sm + S::wo + m * 512 + ch * 16, a.fc_out.qm + ((size_t)m * (kFF / 32) + j) * 512 + ch * 16);
    }
    if (tid < 96)
        sl_cp16(sm + S::wos + tid * 16,
                reinterpret_cast<const uint8_t *>(a.fc_out.sm + ((size_t)(tid >> 1) * (kFF / 32) + j) * 16) + (tid & 1) * 16);
    sl_copy(sm + S::lnw, a.ln_w, kHidden / 4, tid);
    sl_copy(sm + S::lnb, a.ln_b, kHidden / 4, tid);
    if (tid < 8) sl_cp16(sm + S::bi + tid * 16, a.fc_in_b + 32 * j + 4 * tid);
    else if (tid < 32) sl_cp16(sm + S::bo + (tid - 8) * 16, a.fc_out_b + 96 * c + 4 * (tid - 8));
    sl_cp_commit();
    SL_STAMP(1);

    pdl_wait();
    pdl_trigger();
    SL_STAMP(2);

    // ---- 1. x in (cluster 0 keeps its reduce rows of x for the accumulator), LN2 into the planes
    sl_residual_in(a, xs, first_cluster ? xfix : nullptr, 96 * c, tid);
    sl_cp_wait_all();
    __syncthreads();
    sl_layernorm<MAXR>(xs, R, reinterpret_cast<const float *>(sm + S::lnw), reinterpret_cast<const float *>(sm + S::lnb),
                       reinterpret_cast<float *>(sm + S::red), act_hi, act_lo, tid);
    __syncthreads();
    SL_STAMP(3);

    // ---- 2. fc_in: warp w takes blocks 3w..3w+2 of both tiles; the 8 partial sums added in
    //      warp order, + bias, gelu_new, into the h planes (fc_out's B operand)
    {
        float acc[2][4];
        sl_mma<2>(sm + S::wi, reinterpret_cast<const __half *>(sm + S::wis), 24, 3 * warp, 3 * warp + 3, act_hi, act_lo,
                  kHidden, lane, acc);
        __syncthreads();  // every warp is done with the planes, which now take the partials
#pragma unroll
        for (int m = 0; m < 2; ++m)
            *reinterpret_cast<float4 *>(fred + (warp * 2 + m) * 128 + lane * 4) =
                make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
    }
    __syncthreads();
    if (tid < 32 * R) {
        const int r = tid >> 5, f = tid & 31;   // batch row, feature 32j + f
        const int m = f >> 4, row = f & 15;
        const int slot = (row & 7) * 16 + (r >> 1) * 4 + 2 * (row >> 3) + (r & 1);
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += fred[(w * 2 + m) * 128 + slot];
        sl_act(h_hi, h_lo, 32, r, f, gelu_new(__fadd_rn(v, reinterpret_cast<const float *>(sm + S::bi)[f])));
    }
    __syncthreads();
    SL_STAMP(4);

    // ---- 3. fc_out over the 32 features: warp w takes tiles 6w..6w+5 (output rows 96w..96w+95,
    //      which CTA w of the cluster reduces) and pushes its partial sums into slot c of that
    //      CTA's orecv
    cluster_wait();  // every CTA of the cluster runs: its shared memory may be written
    {
        float acc[6][4];
        sl_mma<6>(sm + S::wo + warp * 6 * 512, reinterpret_cast<const __half *>(sm + S::wos) + warp * 6 * 16, 1, 0, 1,
                  h_hi, h_lo, 32, lane, acc);
        // lane (g, t) holds rows 16 m + g + 8 h of batch rows 2t, 2t + 1: 12 contiguous floats
        // a batch row, three 16-byte remote stores
        const int g = lane >> 2, t = lane & 3;
        const uint32_t dst = cluster_map(smem_u32(orecv + c * MAXR * 96 + g * 12), (uint32_t)warp);
#pragma unroll
        for (int par = 0; par < 2; ++par) {
            const int n = 2 * t + par;
            if (n < R) {
                const uint32_t ra = dst + (uint32_t)(n * 96 * 4);
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    sl_st_cluster4(ra + 16 * k, acc[2 * k][par], acc[2 * k][2 + par], acc[2 * k + 1][par],
                                   acc[2 * k + 1][2 + par]);
            }
        }
    }
    SL_STAMP(5);
    cluster_arrive();  // release: this thread's pushes
    cluster_wait();    // acquire: the 8 partials of the CTA's rows are here
    SL_STAMP(6);

    // ---- 4. the cluster's 8 partials of rows 96c..96c+95, summed in rank order, into the
    //      accumulator (cluster 0 adds x and the bias), and this CTA's 8 columns of
    //      D[(p + 2) % 3] zeroed
    float sum[RPT];
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
        const int i = tid + q * kSlThreads;
        sum[q] = 0.f;
        if (i < R * 96) {
            const int r = i / 96, ol = i - r * 96;
#pragma unroll
            const int m = ol >> 4, g = ol & 7, h = (ol >> 3) & 1;
#pragma unroll
            for (int src = 0; src < kSlCluster; ++src) sum[q] += orecv[(src * MAXR + r) * 96 + g * 12 + 2 * m + h];
        }
    }
    SL_STAMP(7);
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
        const int i = tid + q * kSlThreads;
        if (i < R * 96) {
            const int r = i / 96, ol = i - r * 96;
            long long f = float_to_fixed(sum[q]);
            if (first_cluster) f += float_to_fixed(reinterpret_cast<const float *>(sm + S::bo)[ol]) + xfix[r * 96 + ol];
            sl_add_fixed(a.d_out + (size_t)r * kHidden + 96 * c + ol, f);
        }
    }
    if (tid < R * 8) a.d_zero[(size_t)(tid >> 3) * kHidden + blockIdx.x * 8 + (tid & 7)] = 0;
    SL_STAMP(8);
    SL_STAMP(9);
}

}  // namespace
}  // namespace mossgpu

namespace mossgpu {
namespace {
// a CTA of launch A and one of launch B fit on one SM (228 KB of shared memory, 1 KB reserved
// per CTA) up to 4 rows, so each launch's CTAs start beside its predecessor's
static_assert(SlAttnSmem<1>::total + SlMlpSmem<1>::total + 2048 <= 228 * 1024 &&
                  SlAttnSmem<2>::total + SlMlpSmem<2>::total + 2048 <= 228 * 1024 &&
                  SlAttnSmem<4>::total + SlMlpSmem<4>::total + 2048 <= 228 * 1024,
              "launch A and B share an SM");
}  // namespace
}  // namespace mossgpu
