// attn_tc.cuh -- causal flash-prefill attention on the 5th-generation tensor cores, sm_100a.
//
// LlmModel::prefill's attention (llm.cpp:360-384; the score scale 1/8 = 1/sqrt(64)) for a
// prefill pass whose rows are runs of consecutive positions of one stream.  One CTA = one head
// and a tile of up to 128 consecutive rows of one stream (thread i = query row i = TMEM lane i);
// it walks the stream's keys [0, last position] in blocks of 64 positions:
//   - the block's K and V rows (128 B each, from the paged fp16 cache) are copied into shared
//     memory in the SWIZZLE_128B layout, one 128-byte row per position;
//   - S = Q K^T: 8 tcgen05.mma (M = 128, N = 64, K = 16) into TMEM, Q split into fp16 hi + lo
//     parts (q/8 = hi + lo, K exact in fp16), so the scores carry ~fp32 accuracy;
//   - each thread reads its row of S (64 fp32), masks positions after its own, updates the
//     running max / sum (online softmax in fp32) and writes P = exp(s - max) as fp16 hi + lo
//     into shared memory (the A operand of the next MMA);
//   - O_blk = P V: 8 tcgen05.mma with V as an MN-major B operand (the same position-major rows),
//     into a second TMEM region; each thread rescales its register accumulator o[64] and adds
//     its row of O_blk.
// The output o / l goes into the next GEMM's activation image (hi and lo parts).  K and V blocks
// are double-buffered: the asynchronous copies (cp.async, 16 B each, into the swizzled rows) of
// block b + 1 run while block b's MMAs and softmax do.  Two CTAs share an SM (~97 KB of shared
// memory and 128 TMEM columns each).  Every mbarrier
// wait is bounded; a time-out records an error code and the CTA leaves through the normal exit.
#pragma once

#include "gemm_tc.cuh"

namespace mossgpu {
namespace {

constexpr int kPtRows = 128;                      // query rows per CTA
constexpr int kPtBlk = 64;                        // key positions per block
constexpr int kPtThreads = 128;
constexpr int kPtTile = kPtRows * 128;            // a 128-row x 128-byte operand tile (16 KB)
constexpr int kPtKvTile = kPtBlk * 128;           // a 64-row x 128-byte K or V block (8 KB)
constexpr int kPtSmem = 4 * kPtTile + 4 * kPtKvTile + 1024;  // Q hi/lo, P hi/lo, 2 x (K, V) (+align)

// item = {first row, rows (<= 128), position of the first row, stream slot}
struct PtArgs {
    const float *q;           // [R][768]
    const __half *kv;         // layer base of the paged KV
    const int *page_table;
    int pages_per_stream;
    const int4 *items;
    uint8_t *bimg;            // activation image of the proj GEMM (N rows, parts)
    int bimg_N, bimg_parts;
    int *err;
};

// 16 fp32 values (one 8-element unit pair) -> swizzled 128-byte row `row` of a K-major tile:
// element k of the row at unit (k / 8) ^ (row % 8)
__device__ __forceinline__ void pt_store_row_unit(uint8_t *tile, int row, int unit, const __half *h8) {
    *reinterpret_cast<int4 *>(tile + row * 128 + ((unit ^ (row & 7)) << 4)) = *reinterpret_cast<const int4 *>(h8);
}

__device__ __forceinline__ void pt_ld16_nowait(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// a row of 64 fp32 values of TMEM region `col` (this thread's lane)
__device__ __forceinline__ void pt_ld_row64(uint32_t tmem, int warp, int col, float *v) {
    __syncwarp();
    uint32_t r[64];
    const uint32_t base = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)col;
    pt_ld16_nowait(base, r);
    pt_ld16_nowait(base + 16, r + 16);
    pt_ld16_nowait(base + 32, r + 32);
    pt_ld16_nowait(base + 48, r + 48);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kPtThreads, 2) k_attn_prefill_tc(const PtArgs a) {
    extern __shared__ uint8_t pt_smem_raw[];
    __shared__ __align__(8) uint64_t mma_bar;
    __shared__ uint32_t tmem_sh;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(pt_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *q_hi = smem, *q_lo = smem + kPtTile, *p_hi = smem + 2 * kPtTile, *p_lo = smem + 3 * kPtTile;
    uint8_t *kv_buf = smem + 4 * kPtTile;  // [2][K block, V block]
    const int tid = threadIdx.x, warp = tid >> 5;
    const int hd = blockIdx.y;
    const int4 it = a.items[blockIdx.x];
    const int row0 = it.x, nrows = it.y, pos0 = it.z, slot = it.w;
    const int end = pos0 + nrows;                  // keys [0, end)
    const int nblk = (end + kPtBlk - 1) / kPtBlk;

    if (tid == 0) {
        mbar_init(&mma_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(128));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    pdl_enter();
    // query row tid: q / 8 split into fp16 hi + lo (rows past the tile: zeros)
    {
        float qv[64];
        if (tid < nrows) {
            const float4 *qp = reinterpret_cast<const float4 *>(a.q + (size_t)(row0 + tid) * kHidden + hd * kHeadDim);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float4 x = qp[j];
                qv[4 * j] = x.x * 0.125f;
                qv[4 * j + 1] = x.y * 0.125f;
                qv[4 * j + 2] = x.z * 0.125f;
                qv[4 * j + 3] = x.w * 0.125f;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) qv[j] = 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            __align__(16) __half h[8], l[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                h[e] = __float2half_rn(qv[8 * u + e]);
                l[e] = __float2half_rn(qv[8 * u + e] - __half2float(h[e]));
            }
            pt_store_row_unit(q_hi, tid, u, h);
            pt_store_row_unit(q_lo, tid, u, l);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_sh;
    const uint32_t t_s = tmem, t_o = tmem + 64;   // S and O_blk regions (64 columns each)
    // S: M = 128, N = 64 keys; PV: M = 128, N = 64 dims with V MN-major (bit 16)
    const uint32_t idesc_s = (1u << 4) | ((uint32_t)(kPtBlk >> 3) << 17) | ((uint32_t)(kPtRows >> 4) << 24);
    const uint32_t idesc_pv = idesc_s | (1u << 16);
    const int my_lim = tid < nrows ? pos0 + tid + 1 : 0;  // keys < my_lim are visible to this row
    float o[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) o[j] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    const __half *kbase = a.kv + (size_t)hd * kPage * kHeadDim;                    // K of head hd in a page
    const __half *vbase = a.kv + (size_t)(kHeads + hd) * kPage * kHeadDim;         // V of head hd
    // K and V rows of positions 64 b .. 64 b + 63 -> swizzled 128-byte rows of buffer b & 1
    auto copy_block = [&](int b) {
        uint8_t *kt = kv_buf + (b & 1) * 2 * kPtKvTile, *vt = kt + kPtKvTile;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int j = tid + kPtThreads * k;   // 512 units of 16 B per block: row j / 8, unit j % 8
            const int r = j >> 3, u = j & 7;
            const int p = b * kPtBlk + r;
            const uint32_t dk = smem_u32(kt + r * 128 + ((u ^ (r & 7)) << 4));
            const uint32_t dv = smem_u32(vt + r * 128 + ((u ^ (r & 7)) << 4));
            if (p < end) {
                const int page = a.page_table[(size_t)slot * a.pages_per_stream + p / kPage];
                const size_t off = (size_t)page * kPageHalfs + (size_t)(p % kPage) * kHeadDim + u * 8;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk), "l"(kbase + off) : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv), "l"(vbase + off) : "memory");
            } else {
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dk), "r"(0) : "memory");
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dv), "r"(0) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (nblk > 0) copy_block(0);
    for (int b = 0; b < nblk && ok; ++b) {
        // buffer (b + 1) & 1 was read by block b - 1's MMAs, which have completed
        if (b + 1 < nblk) {
            copy_block(b + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        uint8_t *kt = kv_buf + (b & 1) * 2 * kPtKvTile, *vt = kt + kPtKvTile;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        // ---- S = (Q_hi + Q_lo) K^T
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t qh = smem_u32(q_hi), ql = smem_u32(q_lo), kb = smem_u32(kt);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                tc_mma(t_s, sw128_desc(qh + k * 32), sw128_desc(kb + k * 32), idesc_s, k > 0 ? 1u : 0u);
                tc_mma(t_s, sw128_desc(ql + k * 32), sw128_desc(kb + k * 32), idesc_s, 1u);
            }
            tc_commit(&mma_bar);
        }
        ok = mbar_wait(&mma_bar, 0, a.err, 17);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float s[64];
        pt_ld_row64(tmem, warp, 0, s);
        // ---- online softmax over the block (positions >= my_lim masked)
        const int pb = b * kPtBlk;
        float mx = m;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            if (pb + c >= my_lim) s[c] = -INFINITY;
            mx = fmaxf(mx, s[c]);
        }
        const float corr = mx == -INFINITY ? 1.f : __expf(m - mx);
        float sum = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            __align__(16) __half h[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float pw = mx == -INFINITY ? 0.f : __expf(s[8 * u + e] - mx);  // 0 for masked keys
                sum += pw;
                h[e] = __float2half_rn(pw);
                lo[e] = __float2half_rn(pw - __half2float(h[e]));
            }
            pt_store_row_unit(p_hi, tid, u, h);
            pt_store_row_unit(p_lo, tid, u, lo);
        }
        l = l * corr + sum;
        m = mx;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        // ---- O_blk = (P_hi + P_lo) V
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ph = smem_u32(p_hi), pl = smem_u32(p_lo), vb = smem_u32(vt);
#pragma unroll
            for (int k = 0; k < 4; ++k) {  // 16 keys per step: P columns 16k.., V rows 16k..
                tc_mma(t_o, sw128_desc(ph + k * 32), sw128_desc(vb + k * 2048), idesc_pv, k > 0 ? 1u : 0u);
                tc_mma(t_o, sw128_desc(pl + k * 32), sw128_desc(vb + k * 2048), idesc_pv, 1u);
            }
            tc_commit(&mma_bar);
        }
        ok = mbar_wait(&mma_bar, 1, a.err, 18) && ok;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        pt_ld_row64(tmem, warp, 64, s);  // this block's P V row (s is free now)
#pragma unroll
        for (int j = 0; j < 64; ++j) o[j] = fmaf(o[j], corr, s[j]);
        ok = __syncthreads_and(ok);  // K, V and P are free for the next block; a time-out stops all
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // no copy in flight past this point
    // ---- o / l -> the proj GEMM's activation image (row, dims 64 hd ..)
    if (tid < nrows && ok) {
        const float inv = 1.f / l;
        const int r = row0 + tid;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            __align__(16) __half h[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float y = o[8 * u + e] * inv;
                h[e] = __float2half_rn(y);
                lo[e] = __float2half_rn(y - __half2float(h[e]));
            }
            const size_t off = bimg_off(r, hd * kHeadDim + 8 * u, a.bimg_N);
            *reinterpret_cast<int4 *>(a.bimg + off) = *reinterpret_cast<const int4 *>(h);
            if (a.bimg_parts == 2)
                *reinterpret_cast<int4 *>(a.bimg + (size_t)kHidden * a.bimg_N * 2 + off) = *reinterpret_cast<const int4 *>(lo);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128));
    }
}

}  // namespace
}  // namespace mossgpu
