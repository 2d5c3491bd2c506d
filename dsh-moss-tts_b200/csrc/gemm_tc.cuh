// gemm_tc.cuh -- tcgen05 (5th-generation tensor core) W8A16 GEMM for batched rows, sm_100a.
//
//   Y[n][m] = sum_k X[n][k] * W[m][k],   W = int8 Q8_0 blocks x fp16 scales, X fp16
//
// "Swap AB" so the weight rows form the MMA M dimension (128 per tile) and the batch rows the
// N dimension: D[128][N] fp32 lives in tensor memory (TMEM).  Per K chunk (64) of a CTA:
//   - one producer thread bulk-copies (cp.async.bulk, no tensor map, no multicast) the
//     weight tile's int8 quants (8 KB), its fp16 scales (512 B) and the activation tile
//     (N x 128 B, already stored in the SWIZZLE_128B K-major image by the previous kernel);
//   - eight dequant warps (each thread half of a weight row) convert int8 x scale -> fp16
//     into the A tile (SWIZZLE_128B K-major image, 16 KB), fence the async proxy and arrive;
//   - one MMA thread issues four tcgen05.mma.kind::f16 (K = 16 each) per operand part and
//     commits to the stage's "empty" barrier.
// Two forms:
//   split-K (decode batches, <= 64 batch rows per CTA): the K chunks of a weight tile are
//     split over a thread-block cluster of C CTAs.  After the last chunk the eight warps read
//     the partial D back with tcgen05.ld and scatter it through distributed shared memory:
//     CTA j of the cluster receives every CTA's partial of tile rows [128 j / C, 128 (j+1) / C),
//     sums the C partials in a fixed order and runs the epilogue for those rows;
//   direct (prefill passes, <= 256 batch rows per CTA; k_gemm_tp below): one CTA runs every
//     K chunk of its (weight tile, batch slice) tiles and epilogue warps read the
//     accumulators straight from TMEM, double-buffered so that epilogue and MMAs overlap.
// Epilogues: bias / RoPE / KV append, GELU into the next GEMM's activation image, residual
// add, or a plain store.  No atomics; the result does not depend on timing.
// Every mbarrier wait is bounded: on time-out the kernel records an error code and leaves
// through the normal exit path (TMEM is always freed, every CTA reaches the cluster barriers).
//
// Weight layout (repacked from the file at load, a byte permutation):
//   qt [rows/128][K/64][128][64] int8, the four 16-byte pieces of each 64-byte row stored at
//      piece ^ ((row >> 1) & 3) so that the dequant warps read shared memory without bank
//      conflicts;
//   st [rows/128][K/64][128][2] fp16 (the scales of blocks 2c and 2c+1 of each row).
// Activation image ("B image") for N padded rows and K columns:
//   [K/64][N][128 B], element (n, k) at byte ((k/64)*N + n)*128 + (((k%64)/8) ^ (n%8))*16 + (k%8)*2
//   -- exactly what a SWIZZLE_128B K-major operand looks like in shared memory.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "types.h"

namespace mossgpu {
namespace {

constexpr int kTcM = 128;      // weight rows per CTA (MMA M)
constexpr int kTcK = 64;       // K per pipeline stage (one 128-byte swizzle row of fp16)
constexpr int kTcEpiThreads = 256;  // dequant / epilogue threads (8 warps, two per TMEM lane quarter)
constexpr int kTcThreads = 64 + kTcEpiThreads;
constexpr int kTcMaxNS = 64;   // batch rows per CTA (MMA N) with split-K; more rows split over gridDim.z
constexpr int kTcMaxND = 256;  // batch rows per CTA in the direct (no split-K) form
constexpr int kTcMaxCluster = 16;  // 16 is a non-portable cluster size (opted in per kernel)

enum { TC_STORE = 0, TC_QKV = 1, TC_RESID = 2, TC_GELU_B = 3 };

struct TcArgs {
    const int8_t *qt;       // weight quants, tile layout
    const __half *st;       // weight scales, tile layout
    int rows, K;            // weight matrix shape
    const uint8_t *bimg;    // activation image [K/64][N][128 B]
    int N;                  // padded batch rows (multiple of 16, <= 256): rows of the activation image
    int nsub;               // batch rows per CTA along gridDim.z (divides N, multiple of 16, <= 64)
    int R;                  // real batch rows (<= N)
    int csize;              // CTAs per cluster (split-K over the tile's K chunks): 1, 2, 4 or 8
    int stages;             // pipeline stages (<= 4)
    const float *bias;
    float *out;             // TC_STORE: [R][ldo]; TC_RESID: residual [R][ldo] (read, added, written)
    int ldo;
    // TC_QKV
    float *q_out;
    __half *kv;
    const int *page_table;
    int pages_per_stream;
    float *lkv;
    const int *row_slot;
    const int *row_pos;
    int fixed_pos;
    const float2 *rope;
    // TC_GELU_B: output activation image for the next GEMM (K_next = rows)
    uint8_t *bimg_out;
    int *err;               // error flag (0 = fine)
    // tile-persistent TC_STORE only: K split in ksplit equal parts (1 = none); part p stores its
    // partial sums at out + p * part_stride (bias in part 0), for a consumer that adds them
    int ksplit;
    size_t part_stride;
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    // K-major SWIZZLE_128B canonical layout: 8-row atoms of 1024 B, SBO = 1024 B, LBO unused (1),
    // descriptor version 1 (sm100), base offset 0 (atoms are 1024-byte aligned)
    return (uint64_t((saddr >> 4) & 0x3FFF)) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

// A operand from tensor memory (lane = row, two fp16 K elements per 32-bit column)
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float *v) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Precision modes.  TC_F16: one MMA per K step on fp16 operands (fp16 rounding of the
// dequantised weight and of the activation, ~5e-4 relative).  TC_F16X3: each operand is split
// into a high fp16 part and the fp16 of its remainder (w = w_hi + w_lo, x = x_hi + x_lo) and
// three MMAs accumulate w_hi.x_hi + w_hi.x_lo + w_lo.x_hi in fp32 -- close to the fp32
// arithmetic of the reference's W8A16 dot product, at three times the (small) MMA work.
enum { TC_F16 = 1, TC_F16X3 = 3 };

__host__ __device__ constexpr int tc_parts(int prec) { return prec == TC_F16X3 ? 2 : 1; }

__host__ __device__ constexpr int tc_stage_bytes(int N, int prec) {
    // [A tiles 16 KB each][B tiles N*128 each][W8 8 KB][scales 512 B], padded to 1 KB so that
    // every A and B tile starts on a 1 KB boundary
    return (16384 * tc_parts(prec) + N * 128 * tc_parts(prec) + 8192 + 512 + 1023) / 1024 * 1024;
}

// receive buffer of the split-K reduction: C partial slices of NS columns x (128 / C) rows
__host__ __device__ constexpr int tc_recv_bytes(int NS) { return kTcM * NS * 4; }

__host__ __device__ constexpr int tc_smem_bytes(int NS, int prec, int stages) {
    return stages * tc_stage_bytes(NS, prec) + tc_recv_bytes(NS) + 1024;
}

// most stages that fit in 227 KB of shared memory (at most 4)
__host__ __device__ constexpr int tc_max_stages(int NS, int prec) {
    return ((227 * 1024 - 1024 - tc_recv_bytes(NS)) / tc_stage_bytes(NS, prec)) < 4
               ? ((227 * 1024 - 1024 - tc_recv_bytes(NS)) / tc_stage_bytes(NS, prec))
               : 4;
}

// stage of the A-in-TMEM form: [B parts][W8 8 KB][scales 512 B] (the A tile lives in TMEM)
__host__ __device__ constexpr int tc_stage_bytes_atm(int N, int prec) {
    return (N * 128 * tc_parts(prec) + 8192 + 512 + 1023) / 1024 * 1024;
}
__host__ __device__ constexpr int tc_smem_bytes_atm(int NS, int prec, int stages) {
    return stages * tc_stage_bytes_atm(NS, prec) + 1024;
}
// stages of the A-in-TMEM form: shared memory, and 64 TMEM columns each beside 2 x NS
// accumulator columns in 512
__host__ __device__ constexpr int tc_max_stages_atm(int NS, int prec) {
    return ((224 * 1024 - 1024) / tc_stage_bytes_atm(NS, prec)) < ((512 - 2 * NS) / 64)
               ? (((224 * 1024 - 1024) / tc_stage_bytes_atm(NS, prec)) < 4 ? ((224 * 1024 - 1024) / tc_stage_bytes_atm(NS, prec)) : 4)
               : (((512 - 2 * NS) / 64) < 4 ? ((512 - 2 * NS) / 64) : 4);
}

// direct form (one CTA per tile, accumulators read straight from TMEM): no receive buffer;
// 3 KB are left for the static shared memory (barriers, per-row positions)
__host__ __device__ constexpr int tc_smem_bytes_direct(int NS, int prec, int stages) {
    return stages * tc_stage_bytes(NS, prec) + 1024;
}
__host__ __device__ constexpr int tc_max_stages_direct(int NS, int prec) {
    return ((224 * 1024 - 1024) / tc_stage_bytes(NS, prec)) < 4 ? ((224 * 1024 - 1024) / tc_stage_bytes(NS, prec)) : 4;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// shared-memory address `saddr` of this CTA -> the same offset in cluster CTA `rank`
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// int8 pairs -> fp16 pairs, exact: bytes b are placed as the low mantissa byte of 1024.0
// (0x64bb) after flipping the sign bit, so the half is 1024 + (b + 128); subtracting 1152
// leaves b.  `sel` picks bytes 0,1 (0x5140) or 2,3 (0x7362) of the word.
__device__ __forceinline__ __half2 i8x2_to_h2(uint32_t w_flipped, uint32_t sel) {
    const uint32_t h = __byte_perm(w_flipped, 0x64646464u, sel);
    return __hsub2(*reinterpret_cast<const __half2 *>(&h), __half2half2(__ushort_as_half((unsigned short)0x6480)));
}

// Dequantise 16-byte piece j (k = 16 j .. 16 j + 15) of weight row t of a stage: int8 x fp16
// scale -> hi = fp16(q d) and (NP = 2) lo = fp16(q d - hi), one rounding each, as fp16 of the
// exact fp32 product and of its remainder.  k = 16 j + e goes to 16-byte unit 2 j (+1) of the
// row's 128-byte line in the A tile, stored at unit ^ (t % 8) (SWIZZLE_128B).
template <int NP>
__device__ __forceinline__ void tc_dequant_piece(const int8_t *w8, const __half *sc, uint8_t *arow, int t, int j) {
    const int4 q = *reinterpret_cast<const int4 *>(w8 + ((j ^ ((t >> 1) & 3)) << 4));
    const __half2 d2 = __half2half2(sc[j >> 1]);
    const uint32_t words[4] = {(uint32_t)q.x ^ 0x80808080u, (uint32_t)q.y ^ 0x80808080u, (uint32_t)q.z ^ 0x80808080u,
                               (uint32_t)q.w ^ 0x80808080u};
    __align__(16) __half2 h[8];
    __align__(16) __half2 l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const __half2 qq = i8x2_to_h2(words[e >> 1], (e & 1) ? 0x7362u : 0x5140u);
        h[e] = __hmul2_rn(qq, d2);
        if (NP == 2) l[e] = __hfma2(qq, d2, __hneg2(h[e]));
    }
    *reinterpret_cast<int4 *>(arow + (((2 * j) ^ (t & 7)) << 4)) = *reinterpret_cast<const int4 *>(h);
    *reinterpret_cast<int4 *>(arow + (((2 * j + 1) ^ (t & 7)) << 4)) = *reinterpret_cast<const int4 *>(h + 4);
    if (NP == 2) {
        *reinterpret_cast<int4 *>(arow + 16384 + (((2 * j) ^ (t & 7)) << 4)) = *reinterpret_cast<const int4 *>(l);
        *reinterpret_cast<int4 *>(arow + 16384 + (((2 * j + 1) ^ (t & 7)) << 4)) = *reinterpret_cast<const int4 *>(l + 4);
    }
}

// The same conversion into registers: 8 packed fp16 pairs (k = 16 j + 2 e, + 1) of hi and lo,
// for tcgen05.st into an A tile in tensor memory (column 8 j + e of the row).
template <int NP>
__device__ __forceinline__ void tc_dequant_piece_regs(const int8_t *w8, const __half *sc, int t, int j, uint32_t *hi,
                                                      uint32_t *lo) {
    const int4 q = *reinterpret_cast<const int4 *>(w8 + ((j ^ ((t >> 1) & 3)) << 4));
    const __half2 d2 = __half2half2(sc[j >> 1]);
    const uint32_t words[4] = {(uint32_t)q.x ^ 0x80808080u, (uint32_t)q.y ^ 0x80808080u, (uint32_t)q.z ^ 0x80808080u,
                               (uint32_t)q.w ^ 0x80808080u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const __half2 qq = i8x2_to_h2(words[e >> 1], (e & 1) ? 0x7362u : 0x5140u);
        const __half2 h = __hmul2_rn(qq, d2);
        hi[e] = *reinterpret_cast<const uint32_t *>(&h);
        if (NP == 2) {
            const __half2 l = __hfma2(qq, d2, __hneg2(h));
            lo[e] = *reinterpret_cast<const uint32_t *>(&l);
        }
    }
}

// 32 consecutive 32-bit columns of this thread's TMEM lane
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// One element of the direct form's epilogue: weight row gm (this thread's TMEM lane), batch row
// rr, accumulator v, bias b, `pre` = what tc_epi_pre fetched for it.  Uniform over the warp
// for a given rr (the QKV pair exchange is a shuffle between lanes gm and gm ^ 1).
// The global inputs of a group of elements (residual rows, RoPE table entries) are fetched
// for the whole group first: interleaved with the group's stores, each load would wait a
// full L2 round trip behind the previous element's store.
template <int EPI>
__device__ __forceinline__ float2 tc_epi_pre(const TcArgs &a, int gm, int rr, int pos) {
    if (EPI == TC_RESID) return make_float2(rr < a.R ? a.out[(size_t)rr * a.ldo + gm] : 0.f, 0.f);
    if (EPI == TC_QKV && gm < 2 * kHidden && rr < a.R) return a.rope[(size_t)pos * (kHeadDim / 2) + ((gm % kHeadDim) >> 1)];
    return make_float2(0.f, 0.f);
}

template <int EPI, int NP>
__device__ __forceinline__ void tc_epi_one(const TcArgs &a, float *out, int gm, int rr, int N, float v, float b, int pos,
                                           int dst, float2 pre) {
    if (EPI == TC_STORE) {
        if (rr < a.R) out[(size_t)rr * a.ldo + gm] = b != 0.f ? __fadd_rn(v, b) : v;
    } else if (EPI == TC_RESID) {
        if (rr < a.R) out[(size_t)rr * a.ldo + gm] = __fadd_rn(pre.x, __fadd_rn(v, b));
    } else if (EPI == TC_GELU_B) {
        const float g = rr < a.R ? gelu_new(__fadd_rn(v, b)) : 0.f;
        const __half h = __float2half_rn(g);
        const size_t off = bimg_off(rr, gm, N);
        *reinterpret_cast<__half *>(a.bimg_out + off) = h;
        if (NP == 2) *reinterpret_cast<__half *>(a.bimg_out + (size_t)a.rows * N * 2 + off) = __float2half_rn(g - __half2float(h));
    } else if (rr < a.R) {  // TC_QKV
        const float y = __fadd_rn(v, b);
        const float yp = __shfl_xor_sync(0xffffffffu, y, 1);  // the other row of the RoPE pair
        float o = y;
        if (gm < 2 * kHidden) {
            const float2 cs = pre;
            o = (gm & 1) ? __fadd_rn(__fmul_rn(y, cs.x), __fmul_rn(yp, cs.y))
                         : __fsub_rn(__fmul_rn(y, cs.x), __fmul_rn(yp, cs.y));
        }
        if (gm < kHidden) {
            a.q_out[(size_t)rr * kHidden + gm] = o;
        } else {
            const int kvsel = gm < 2 * kHidden ? 0 : 1;
            const int c = gm - kHidden * (1 + kvsel);
            if (a.kv)
                a.kv[(size_t)dst * kPageHalfs + ((kvsel * kHeads + c / kHeadDim) * kPage + pos % kPage) * kHeadDim +
                     (c % kHeadDim)] = __float2half_rn(o);
            else
                a.lkv[(((size_t)dst * 2 + kvsel) * kLocalLen + pos) * kHidden + c] = o;
        }
    }
}

// Split-K epilogue items are (pair of tile rows, batch row); thread u takes items u,
// u + 256, ...  Global inputs of kTcPreB items starting at `base`: the residual pair (RESID) or
// the RoPE entry (QKV).
constexpr int kTcPreB = 4;
template <int EPI>
__device__ __forceinline__ void tc_splitk_pre(const TcArgs &a, int base, int tile, int rank, int RS, int NS, int r0,
                                              const int *s_pos, float2 *pre) {
    const int HP = RS / 2, total = HP * NS;
#pragma unroll
    for (int bi = 0; bi < kTcPreB; ++bi) {
        const int idx = base + bi * kTcEpiThreads;
        pre[bi] = make_float2(0.f, 0.f);
        if (idx < total) {
            const int pr = idx % HP, n = idx / HP;
            const int gm = tile * kTcM + rank * RS + 2 * pr;
            const int rr = r0 + n;
            if (EPI == TC_RESID && rr < a.R) pre[bi] = *reinterpret_cast<const float2 *>(a.out + (size_t)rr * a.ldo + gm);
            if (EPI == TC_QKV && rr < a.R && gm < 2 * kHidden)
                pre[bi] = a.rope[(size_t)s_pos[n] * (kHeadDim / 2) + ((gm % kHeadDim) >> 1)];
        }
    }
}

// Split-K form (decode batches): a cluster of a.csize CTAs shares a weight tile's K chunks,
// partials reduce-scattered through DSMEM, <= 64 batch rows per CTA.
template <int EPI, int PREC>
__global__ void __launch_bounds__(kTcThreads, 1) k_gemm_tc(const TcArgs a) {
    extern __shared__ uint8_t tc_smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[4], bfull_bar[4], dq_bar[4], empty_bar[4], acc_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_pos[kTcMaxNS], s_dst[kTcMaxNS];  // TC_QKV: per batch row position and page/slot
    constexpr int NP = tc_parts(PREC);  // operand parts (hi, lo)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = a.N;                  // rows of the activation image
    const int NS = a.nsub;              // rows handled by this CTA (MMA N)
    const int C = a.csize;              // CTAs of the cluster (split-K)
    const int S = a.stages;
    const int rank = (int)cluster_rank();
    const int tile = blockIdx.x / C;
    const int r0 = blockIdx.z * NS;     // first batch row of this CTA
    const int SB = tc_stage_bytes(NS, PREC);
    // stage layout: [A part 0..NP-1: 16 KB each][B part 0..NP-1: NS*128 each][W8 8 KB][scales]
    const int OFF_B = 16384 * NP;
    const int OFF_W8 = OFF_B + NS * 128 * NP;
    const int OFF_SC = OFF_W8 + 8192;
    const size_t bimg_part = (size_t)a.K * N * 2;  // bytes of one activation image part
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    float *recv = reinterpret_cast<float *>(smem + (size_t)S * SB);  // [C][NS][RS] partial slices
    float2 pre0[kTcPreB];  // split-K epilogue: first batch of global inputs, fetched early
    const int RS = kTcM / C;                                         // tile rows reduced here
    const int nchunks_total = a.K / kTcK;
    const int c0 = rank * nchunks_total / C;
    const int c1 = (rank + 1) * nchunks_total / C;
    const int nch = c1 - c0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_bar[s], 1);   // weight quants + scales of the stage landed
            mbar_init(&bfull_bar[s], 1);  // activation tile(s) of the stage landed
            mbar_init(&dq_bar[s], kTcEpiThreads);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    uint32_t ncols = 32;
    while (ncols < (uint32_t)NS) ncols <<= 1;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    cluster_arrive_relaxed();  // this CTA runs; matched by the wait before the first remote store
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_sh;

    const size_t wtile = (size_t)tile * nchunks_total;  // (tile, chunk) index base
    if (warp == 0) {
        // ---------------- producer
        if (lane == 0 && nch > 0) {
            auto load_w = [&](int i) {
                const int s = i % S;
                uint8_t *st = smem + (size_t)s * SB;
                const int c = c0 + i;
                mbar_expect_tx(&full_bar[s], 8192 + 512);
                bulk_g2s(st + OFF_W8, a.qt + (wtile + c) * 8192, 8192, &full_bar[s]);
                bulk_g2s(st + OFF_SC, a.st + (wtile + c) * 256, 512, &full_bar[s]);
            };
            auto load_b = [&](int i) {
                const int s = i % S;
                uint8_t *st = smem + (size_t)s * SB;
                const int c = c0 + i;
                mbar_expect_tx(&bfull_bar[s], (uint32_t)(NS * 128 * NP));
#pragma unroll
                for (int p = 0; p < NP; ++p)
                    bulk_g2s(st + OFF_B + p * NS * 128, a.bimg + p * bimg_part + ((size_t)c * N + r0) * 128,
                             (uint32_t)NS * 128, &bfull_bar[s]);
            };
            // weights are static: the first stages are fetched (and dequantised) while the
            // kernel that produces the activations may still be running
            const int pre = min(S, nch);
            for (int i = 0; i < pre; ++i) load_w(i);
            pdl_wait();
            pdl_trigger();
            for (int i = 0; i < pre; ++i) load_b(i);
            int issued = pre;
            for (int i = pre; i < nch; ++i) {
                const int s = i % S;
                if (!mbar_wait(&empty_bar[s], ((i / S) - 1) & 1, a.err, 1)) break;
                load_w(i);
                load_b(i);
                ++issued;
            }
            // leave only after every copy this CTA issued has landed
            for (int i = max(0, issued - S); i < issued; ++i) {
                mbar_wait(&full_bar[i % S], (i / S) & 1, a.err, 2);
                mbar_wait(&bfull_bar[i % S], (i / S) & 1, a.err, 2);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0 && nch > 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(NS >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
            for (int i = 0; i < nch; ++i) {
                const int s = i % S;
                if (!mbar_wait(&dq_bar[s], (i / S) & 1, a.err, 3)) break;
                if (!mbar_wait(&bfull_bar[s], (i / S) & 1, a.err, 6)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                uint8_t *st = smem + (size_t)s * SB;
                const uint32_t abase = smem_u32(st), bbase = smem_u32(st + OFF_B);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    tc_mma(tmem, sw128_desc(abase + k * 32), sw128_desc(bbase + k * 32), idesc, (i > 0 || k > 0) ? 1u : 0u);
                    if (NP == 2) {  // + w_hi.x_lo + w_lo.x_hi
                        tc_mma(tmem, sw128_desc(abase + k * 32), sw128_desc(bbase + NS * 128 + k * 32), idesc, 1u);
                        tc_mma(tmem, sw128_desc(abase + 16384 + k * 32), sw128_desc(bbase + k * 32), idesc, 1u);
                    }
                }
                tc_commit(&empty_bar[s]);
            }
            // acc_bar completes when every MMA issued above has finished (also on the error path)
            tc_commit(&acc_bar);
        }
    } else {
        // ---------------- dequant (then epilogue): warps 2..9, 256 threads; thread u converts
        // half hf of weight row t (16-byte pieces 2 hf and 2 hf + 1, k 32 hf .. 32 hf + 31)
        const int u = threadIdx.x - 64;
        const int t = u & (kTcM - 1), hf = u >> 7;
        bool ok = true;
        for (int i = 0; i < nch && ok; ++i) {
            const int s = i % S;
            if (!mbar_wait(&full_bar[s], (i / S) & 1, a.err, 4)) {
                ok = false;
                break;
            }
            uint8_t *st = smem + (size_t)s * SB;
            const int8_t *w8 = reinterpret_cast<const int8_t *>(st + OFF_W8) + t * 64;
            const __half *sc = reinterpret_cast<const __half *>(st + OFF_SC) + t * 2;
            uint8_t *arow = st + t * 128;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) tc_dequant_piece<NP>(w8, sc, arow, t, 2 * hf + jj);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&dq_bar[s]);
        }
        // ---------------- partial results -> the CTA of the cluster that reduces each row
        pdl_wait();  // from here on this warp touches data of earlier kernels (outputs, row metadata)
        if (EPI == TC_QKV) {
            // per-row position and KV page (or local slot), fetched once per CTA
            for (int j = u; j < NS; j += kTcEpiThreads) {
                const int rr = r0 + j;
                int pos = 0, dst = 0;
                if (rr < a.R) {
                    pos = a.row_pos ? a.row_pos[rr] : a.fixed_pos;
                    const int slot = a.row_slot[rr];
                    dst = a.kv ? a.page_table[(size_t)slot * a.pages_per_stream + pos / kPage] : slot;
                }
                s_pos[j] = pos;
                s_dst[j] = dst;
            }
        }
        // the epilogue's first batch of global inputs (residual rows, RoPE entries: outputs of
        // earlier kernels) is fetched now, while the MMAs run
        asm volatile("barrier.sync 1, %0;" ::"n"(kTcEpiThreads) : "memory");  // s_pos visible
        tc_splitk_pre<EPI>(a, u, tile, rank, RS, NS, r0, s_pos, pre0);
        const int q = warp & 3;                 // TMEM lane quarter this warp may read
        const int m = q * 32 + lane;            // weight row within the tile
        // the two warps of a lane quarter split the columns: [0, split) and [split, NS)
        const int split = ((NS / 16 + 1) / 2) * 16;
        const int cb = hf ? split : 0, ce = hf ? NS : split;
        const bool acc_ok = nch > 0 && mbar_wait(&acc_bar, 0, a.err, 5);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        {
            cluster_wait();  // every CTA of the cluster is running: its shared memory may be written
            const uint32_t dst_rank = (uint32_t)(m / RS);
            const uint32_t rbase =
                cluster_map(smem_u32(recv), dst_rank) + (uint32_t)(((rank * NS) * RS + (m % RS)) * 4);
            for (int n0 = cb; n0 < ce; n0 += 16) {
                float v[16];
                if (acc_ok && ok) {
                    tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)n0, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0.f;
                }
                // a warp's stores for one column land as two 64-byte runs (lanes = consecutive
                // rows); 16-byte stores along the columns measured slower
#pragma unroll
                for (int j = 0; j < 16; ++j) st_cluster_f32(rbase + (uint32_t)((n0 + j) * RS * 4), v[j]);
            }
        }
    }
    // every thread of every CTA: the partial slices are delivered (release / acquire)
    __syncwarp();
    if (warp < 2) cluster_wait();  // matches the arrive at the start (warps 2..5 waited above)
    cluster_arrive();
    cluster_wait();

    if (warp >= 2) {
        // ---------------- reduce this CTA's rows and run the epilogue, two rows per item, in
        // batches of 4 items per thread whose global inputs are fetched before any store
        const int u = threadIdx.x - 64;
        const int HP = RS / 2;
        const int total = HP * NS;
        for (int base = u; base < total; base += kTcPreB * kTcEpiThreads) {
            float2 pre[kTcPreB];
            if (base == u) {
#pragma unroll
                for (int bi = 0; bi < kTcPreB; ++bi) pre[bi] = pre0[bi];
            } else {
                tc_splitk_pre<EPI>(a, base, tile, rank, RS, NS, r0, s_pos, pre);
            }
#pragma unroll
            for (int bi = 0; bi < kTcPreB; ++bi) {
                const int idx = base + bi * kTcEpiThreads;
                if (idx >= total) break;
                const int pr = idx % HP, n = idx / HP;
                float v0 = 0.f, v1 = 0.f;
                for (int src = 0; src < C; ++src) {
                    const float2 pv = reinterpret_cast<const float2 *>(recv)[((size_t)src * NS + n) * HP + pr];
                    v0 += pv.x;
                    v1 += pv.y;
                }
                const int gm = tile * kTcM + rank * RS + 2 * pr;  // even global weight row
                const int rr = r0 + n;
                const float b0 = a.bias ? a.bias[gm] : 0.f, b1 = a.bias ? a.bias[gm + 1] : 0.f;
                if (EPI == TC_STORE) {
                    if (rr < a.R)
                        *reinterpret_cast<float2 *>(a.out + (size_t)rr * a.ldo + gm) =
                            a.bias ? make_float2(__fadd_rn(v0, b0), __fadd_rn(v1, b1)) : make_float2(v0, v1);
                } else if (EPI == TC_RESID) {
                    if (rr < a.R) {
                        const float2 x = pre[bi];
                        *reinterpret_cast<float2 *>(a.out + (size_t)rr * a.ldo + gm) =
                            make_float2(__fadd_rn(x.x, __fadd_rn(v0, b0)), __fadd_rn(x.y, __fadd_rn(v1, b1)));
                    }
                } else if (EPI == TC_GELU_B) {
                    const float g0 = rr < a.R ? gelu_new(__fadd_rn(v0, b0)) : 0.f;
                    const float g1 = rr < a.R ? gelu_new(__fadd_rn(v1, b1)) : 0.f;
                    const __half2 gh = __floats2half2_rn(g0, g1);
                    const size_t off = bimg_off(rr, gm, N);  // gm even: both halves in one 16-byte unit
                    *reinterpret_cast<__half2 *>(a.bimg_out + off) = gh;
                    if (NP == 2)  // the next GEMM's K is this one's rows
                        *reinterpret_cast<__half2 *>(a.bimg_out + (size_t)a.rows * N * 2 + off) =
                            __floats2half2_rn(g0 - __low2float(gh), g1 - __high2float(gh));
                } else if (rr < a.R) {  // TC_QKV: bias, RoPE on the (gm, gm + 1) pair, q out / KV append
                    const int pos = s_pos[n];
                    const float yb = __fadd_rn(v0, b0), other = __fadd_rn(v1, b1);
                    float o0 = yb, o1 = other;
                    if (gm < 2 * kHidden) {
                        const float2 cs = pre[bi];
                        o0 = __fsub_rn(__fmul_rn(yb, cs.x), __fmul_rn(other, cs.y));
                        o1 = __fadd_rn(__fmul_rn(other, cs.x), __fmul_rn(yb, cs.y));
                    }
                    if (gm < kHidden) {
                        *reinterpret_cast<float2 *>(a.q_out + (size_t)rr * kHidden + gm) = make_float2(o0, o1);
                    } else {
                        const int kvsel = gm < 2 * kHidden ? 0 : 1;
                        const int c = gm - kHidden * (1 + kvsel);
                        if (a.kv) {
                            __half *dst = a.kv + (size_t)s_dst[n] * kPageHalfs +
                                          ((kvsel * kHeads + c / kHeadDim) * kPage + pos % kPage) * kHeadDim +
                                          (c % kHeadDim);
                            *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(o0, o1);
                        } else {
                            float *dst = a.lkv + (((size_t)s_dst[n] * 2 + kvsel) * kLocalLen + pos) * kHidden + c;
                            *reinterpret_cast<float2 *>(dst) = make_float2(o0, o1);
                        }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
}

// Tile-persistent form of the direct GEMM (prefill passes): a grid of <= 148 CTAs walks the
// (weight tile, batch slice) tiles round-robin.  The producer, dequant and MMA roles stream
// every K chunk of every tile of the CTA through one stage ring, and the accumulators are
// double-buffered in TMEM (2 x NS columns), so the epilogue warps drain tile j while the MMAs
// of tile j + 1 run.  Roles: warp 0 producer, warp 1 MMA issuer, warps 2..5 dequant (a weight
// row per thread), warps 6..13 epilogue (two per TMEM lane quarter, splitting the columns).
// acc_full[b]: the MMAs of the tile in buffer b are done; acc_empty[b]: its epilogue has read
// it.  Every wait is bounded.
constexpr int kTpDqThreads = 128;
constexpr int kTpEpiThreads = 256;
constexpr int kTpThreads = 64 + kTpDqThreads + kTpEpiThreads;

// ATM = true: the dequantised A tiles go to tensor memory (tcgen05.st, 64 columns per stage
// beside the two accumulators) and the MMAs read A from there, which takes 48 KB of operand
// reads and 32 KB of stores per K chunk off shared memory (the main loop's bound).
template <int EPI, int PREC, bool ATM>
__global__ void __launch_bounds__(kTpThreads, 1) k_gemm_tp(const TcArgs a) {
    extern __shared__ uint8_t tc_smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[4], bfull_bar[4], dq_bar[4], empty_bar[4], accf_bar[2], acce_bar[2];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_pos[kTcMaxND], s_dst[kTcMaxND];
    constexpr int NP = tc_parts(PREC);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = a.N, NS = a.nsub, S = a.stages;
    const int SB = ATM ? tc_stage_bytes_atm(NS, PREC) : tc_stage_bytes(NS, PREC);
    const int OFF_B = ATM ? 0 : 16384 * NP;
    const int OFF_W8 = OFF_B + NS * 128 * NP;
    const int OFF_SC = OFF_W8 + 8192;
    const size_t bimg_part = (size_t)a.K * N * 2;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int nchunks = a.K / kTcK;
    const int n_m = a.rows / kTcM;
    const int acol0 = 2 * NS;  // ATM: A stage s at TMEM columns acol0 + 64 s (hi) and + 32 (lo)
    const int n_tiles = n_m * (N / NS);
    // work units = (K part, tile): part kp of unit u = u / n_tiles covers K chunks
    // [kp nchu, (kp + 1) nchu) of tile u % n_tiles
    const int KS = (EPI == TC_STORE && a.ksplit > 1) ? a.ksplit : 1;
    const int nchu = nchunks / KS;
    const int n_units = n_tiles * KS;
    const int G = gridDim.x;
    const int my_tiles = (int)blockIdx.x < n_units ? (n_units - 1 - (int)blockIdx.x) / G + 1 : 0;
    const int total = my_tiles * nchu;  // K chunks this CTA streams

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&bfull_bar[s], 1);
            mbar_init(&dq_bar[s], kTpDqThreads);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf_bar[b], 1);
            mbar_init(&acce_bar[b], kTpEpiThreads);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    uint32_t ncols = 32;
    while (ncols < (uint32_t)(2 * NS + (ATM ? 64 * S : 0))) ncols <<= 1;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_sh;

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0 && total > 0) {
            auto src = [&](int seq, int &mt, int &z, int &c) {
                const int u = (int)blockIdx.x + (seq / nchu) * G;
                const int t = u % n_tiles;
                c = (u / n_tiles) * nchu + seq % nchu;
                mt = t % n_m;
                z = t / n_m;
            };
            auto load_w = [&](int seq) {
                int mt, z, c;
                src(seq, mt, z, c);
                const int s = seq % S;
                uint8_t *st = smem + (size_t)s * SB;
                mbar_expect_tx(&full_bar[s], 8192 + 512);
                bulk_g2s(st + OFF_W8, a.qt + ((size_t)mt * nchunks + c) * 8192, 8192, &full_bar[s]);
                bulk_g2s(st + OFF_SC, a.st + ((size_t)mt * nchunks + c) * 256, 512, &full_bar[s]);
            };
            auto load_b = [&](int seq) {
                int mt, z, c;
                src(seq, mt, z, c);
                const int s = seq % S;
                uint8_t *st = smem + (size_t)s * SB;
                mbar_expect_tx(&bfull_bar[s], (uint32_t)(NS * 128 * NP));
#pragma unroll
                for (int p = 0; p < NP; ++p)
                    bulk_g2s(st + OFF_B + p * NS * 128, a.bimg + p * bimg_part + ((size_t)c * N + (size_t)z * NS) * 128,
                             (uint32_t)NS * 128, &bfull_bar[s]);
            };
            const int pre = min(S, total);
            for (int i = 0; i < pre; ++i) load_w(i);
            pdl_wait();
            pdl_trigger();
            for (int i = 0; i < pre; ++i) load_b(i);
            int issued = pre;
            for (int i = pre; i < total; ++i) {
                const int s = i % S;
                if (!mbar_wait(&empty_bar[s], ((i / S) - 1) & 1, a.err, 11)) break;
                load_w(i);
                load_b(i);
                ++issued;
            }
            for (int i = max(0, issued - S); i < issued; ++i) {
                mbar_wait(&full_bar[i % S], (i / S) & 1, a.err, 12);
                mbar_wait(&bfull_bar[i % S], (i / S) & 1, a.err, 12);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0 && total > 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(NS >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
            int seq = 0;
            bool ok = true;
            for (int j = 0; j < my_tiles && ok; ++j) {
                const int ab = j & 1;
                if (j >= 2 && !mbar_wait(&acce_bar[ab], ((j >> 1) - 1) & 1, a.err, 13)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dcol = tmem + (uint32_t)(ab * NS);
                for (int c = 0; c < nchu; ++c, ++seq) {
                    const int s = seq % S;
                    if (!mbar_wait(&dq_bar[s], (seq / S) & 1, a.err, 14) ||
                        !mbar_wait(&bfull_bar[s], (seq / S) & 1, a.err, 14)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    uint8_t *st = smem + (size_t)s * SB;
                    const uint32_t abase = smem_u32(st), bbase = smem_u32(st + OFF_B);
                    const uint32_t ahi = tmem + (uint32_t)(acol0 + 64 * s), alo = ahi + 32;  // ATM
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
                        if (ATM) {
                            tc_mma_ts(dcol, ahi + 8 * k, sw128_desc(bbase + k * 32), idesc, acc);
                            if (NP == 2) {
                                tc_mma_ts(dcol, ahi + 8 * k, sw128_desc(bbase + NS * 128 + k * 32), idesc, 1u);
                                tc_mma_ts(dcol, alo + 8 * k, sw128_desc(bbase + k * 32), idesc, 1u);
                            }
                        } else {
                            tc_mma(dcol, sw128_desc(abase + k * 32), sw128_desc(bbase + k * 32), idesc, acc);
                            if (NP == 2) {
                                tc_mma(dcol, sw128_desc(abase + k * 32), sw128_desc(bbase + NS * 128 + k * 32), idesc, 1u);
                                tc_mma(dcol, sw128_desc(abase + 16384 + k * 32), sw128_desc(bbase + k * 32), idesc, 1u);
                            }
                        }
                    }
                    tc_commit(&empty_bar[s]);
                }
                tc_commit(&accf_bar[ab]);  // also on the error path: the epilogue leaves on its own
            }
        }
    } else if (warp < 2 + kTpDqThreads / 32) {
        // ---------------- dequant: thread t converts weight row t of every chunk (ATM: the row
        // of this warp's TMEM lane quarter)
        const int t = ATM ? ((warp & 3) * 32 + lane) : (int)threadIdx.x - 64;
        for (int i = 0; i < total; ++i) {
            const int s = i % S;
            if (!mbar_wait(&full_bar[s], (i / S) & 1, a.err, 15)) break;
            uint8_t *st = smem + (size_t)s * SB;
            const int8_t *w8 = reinterpret_cast<const int8_t *>(st + OFF_W8) + t * 64;
            const __half *sc = reinterpret_cast<const __half *>(st + OFF_SC) + t * 2;
            if (ATM) {
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) tc_dequant_piece_regs<NP>(w8, sc, t, j, hi + 8 * j, lo + 8 * j);
                const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(acol0 + 64 * s);
                tc_st32(ta, hi);
                if (NP == 2) tc_st32(ta + 32, lo);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            } else {
                uint8_t *arow = st + t * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j) tc_dequant_piece<NP>(w8, sc, arow, t, j);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            mbar_arrive(&dq_bar[s]);
        }
    } else {
        // ---------------- epilogue: tile j's accumulators from TMEM buffer j & 1
        const int e = threadIdx.x - 64 - kTpDqThreads;  // 0..255
        const int q = warp & 3;                         // TMEM lane quarter of this warp
        const int hf = e >> 7;                          // column half
        const int mrow = q * 32 + lane;
        const int split = ((NS / 16 + 1) / 2) * 16;
        const int cb = hf ? split : 0, ce = hf ? NS : split;
        pdl_wait();
        for (int j = 0; j < my_tiles; ++j) {
            const int uu = (int)blockIdx.x + j * G;
            const int t = uu % n_tiles, kp = uu / n_tiles;
            const int mt = t % n_m, r0 = (t / n_m) * NS, ab = j & 1;
            float *outp = a.out ? a.out + (size_t)kp * a.part_stride : nullptr;
            if (EPI == TC_QKV) {
                asm volatile("barrier.sync 2, %0;" ::"n"(kTpEpiThreads) : "memory");  // previous tile's readers
                for (int jj = e; jj < NS; jj += kTpEpiThreads) {
                    const int rr = r0 + jj;
                    int pos = 0, dst = 0;
                    if (rr < a.R) {
                        pos = a.row_pos ? a.row_pos[rr] : a.fixed_pos;
                        const int slot = a.row_slot[rr];
                        dst = a.kv ? a.page_table[(size_t)slot * a.pages_per_stream + pos / kPage] : slot;
                    }
                    s_pos[jj] = pos;
                    s_dst[jj] = dst;
                }
                asm volatile("barrier.sync 2, %0;" ::"n"(kTpEpiThreads) : "memory");
            }
            const bool acc_ok = mbar_wait(&accf_bar[ab], (j >> 1) & 1, a.err, 16);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int gm = mt * kTcM + mrow;
            const float b = (a.bias && kp == 0) ? a.bias[gm] : 0.f;
            for (int n0 = cb; n0 < ce; n0 += 16) {
                float2 pre[16];
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                    pre[jj] = tc_epi_pre<EPI>(a, gm, r0 + n0 + jj, EPI == TC_QKV ? s_pos[n0 + jj] : 0);
                float v[16];
                if (acc_ok) {
                    tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * NS + n0), v);
                } else {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) v[jj] = 0.f;
                }
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    const int n = n0 + jj;
                    tc_epi_one<EPI, NP>(a, outp, gm, r0 + n, N, v[jj], b, EPI == TC_QKV ? s_pos[n] : 0,
                                        EPI == TC_QKV ? s_dst[n] : 0, pre[jj]);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(&acce_bar[ab]);
            if (!acc_ok) break;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
}

// x fp32 [R][768] (optionally LayerNormed) -> activation image with N padded rows; rows
// R..N-1 are written as zeros.  parts = 2 also writes the image of the fp16 remainders
// (x - fp16(x)) right after the first one.  add != null: first the residual add x += add
// (written back to x; the preceding GEMM stored its output, bias included, in add -- or in
// n_add K parts add_stride floats apart, summed in order).  One
// warp per row: lane l holds the 8-element units l, l + 32, l + 64 of the row (one 16-byte
// unit of the image each), the LayerNorm statistics are warp reductions.
constexpr int kBimgUnits = kBimgRowUnits;  // 8-element units per lane
__global__ void __launch_bounds__(256) k_build_bimg(float *__restrict__ x, int ldx, int R, int N,
                                                    const float *__restrict__ ln_w, const float *__restrict__ ln_b,
                                                    int parts, uint8_t *__restrict__ bimg,
                                                    const float *__restrict__ add, int n_add, size_t add_stride) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (n >= N) return;
    const size_t part = (size_t)kHidden * N * 2;
    if (n >= R) {
#pragma unroll
        for (int j = 0; j < kBimgUnits; ++j)
            for (int p = 0; p < parts; ++p)
                *reinterpret_cast<int4 *>(bimg + p * part + bimg_off(n, 8 * (lane + 32 * j), N)) = make_int4(0, 0, 0, 0);
        return;
    }
    float v[kBimgUnits][8];
#pragma unroll
    for (int j = 0; j < kBimgUnits; ++j) {
        float4 *xp = reinterpret_cast<float4 *>(x + (size_t)n * ldx + 8 * (lane + 32 * j));
        float4 a0 = xp[0], a1 = xp[1];
        if (add) {
            // the GEMM's output, or its K parts in order: x + (p0 + p1 + ...)
            const float4 *ap = reinterpret_cast<const float4 *>(add + (size_t)n * ldx + 8 * (lane + 32 * j));
            float4 b0 = ap[0], b1 = ap[1];
            for (int p = 1; p < n_add; ++p) {
                const float4 *cp = reinterpret_cast<const float4 *>(reinterpret_cast<const char *>(ap) + p * add_stride * 4);
                const float4 c0 = cp[0], c1 = cp[1];
                b0 = make_float4(__fadd_rn(b0.x, c0.x), __fadd_rn(b0.y, c0.y), __fadd_rn(b0.z, c0.z), __fadd_rn(b0.w, c0.w));
                b1 = make_float4(__fadd_rn(b1.x, c1.x), __fadd_rn(b1.y, c1.y), __fadd_rn(b1.z, c1.z), __fadd_rn(b1.w, c1.w));
            }
            a0 = make_float4(__fadd_rn(a0.x, b0.x), __fadd_rn(a0.y, b0.y), __fadd_rn(a0.z, b0.z), __fadd_rn(a0.w, b0.w));
            a1 = make_float4(__fadd_rn(a1.x, b1.x), __fadd_rn(a1.y, b1.y), __fadd_rn(a1.z, b1.z), __fadd_rn(a1.w, b1.w));
            xp[0] = a0;
            xp[1] = a1;
        }
        v[j][0] = a0.x; v[j][1] = a0.y; v[j][2] = a0.z; v[j][3] = a0.w;
        v[j][4] = a1.x; v[j][5] = a1.y; v[j][6] = a1.z; v[j][7] = a1.w;
    }
    bimg_row_write(v, lane, n, N, ln_w, ln_b, parts, bimg);
}

// The QKV epilogue of a prefill pass as its own pass over the GEMM's stored output (bias
// included): raw [R][2304] -> RoPE on (2i, 2i + 1) pairs of q and k, q to q_out [R][768], k
// and v appended to the paged fp16 KV -- the same arithmetic as the fused epilogue.  One block
// per row (its position, RoPE row and KV page looked up once), one thread per 4 columns.
constexpr int kQkvRopeThreads = 192;
__global__ void __launch_bounds__(kQkvRopeThreads) k_qkv_rope(const float *__restrict__ raw, int R,
                                                              const int *__restrict__ row_slot,
                                                              const int *__restrict__ row_pos,
                                                              const float2 *__restrict__ rope, float *__restrict__ q_out,
                                                              __half *__restrict__ kv, const int *__restrict__ page_table,
                                                              int pages_per_stream) {
    pdl_enter();
    const int rr = blockIdx.x;
    if (rr >= R) return;
    const int pos = row_pos[rr];
    const int page = page_table[(size_t)row_slot[rr] * pages_per_stream + pos / kPage];
    const float2 *rp = rope + (size_t)pos * (kHeadDim / 2);
    for (int q4 = threadIdx.x; q4 < kQKV / 4; q4 += kQkvRopeThreads) {
        const int gm = 4 * q4;
        const float4 y = *reinterpret_cast<const float4 *>(raw + (size_t)rr * kQKV + gm);
        float o[4] = {y.x, y.y, y.z, y.w};
        if (gm < 2 * kHidden) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const float2 cs = rp[((gm + 2 * p) % kHeadDim) >> 1];
                const float y0 = o[2 * p], y1 = o[2 * p + 1];
                o[2 * p] = __fsub_rn(__fmul_rn(y0, cs.x), __fmul_rn(y1, cs.y));
                o[2 * p + 1] = __fadd_rn(__fmul_rn(y1, cs.x), __fmul_rn(y0, cs.y));
            }
        }
        if (gm < kHidden) {
            *reinterpret_cast<float4 *>(q_out + (size_t)rr * kHidden + gm) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
            const int kvsel = gm < 2 * kHidden ? 0 : 1;
            const int c = gm - kHidden * (1 + kvsel);  // 4 columns of one head
            __half *dst = kv + (size_t)page * kPageHalfs +
                          ((kvsel * kHeads + c / kHeadDim) * kPage + pos % kPage) * kHeadDim + (c % kHeadDim);
            const __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t *>(&h01);
            w.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(dst) = w;
        }
    }
}

// File bytes of one Q8_0_4X4 matrix -> tile layout (qt, st).  One thread per (row, block).
__global__ void k_repack_tiles(const uint8_t *__restrict__ src, int rows, int K, int8_t *__restrict__ qt,
                               __half *__restrict__ st) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = K / 32;
    if (t >= (long long)rows * nb) return;
    const int m = int(t / nb), b = int(t % nb);
    const uint8_t *blk = src + ((size_t)(m >> 2) * nb + b) * 136;
    const int k4 = m & 3;
    const int tile = m / kTcM, mm = m % kTcM, c = b >> 1, hb = b & 1;
    const size_t base = ((size_t)tile * (K / kTcK) + c) * kTcM + mm;
    int8_t *row = qt + base * 64;
    const uint8_t *qs = blk + 8 + k4 * 32;  // 8-byte aligned
#pragma unroll
    for (int p = 0; p < 2; ++p) {  // 16-byte piece j = 2*hb + p
        const int j = 2 * hb + p;
        const uint2 lo = *reinterpret_cast<const uint2 *>(qs + 16 * p);
        const uint2 hi = *reinterpret_cast<const uint2 *>(qs + 16 * p + 8);
        int8_t *dst = row + ((j ^ ((mm >> 1) & 3)) << 4);
        *reinterpret_cast<uint2 *>(dst) = lo;
        *reinterpret_cast<uint2 *>(dst + 8) = hi;
    }
    uint16_t d;
    memcpy(&d, blk + k4 * 2, 2);
    reinterpret_cast<uint16_t *>(st)[base * 2 + hb] = d;
}

}  // namespace
}  // namespace mossgpu
