// codec.cu -- the audio codec decoder (MOSS-Audio-Tokenizer-Nano decoder; reference
// csrc/src/decoder.cpp, csrc/src/audio_layer.cpp, csrc/src/attn_scalar.cpp) on the GPU: the
// step after the LLM path, turning each chunk of 16 x frames codes into 48 kHz stereo samples.
//
//   codes [16][frames] -> 16 codebook rows, each projected 8 -> 512 and summed
//                    (decoder.cpp:226-253 quantize_front) -> q.out [C0 x 512] + bias
//   4 stages: time patch p (x [t][c] -> [t p][c / p], decoder.cpp:73-87), in.w -> d_model
//             256, L transformer layers, out.w;  then a final patch of 240 that turns [t][240]
//             into the interleaved samples (decoder.cpp:221).
//   layer:    x += ls1 * proj(attn(RoPE(qkv(LN1 x))));  x += ls2 * f2(GELU(f1(LN2 x)))
//             (decoder.cpp:116-196); attention has 4 heads x 64, is causal, and each row sees
//             the last `context` rows of its stage (500 / 800 / 1200 / 1600), across chunks
//             through a per-layer K/V ring.
//
// Batched streams.  The reference holds one utterance per AudioDecoder; here one codec holds
// up to max_streams utterances ("codec streams"), each with the reference's streaming state
// (the RoPE offset of every stage, the last `context` K and V rows of every layer), and one
// call decodes a chunk of the same length for any set of them: the rows of all streams run
// through each GEMM together, attention is tiled per (stream, head, 64 rows).
//
// Arithmetic.  The reference computes in fp32 with fp16 matrices (gemm_par on f16 matrices,
// gemv.cpp:331-359).  Here the products run on the tensor cores (mma.sync m16n8k16, fp16
// operands, fp32 accumulation) with every fp32 operand split into fp16 hi + lo (hi = fp16(x),
// lo = fp16(x - hi), ~22 significant bits): a GEMM is W.x_hi + W.x_lo (the fp16 weights are
// exact), a score q.k_hi + q.k_lo... as q_hi.k_hi + q_hi.k_lo + q_lo.k_hi, and p.v likewise.
// The residual stream and each stage's output stay fp32 [rows][channels]; every GEMM input is
// kept as two fp16 planes (hi, lo) that the kernel producing it writes.  The qkv GEMM's
// epilogue applies RoPE and writes q / 8 (exact scaling) and k, v as fp16 hi/lo planes, which is
// also the format of the K/V rings ([slot][context][kh, kl, vh, vl][256] fp16, slot = stream id).  A value that fp16
// cannot hold (|x| >= 65504, or NaN) sets the codec's range flag: the host entry points then
// fail, and the device entry point reports it through mossgpu_codec_status.
#include "../../include/mossgpu.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace mossgpu {
namespace codec {

constexpr int kDModel = 256, kHeads = 4, kHeadDim = 64, kZ = 512, kCbDim = 8, kNCb = 16, kCbSize = 1024;
constexpr int kStages = 4, kLayersTotal = 12;
constexpr int kPatch[kStages] = {4, 2, 2, 2};
constexpr int kContext[kStages] = {500, 800, 1200, 1600};
constexpr int kStageIds[kStages] = {1, 3, 5, 7};
constexpr int kLayerCount[kStages] = {4, 2, 2, 4};
constexpr int kFinalPatch = 240;
constexpr int kRowsPerFrame = 4 * 2 * 2 * 2;  // rows of the last stage per code frame

#define CK(x)                                                                                          \
    do {                                                                                               \
        cudaError_t e_ = (x);                                                                          \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// ------------------------------------------------------------------------------- kernels

// Per-call stream metadata, int32 on the device: sid[n], offset[4][n] (RoPE position of the
// chunk's first row, per stage), ring_start[12][n] and ring_count[12][n] (per layer: physical
// slot of the oldest kept row, rows kept).
struct Meta {
    const int *sid, *offset, *rstart, *rcount;
};

// ---- tensor-core building blocks: mma.sync m16n8k16 (fp16 in, fp32 accumulate), ldmatrix,
// and cp.async (16-byte asynchronous copies from this GPU's own memory; no multicast)
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// (not volatile: a pure register operation, so the compiler may interleave independent ones)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
// src_bytes = 0 reads nothing and fills the 16 destination bytes with zeros
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// (a, b) -> fp16 pairs hi and lo, hi + lo == (a, b) to ~22 significant bits
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// the same, flagging a value outside fp16's range (or a NaN) in *err
__device__ __forceinline__ void split_pair_checked(float a, float b, uint32_t &hi, uint32_t &lo, int *err) {
    if (!(fabsf(a) < 65504.f) || !(fabsf(b) < 65504.f)) *err = 1;
    split_pair(a, b, hi, lo);
}

__device__ __forceinline__ float gelu_erf(float v) {  // audio_layer.cpp:46
    return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
}

// Activation planes: an fp32 activation x [T][K] that a GEMM consumes is kept as two fp16
// planes, hi = fp16(x) and lo = fp16(x - hi) (~22 significant bits), written by the kernel that
// produces x (k_front, k_patch, k_layernorm256, k_window_attn, the GELU epilogue, k_split_rows),
// which also flags a value that fp16 cannot hold.  The GEMMs then only copy and multiply.
struct Planes {
    __half *hi = nullptr, *lo = nullptr;
};

// y[t][r] = sum_k W[r][k] (xh[t][k] + xl[t][k]) (W fp16 [R][K], x as planes [T][K]), then:
//   EPI_PLAIN       y = acc (+ vec[r] when vec is given), fp32
//   EPI_GELU        gelu(acc) as hi/lo planes (the next GEMM's input)
//   EPI_SCALED_ADD  y = y + vec[r] * acc (the layer-scale residual, decoder.cpp:173-177), fp32
//   EPI_QKV         r < 256: q, 256..511: k, 512..767: v of the row; RoPE on q and k at the
//                   row's position (audio_layer.cpp:31-44: frequency exp(-ln(1e4) 2i / 64) of
//                   pair (2i, 2i+1) in each 64-wide head), then q / 8 -> q16 planes and k, v ->
//                   kv16 planes as fp16 hi/lo (an accumulator pair is a RoPE pair)
// Block tile 128 rows x 128 outputs, k step 32, three stages of cp.async copies (x hi, x lo,
// W); 8 warps as 2 x 4, each 64 rows x 32 outputs.  Each k16 step starts its two products from
// zero and is added to the fp32 accumulators with a rounded add: the tensor cores' own
// accumulation does not round to nearest, and a long chain of it into one accumulator biases
// the sum toward zero (~2^-24 per step).
enum { EPI_PLAIN = 0, EPI_GELU = 1, EPI_SCALED_ADD = 2, EPI_QKV = 3 };

// RoPE frequencies exp(-ln(1e4) 2i / 64) of the 32 pairs of a head, computed on the device
// with the expression of audio_layer.cpp:36 (k_rope_freq runs when a codec is created)
__device__ float g_rope_freq[kHeadDim / 2];
__global__ void k_rope_freq() {
    const int i = threadIdx.x;
    if (i < kHeadDim / 2) g_rope_freq[i] = expf(-logf(10000.0f) * 2.0f * (float)i / (float)kHeadDim);
}
constexpr int kTM = 128, kTN = 128, kTK = 32, kTS = 40;  // tile rows, tile outputs, k step, smem row (halves)
constexpr int kGemmStages = 3;
constexpr int kStageHalves = 3 * kTM * kTS;  // x hi, x lo, W
constexpr size_t kGemmSmem = kGemmStages * kStageHalves * sizeof(__half);  // 92,160 bytes

struct Epi {
    const float *vec = nullptr;    // bias (PLAIN) or layer scale (SCALED_ADD)
    float *y = nullptr;            // [T][R] (PLAIN, SCALED_ADD)
    Planes out;                    // GELU: [T][R] hi, lo
    __half *q16 = nullptr;         // QKV: [T][2][256] hi, lo of q / 8
    __half *kv16 = nullptr;        // QKV: [T][4][256] hi, lo of k; hi, lo of v
    const int *offset = nullptr;   // QKV: RoPE position of each stream's first chunk row
    int t_per_stream = 1;          // QKV: rows of one stream in this stage
    int *err = nullptr;            // range flag
};

template <int EPI>
__global__ void __launch_bounds__(256, 2) k_gemm_mma(const __half *__restrict__ W, const __half *__restrict__ xh,
                                                  const __half *__restrict__ xl, int T, int R, int K, Epi ep) {
    extern __shared__ __align__(16) __half gsm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 2, wn = warp & 3, g = lane >> 2, tg = lane & 3;
    const int t0 = blockIdx.y * kTM, r0 = blockIdx.x * kTN;
    // stage st <- k columns k0..k0+31 of the tile's 128 x rows (hi, lo) and 128 W rows: each
    // 512 chunks of 16 bytes, chunk c = row c / 4, columns 8 (c % 4)..+7; thread tid copies
    // chunks tid and tid + 256 of each (rows past T or R, columns past K: zeros)
    auto issue = [&](int st, int k0) {
        __half *ah = gsm + st * kStageHalves, *al = ah + kTM * kTS, *bt = al + kTM * kTS;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int c = tid + 256 * j, row = c >> 2, kc = (c & 3) * 8;
            const int t = t0 + row, r = r0 + row, k = k0 + kc;
            const bool okx = t < T && k < K, okw = r < R && k < K;
            const size_t xo = okx ? (size_t)t * K + k : 0;
            cp_async16(ah + row * kTS + kc, xh + xo, okx ? 16 : 0);
            cp_async16(al + row * kTS + kc, xl + xo, okx ? 16 : 0);
            cp_async16(bt + row * kTS + kc, okw ? W + (size_t)r * K + k : W, okw ? 16 : 0);
        }
        cp_async_commit();
    };
    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;
    const int nk = (K + kTK - 1) / kTK;
    // prologue: stages 0 .. S-2 in flight (empty commit groups keep the group count uniform)
#pragma unroll
    for (int s = 0; s < kGemmStages - 1; ++s) {
        if (s < nk)
            issue(s, s * kTK);
        else
            cp_async_commit();
    }
    for (int it = 0; it < nk; ++it) {
        cp_async_wait<kGemmStages - 2>();  // this thread's copies of stage `it` have landed
        __syncthreads();                   // everyone's; and stage it-1's buffer is free again
        const int nxt = it + kGemmStages - 1;
        if (nxt < nk)
            issue(nxt % kGemmStages, nxt * kTK);
        else
            cp_async_commit();
        const int st = it % kGemmStages;
        const __half *ah = gsm + st * kStageHalves, *al = ah + kTM * kTS, *bt = ah + 2 * kTM * kTS;
#pragma unroll
        for (int kk = 0; kk < kTK; kk += 16) {
            uint32_t bf[4][2];
#pragma unroll
            for (int nj = 0; nj < 4; nj += 2) {
                uint32_t r[4];
                ldsm_x4(r, bt + (wn * 32 + nj * 8 + (lane & 7) + ((lane >> 4) << 3)) * kTS + kk + ((lane >> 3) & 1) * 8);
                bf[nj][0] = r[0];
                bf[nj][1] = r[1];
                bf[nj + 1][0] = r[2];
                bf[nj + 1][1] = r[3];
            }
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) {
                uint32_t fh[4], fl[4];
                const int off = (wm * 64 + mi * 16 + (lane & 15)) * kTS + kk + (lane >> 4) * 8;
                ldsm_x4(fh, ah + off);
                ldsm_x4(fl, al + off);
#pragma unroll
                for (int nj = 0; nj < 4; ++nj) {
                    float part[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(part, fh, bf[nj][0], bf[nj][1]);
                    mma16816(part, fl, bf[nj][0], bf[nj][1]);
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[mi][nj][c] += part[c];
                }
            }
        }
    }
    cp_async_wait<0>();  // only empty groups can be pending here
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int nj = 0; nj < 4; ++nj) {
            const int c = r0 + wn * 32 + nj * 8 + 2 * tg;  // even; R is a multiple of 8
            if (c >= R) continue;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int t = t0 + wm * 64 + mi * 16 + g + 8 * h;
                if (t >= T) continue;
                float v0 = acc[mi][nj][2 * h], v1 = acc[mi][nj][2 * h + 1];
                if (EPI == EPI_QKV) {
                    const int which = c >> 8, d = c & 255;
                    if (which < 2) {
                        const int b = t / ep.t_per_stream;
                        const int pos = ep.offset[b] + (t - b * ep.t_per_stream);
                        const float ang = (float)pos * g_rope_freq[(d & 63) >> 1];
                        const float cs = cosf(ang), sn = sinf(ang);
                        const float x0 = v0, x1 = v1;
                        v0 = x0 * cs - x1 * sn;
                        v1 = x0 * sn + x1 * cs;
                    }
                    uint32_t hi, lo;
                    if (which == 0) {
                        split_pair_checked(v0 * 0.125f, v1 * 0.125f, hi, lo, ep.err);
                        *reinterpret_cast<uint32_t *>(ep.q16 + ((size_t)t * 2 + 0) * kDModel + d) = hi;
                        *reinterpret_cast<uint32_t *>(ep.q16 + ((size_t)t * 2 + 1) * kDModel + d) = lo;
                    } else {
                        const int plane = which == 1 ? 0 : 2;
                        split_pair_checked(v0, v1, hi, lo, ep.err);
                        *reinterpret_cast<uint32_t *>(ep.kv16 + ((size_t)t * 4 + plane) * kDModel + d) = hi;
                        *reinterpret_cast<uint32_t *>(ep.kv16 + ((size_t)t * 4 + plane + 1) * kDModel + d) = lo;
                    }
                } else if (EPI == EPI_GELU) {
                    uint32_t hi, lo;
                    split_pair_checked(gelu_erf(v0), gelu_erf(v1), hi, lo, ep.err);
                    *reinterpret_cast<uint32_t *>(ep.out.hi + (size_t)t * R + c) = hi;
                    *reinterpret_cast<uint32_t *>(ep.out.lo + (size_t)t * R + c) = lo;
                } else {
                    float2 *dst = reinterpret_cast<float2 *>(ep.y + (size_t)t * R + c);
                    if (EPI == EPI_PLAIN) {
                        if (ep.vec) {
                            v0 += ep.vec[c];
                            v1 += ep.vec[c + 1];
                        }
                        *dst = make_float2(v0, v1);
                    } else {
                        const float2 o = *dst;
                        *dst = make_float2(o.x + ep.vec[c] * v0, o.y + ep.vec[c + 1] * v1);
                    }
                }
            }
        }
}

// z[row][r] = sum_i (b_i[r] + sum_k W_i[r][k] e_i[k]), e_i = codebook i's row for the row's code
// (decoder.cpp:229-244: the same per-element order).  codes [n][16][frames], row = b frames + f;
// a code outside [0, 1024) is clamped (the host entry points reject such codes first).
__global__ void k_front(const int *__restrict__ codes, int frames, const float *const *__restrict__ cb,
                        const float *const *__restrict__ ow, const float *const *__restrict__ ob, Planes z,
                        int *__restrict__ err) {
    const int row = blockIdx.x;
    const int b = row / frames, f = row - b * frames;
    __shared__ float emb[kNCb][kCbDim];
    if (threadIdx.x < kNCb * kCbDim) {
        const int i = threadIdx.x / kCbDim, k = threadIdx.x % kCbDim;
        int code = codes[((size_t)b * kNCb + i) * frames + f];
        code = code < 0 ? 0 : (code >= kCbSize ? kCbSize - 1 : code);
        emb[i][k] = cb[i][(size_t)code * kCbDim + k];
    }
    __syncthreads();
    __shared__ float zs[kZ];
    for (int r = threadIdx.x; r < kZ; r += blockDim.x) {
        float zi = 0.f;
        for (int i = 0; i < kNCb; ++i) {
            const float *w = ow[i] + (size_t)r * kCbDim;
            float acc = ob[i][r];
#pragma unroll
            for (int k = 0; k < kCbDim; ++k) acc += w[k] * emb[i][k];
            zi += acc;
        }
        zs[r] = zi;
    }
    __syncthreads();
    for (int r2 = threadIdx.x; r2 < kZ / 2; r2 += blockDim.x) {
        uint32_t hi, lo;
        split_pair_checked(zs[2 * r2], zs[2 * r2 + 1], hi, lo, err);
        reinterpret_cast<uint32_t *>(z.hi + (size_t)row * kZ)[r2] = hi;
        reinterpret_cast<uint32_t *>(z.lo + (size_t)row * kZ)[r2] = lo;
    }
}

// x [t][c] -> out [t p][c / p]: out[t p + j][ci] = x[t][ci p + j] (decoder.cpp:73-87), written
// as hi/lo planes two columns at a time (c / p is even)
__global__ void k_patch(const float *__restrict__ x, size_t T, int c, int p, Planes out, int *__restrict__ err) {
    const size_t n2 = T * c / 2;
    const int d = c / p;
    for (size_t i2 = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i2 < n2; i2 += (size_t)gridDim.x * blockDim.x) {
        const size_t i = 2 * i2;
        const size_t row = i / d;
        const int ci = (int)(i - row * d);
        const size_t t = row / p;
        const int j = (int)(row - t * p);
        const float *src = x + t * c + (size_t)ci * p + j;
        uint32_t hi, lo;
        split_pair_checked(src[0], src[p], hi, lo, err);
        reinterpret_cast<uint32_t *>(out.hi)[i2] = hi;
        reinterpret_cast<uint32_t *>(out.lo)[i2] = lo;
    }
}

// y [n] fp32 -> hi/lo planes (the input of a stage's out.w, read from the residual stream)
__global__ void k_split_rows(const float *__restrict__ y, size_t n, Planes out, int *__restrict__ err) {
    const size_t n2 = n / 2;
    for (size_t i2 = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i2 < n2; i2 += (size_t)gridDim.x * blockDim.x) {
        const float2 v = reinterpret_cast<const float2 *>(y)[i2];
        uint32_t hi, lo;
        split_pair_checked(v.x, v.y, hi, lo, err);
        reinterpret_cast<uint32_t *>(out.hi)[i2] = hi;
        reinterpret_cast<uint32_t *>(out.lo)[i2] = lo;
    }
}

// LayerNorm of 256-wide rows, one warp per row, lane l holding the column pairs l + 32 j
// (audio_layer.cpp:17-29), written as hi/lo planes
__global__ void k_layernorm256(const float *__restrict__ x, int T, const float *__restrict__ w,
                               const float *__restrict__ bias, Planes out, int *__restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const float2 *row = reinterpret_cast<const float2 *>(x + (size_t)t * kDModel);
    float2 v[4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[j] = row[lane + 32 * j];
        s += v[j].x + v[j].y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)kDModel;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float d0 = v[j].x - mean, d1 = v[j].y - mean;
        q += d0 * d0 + d1 * d1;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = 1.0f / sqrtf(q / (float)kDModel + 1e-5f);
    uint32_t *oh = reinterpret_cast<uint32_t *>(out.hi + (size_t)t * kDModel);
    uint32_t *ol = reinterpret_cast<uint32_t *>(out.lo + (size_t)t * kDModel);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int k = 2 * (lane + 32 * j);
        uint32_t hi, lo;
        split_pair_checked((v[j].x - mean) * inv * w[k] + bias[k], (v[j].y - mean) * inv * w[k + 1] + bias[k + 1], hi,
                           lo, err);
        oh[lane + 32 * j] = hi;
        ol[lane + 32 * j] = lo;
    }
}

// Windowed causal attention of a chunk (attn_scalar.cpp:165-203 attention_window_scalar):
// chunk row i of a stream sees keys u in [max(0, i + n - window + 1), i + n], where keys
// 0..n-1 are the stream's ring (physical slot (start + u) % window) and keys n.. the chunk's
// own rows.  Block = (64 rows, head, stream), 4 warps of 16 rows; keys in tiles of 64 copied
// (cp.async, two stages) into shared memory as fp16 hi/lo planes of k and v; scores and the
// weighted sum on the tensor cores (3 products each for the hi/lo split), softmax online
// across tiles with the probabilities scaled by 1024 (exact) so that small ones stay normal
// fp16 numbers in the split.  Output: hi/lo planes [rows][256] (the proj GEMM's input); each
// output is a convex combination of v values, which the qkv epilogue range-checked already.
constexpr int kQT = 64, kKT = 64, kAS = 72;  // rows per block, keys per tile, smem row (halves)
constexpr int kPlane = kKT * kAS;            // halves per plane of a tile
constexpr size_t kAttnSmem = 2 * 4 * kPlane * sizeof(__half);  // 73,728 bytes

__global__ void __launch_bounds__(128, 3) k_window_attn(const __half *__restrict__ q16, const __half *__restrict__ kv16,
                                                     int t, const __half *__restrict__ ring, int window, int layer,
                                                     Meta meta, int n_streams, Planes out) {
    extern __shared__ __align__(16) __half asmem[];
    const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * kQT;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tg = lane & 3;
    const int n = meta.rcount[layer * n_streams + b], start = meta.rstart[layer * n_streams + b];
    const __half *rbase = ring + (size_t)meta.sid[b] * window * 4 * kDModel;
    const size_t row0 = (size_t)b * t;  // the stream's first chunk row
    const int nq = min(kQT, t - q0);
    const int ulo = max(0, q0 + n - window + 1), uhi = q0 + nq - 1 + n;
    const int i0 = q0 + warp * 16;       // this warp's first chunk row
    const bool wact = warp * 16 < nq;
    const int wlo = max(0, i0 + n - window + 1), whi = min(i0 + 15, q0 + nq - 1) + n;
    const int ra = i0 + g, rb = ra + 8;  // this thread's two rows
    const bool oka = ra - q0 < nq, okb = rb - q0 < nq;

    auto issue_tile = [&](int st, int u0) {
        __half *dst = asmem + st * 4 * kPlane;
        for (int c = tid; c < kKT * 32; c += 128) {  // 64 keys x 4 planes x 8 chunks of 16 bytes
            const int key = c >> 5, plane = (c >> 3) & 3, ch = c & 7;
            const int u = u0 + key;
            const __half *src = ring;
            int bytes = 0;
            if (u <= uhi) {
                src = u < n ? rbase + ((size_t)((start + u) % window) * 4 + plane) * kDModel + h * kHeadDim + ch * 8
                            : kv16 + ((row0 + (size_t)(u - n)) * 4 + plane) * kDModel + h * kHeadDim + ch * 8;
                bytes = 16;
            }
            cp_async16(dst + plane * kPlane + key * kAS + ch * 8, src, bytes);
        }
        cp_async_commit();
    };

    // q fragments (hi, lo) of rows ra, rb: a0 (ra, d), a1 (rb, d), a2 (ra, d + 8), a3 (rb, d + 8)
    uint32_t qh[4][4], ql[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int row = (r & 1) ? rb : ra;
            const bool ok = (r & 1) ? okb : oka;
            const int d = h * kHeadDim + ks * 16 + 2 * tg + (r >> 1) * 8;
            qh[ks][r] = ok ? *reinterpret_cast<const uint32_t *>(q16 + ((row0 + row) * 2 + 0) * kDModel + d) : 0u;
            ql[ks][r] = ok ? *reinterpret_cast<const uint32_t *>(q16 + ((row0 + row) * 2 + 1) * kDModel + d) : 0u;
        }

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[i][c] = 0.f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
    const int ntiles = (uhi - ulo) / kKT + 1;
    issue_tile(0, ulo);
    for (int it = 0; it < ntiles; ++it) {
        const int st = it & 1, u0 = ulo + it * kKT;
        if (it + 1 < ntiles) {
            issue_tile(st ^ 1, u0 + kKT);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (wact && u0 <= whi && u0 + kKT - 1 >= wlo) {
            const __half *kh = asmem + st * 4 * kPlane, *kl = kh + kPlane, *vh = kh + 2 * kPlane,
                         *vl = kh + 3 * kPlane;
            float s[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                for (int nj = 0; nj < 8; nj += 2) {
                    uint32_t rh[4], rl[4];
                    const int off = (nj * 8 + (lane & 7) + ((lane >> 4) << 3)) * kAS + ks * 16 + ((lane >> 3) & 1) * 8;
                    ldsm_x4(rh, kh + off);
                    ldsm_x4(rl, kl + off);
                    mma16816(s[nj], qh[ks], rh[0], rh[1]);
                    mma16816(s[nj + 1], qh[ks], rh[2], rh[3]);
                    mma16816(s[nj], qh[ks], rl[0], rl[1]);
                    mma16816(s[nj + 1], qh[ks], rl[2], rl[3]);
                    mma16816(s[nj], ql[ks], rh[0], rh[1]);
                    mma16816(s[nj + 1], ql[ks], rh[2], rh[3]);
                }
            // mask to each row's window (only tiles at the window's edges, or with rows past the
            // chunk, need it), then the online softmax of rows ra (c = 0, 1) and rb (c = 2, 3)
            const bool inner = i0 + 15 < q0 + nq && u0 >= i0 + 15 + n - window + 1 && u0 + kKT - 1 <= i0 + n;
            if (!inner) {
                const int alo = ra + n - window + 1, ahi = ra + n, blo = alo + 8, bhi = ahi + 8;
#pragma unroll
                for (int nj = 0; nj < 8; ++nj)
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const int u = u0 + nj * 8 + 2 * tg + c;
                        s[nj][c] = (oka && u >= alo && u <= ahi) ? s[nj][c] : -INFINITY;
                        s[nj][2 + c] = (okb && u >= blo && u <= bhi) ? s[nj][2 + c] : -INFINITY;
                    }
            }
            float xa = -INFINITY, xb = -INFINITY;
#pragma unroll
            for (int nj = 0; nj < 8; ++nj) {
                xa = fmaxf(xa, fmaxf(s[nj][0], s[nj][1]));
                xb = fmaxf(xb, fmaxf(s[nj][2], s[nj][3]));
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, off));
                xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, off));
            }
            const float na = fmaxf(ma, xa), nb = fmaxf(mb, xb);
            // __expf: the hardware exponential (relative error ~1e-7 near 0, growing with |x| where
            // the weights are negligible); a row with no valid key yet keeps weight 0
            const float fa = na == -INFINITY ? 1.f : __expf(ma - na), fb = nb == -INFINITY ? 1.f : __expf(mb - nb);
            const float ca = na == -INFINITY ? 0.f : na, cb = nb == -INFINITY ? 0.f : nb;
            float sa = 0.f, sb = 0.f;
#pragma unroll
            for (int nj = 0; nj < 8; ++nj)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    s[nj][c] = __expf(s[nj][c] - ca) * 1024.f;
                    s[nj][2 + c] = __expf(s[nj][2 + c] - cb) * 1024.f;
                    sa += s[nj][c];
                    sb += s[nj][2 + c];
                }
            la = la * fa + sa;
            lb = lb * fb + sb;
            ma = na;
            mb = nb;
            // ov = p v over the tile's 64 keys, 16 at a time, from zero; then o = o f + ov with
            // rounded fp32 arithmetic (a short tensor-core chain per tile, see k_gemm_mma)
            float ov[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) ov[i][c] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t ph[4], pl[4];
                split_pair(s[2 * ks][0], s[2 * ks][1], ph[0], pl[0]);
                split_pair(s[2 * ks][2], s[2 * ks][3], ph[1], pl[1]);
                split_pair(s[2 * ks + 1][0], s[2 * ks + 1][1], ph[2], pl[2]);
                split_pair(s[2 * ks + 1][2], s[2 * ks + 1][3], ph[3], pl[3]);
#pragma unroll
                for (int nd = 0; nd < 8; nd += 2) {
                    uint32_t rh[4], rl[4];
                    const int off = (ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3)) * kAS + (nd + (lane >> 4)) * 8;
                    ldsm_x4_t(rh, vh + off);
                    ldsm_x4_t(rl, vl + off);
                    mma16816(ov[nd], ph, rh[0], rh[1]);
                    mma16816(ov[nd + 1], ph, rh[2], rh[3]);
                    mma16816(ov[nd], ph, rl[0], rl[1]);
                    mma16816(ov[nd + 1], ph, rl[2], rl[3]);
                    mma16816(ov[nd], pl, rh[0], rh[1]);
                    mma16816(ov[nd + 1], pl, rh[2], rh[3]);
                }
            }
#pragma unroll
            for (int nd = 0; nd < 8; ++nd) {
                o[nd][0] = o[nd][0] * fa + ov[nd][0];
                o[nd][1] = o[nd][1] * fa + ov[nd][1];
                o[nd][2] = o[nd][2] * fb + ov[nd][2];
                o[nd][3] = o[nd][3] * fb + ov[nd][3];
            }
        }
        __syncthreads();  // every warp is done with this stage before the next issue refills it
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
        la += __shfl_xor_sync(0xffffffffu, la, off);
        lb += __shfl_xor_sync(0xffffffffu, lb, off);
    }
    if (!wact) return;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
        const int d = h * kHeadDim + nd * 8 + 2 * tg;
        uint32_t hi, lo;
        if (oka) {
            split_pair(o[nd][0] / la, o[nd][1] / la, hi, lo);
            *reinterpret_cast<uint32_t *>(out.hi + (row0 + ra) * kDModel + d) = hi;
            *reinterpret_cast<uint32_t *>(out.lo + (row0 + ra) * kDModel + d) = lo;
        }
        if (okb) {
            split_pair(o[nd][2] / lb, o[nd][3] / lb, hi, lo);
            *reinterpret_cast<uint32_t *>(out.hi + (row0 + rb) * kDModel + d) = hi;
            *reinterpret_cast<uint32_t *>(out.lo + (row0 + rb) * kDModel + d) = lo;
        }
    }
}

// Append each stream's chunk K and V rows (kv16 planes) to its ring (decoder.cpp:150-169):
// chunk row i goes to slot (start + n + i) % window; only the last `window` rows of a chunk can
// survive, so only they are written.  One row = 4 planes x 256 halves = 128 x 16 bytes.
__global__ void k_ring_append(const __half *__restrict__ kv16, int t, int n_streams, __half *__restrict__ ring,
                              int window, int layer, Meta meta) {
    const int first = max(0, t - window);
    const int rows = t - first;
    const size_t total = (size_t)n_streams * rows * 128;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx & 127);
        const size_t rr = idx >> 7;
        const int b = (int)(rr / rows), i = first + (int)(rr % rows);
        const int n = meta.rcount[layer * n_streams + b], start = meta.rstart[layer * n_streams + b];
        const size_t slot = (size_t)meta.sid[b] * window + (size_t)((start + n + i) % window);
        reinterpret_cast<uint4 *>(ring + slot * 4 * kDModel)[c] =
            reinterpret_cast<const uint4 *>(kv16 + ((size_t)b * t + i) * 4 * kDModel)[c];
    }
}

// ------------------------------------------------------------------------------- host

// kernel classes of the optional per-launch profile (mossgpu_codec_profile)
enum Kind { KD_FRONT = 0, KD_GEMM, KD_PATCH, KD_LAYERNORM, KD_ATTN, KD_RING, KD_SPLIT, KD_COUNT };
const char *const kKindNames[KD_COUNT] = {"k_front", "k_gemm_mma", "k_patch", "k_layernorm256",
                                          "k_window_attn", "k_ring_append", "k_split_rows"};

struct Mat {
    __half *w = nullptr;
    int rows = 0, cols = 0;
};

struct Layer {
    Mat attn, proj, f1, f2;
    float *n1w, *n1b, *n2w, *n2b, *ls1, *ls2;
    __half *ring = nullptr;  // [slots][context][kh, kl, vh, vl][256]
};

struct Stage {
    Mat in, out;
    std::vector<Layer> layers;
};

// one codec stream's place in the reference's streaming state (decoder.h:48-56)
struct SlotState {
    bool open = false;
    int offset[kStages] = {};
    int start[kLayersTotal] = {};
    int count[kLayersTotal] = {};
};

class Codec {
public:
    Codec(const std::string &path, int device, int max_streams, int max_batch_frames)
        : device_(device), max_streams_(max_streams), max_frames_(max_batch_frames) {
        if (max_streams <= 0 || max_batch_frames <= 0)
            throw std::runtime_error("max_streams and max_batch_frames must be positive");
        if (max_streams > 65535) throw std::runtime_error("max_streams must be at most 65535");
        if (max_batch_frames > (1 << 20)) throw std::runtime_error("max_batch_frames must be at most 1048576");
        CK(cudaSetDevice(device));
        k_rope_freq<<<1, 32>>>();
        CK(cudaGetLastError());
        CK(cudaDeviceSynchronize());
        CK(cudaFuncSetAttribute(k_window_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem)));
        CK(cudaFuncSetAttribute(k_gemm_mma<EPI_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemmSmem)));
        CK(cudaFuncSetAttribute(k_gemm_mma<EPI_GELU>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemmSmem)));
        CK(cudaFuncSetAttribute(k_gemm_mma<EPI_SCALED_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kGemmSmem)));
        CK(cudaFuncSetAttribute(k_gemm_mma<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemmSmem)));
        slots_.resize(size_t(max_streams) + 1);  // the last slot serves decode()
        load(path);
        // activation buffers, each sized for its widest use over the stages
        const size_t F = size_t(max_frames_);
        size_t x_elems = F * size_t(std::max(c0_, kZ)), y_elems = 0, ffn_elems = 0;
        size_t rows = F;
        for (int s = 0; s < kStages; ++s) {
            rows *= kPatch[s];
            x_elems = std::max(x_elems, rows * size_t(stages_[size_t(s)].out.rows));
            y_elems = std::max(y_elems, rows * kDModel);
            for (auto &l : stages_[size_t(s)].layers) ffn_elems = std::max(ffn_elems, rows * size_t(l.f1.rows));
        }
        xa_ = alloc<float>(x_elems);
        y_ = alloc<float>(y_elems);
        q16_ = alloc<__half>(y_elems * 2);
        kv16_ = alloc<__half>(y_elems * 4);
        // every GEMM input: the front's [F][512], a patched [rows][c / p] (x_elems), the
        // [rows][256] activations, the [rows][FFN] GELU output
        const size_t plane = std::max({F * kZ, x_elems, y_elems, ffn_elems});
        for (Planes *pl : {&p0_, &p1_}) {
            pl->hi = alloc<__half>(plane);
            pl->lo = alloc<__half>(plane);
        }
        err_ = alloc<int>(1);
        CK(cudaMemset(err_, 0, sizeof(int)));
        codes_ = alloc<int>(size_t(kNCb) * F);
        meta_d_ = alloc<int>(size_t(1 + kStages + 2 * kLayersTotal) * (size_t(max_streams_) + 1));
        pcm_ = alloc<float>(F * size_t(samples_per_frame()));
    }
    ~Codec() {
        cudaSetDevice(device_);
        cudaDeviceSynchronize();
        for (cudaEvent_t e : events_) cudaEventDestroy(e);
        for (void *p : owned_) cudaFree(p);
    }

    // Per-launch profile: while enabled, every launch is bracketed by two events on the
    // codec's stream; profile_read synchronises, adds up the time of each kernel class and
    // starts over.  The events add a gap to every launch; callers subtract it.
    void set_profile(bool on) {
        profile_ = on;
        marks_.clear();
    }
    void profile_read(float *ms, int *launches) {
        CK(cudaStreamSynchronize(stream_));
        for (int k = 0; k < KD_COUNT; ++k) {
            ms[k] = 0.f;
            launches[k] = 0;
        }
        for (size_t i = 0; i < marks_.size(); ++i) {
            float t = 0.f;
            CK(cudaEventElapsedTime(&t, events_[2 * i], events_[2 * i + 1]));
            ms[marks_[i]] += t;
            launches[marks_[i]] += 1;
        }
        marks_.clear();
    }

    int device() const { return device_; }
    int samples_per_frame() const { return kRowsPerFrame * kFinalPatch; }
    size_t device_bytes() const { return allocated_; }
    void set_stream(cudaStream_t s) { stream_ = s; }

    int open() {
        for (int i = 0; i < max_streams_; ++i)
            if (!slots_[size_t(i)].open) {
                slots_[size_t(i)] = SlotState{};
                slots_[size_t(i)].open = true;
                return i;
            }
        throw std::runtime_error("all " + std::to_string(max_streams_) + " codec streams are open");
    }
    void close(int sid) {
        check_sid(sid);
        slots_[size_t(sid)].open = false;
    }
    void reset(int sid) {  // AudioDecoder::reset_stream (decoder.cpp:105-114)
        check_sid(sid);
        slots_[size_t(sid)] = SlotState{};
        slots_[size_t(sid)].open = true;
    }

    // Enqueue the decode of `frames` frames for n streams; codes (device) [n][16][frames],
    // pcm (device) [n][frames * samples_per_frame].
    void decode_device(const int *sids, int n, const int *codes_dev, int frames, float *pcm_dev) {
        if (n <= 0 || frames <= 0) return;
        if (size_t(n) * size_t(frames) > size_t(max_frames_))
            throw std::runtime_error("a call decodes at most max_batch_frames = " + std::to_string(max_frames_) +
                                     " frames (streams x frames)");
        std::vector<char> seen(slots_.size(), 0);
        for (int b = 0; b < n; ++b) {
            const int s = sids[b];
            if (s < 0 || s >= int(slots_.size()) || !slots_[size_t(s)].open)
                throw std::runtime_error("codec stream " + std::to_string(s) + " is not open");
            if (seen[size_t(s)]++) throw std::runtime_error("codec stream " + std::to_string(s) + " repeats in a call");
        }
        // metadata: sid[n], offset[4][n], start[12][n], count[12][n]
        std::vector<int> meta(size_t(1 + kStages + 2 * kLayersTotal) * size_t(n));
        int *m_sid = meta.data(), *m_off = m_sid + n, *m_start = m_off + kStages * n,
            *m_cnt = m_start + kLayersTotal * n;
        for (int b = 0; b < n; ++b) {
            const SlotState &st = slots_[size_t(sids[b])];
            m_sid[b] = sids[b];
            for (int s = 0; s < kStages; ++s) m_off[s * n + b] = st.offset[s];
            for (int l = 0; l < kLayersTotal; ++l) {
                m_start[l * n + b] = st.start[l];
                m_cnt[l * n + b] = st.count[l];
            }
        }
        // pageable source: the copy has read it by the time the call returns
        CK(cudaMemcpyAsync(meta_d_, meta.data(), meta.size() * sizeof(int), cudaMemcpyHostToDevice, stream_));
        const Meta md{meta_d_, meta_d_ + n, meta_d_ + (1 + kStages) * n, meta_d_ + (1 + kStages + kLayersTotal) * n};
        run(md, n, codes_dev, frames, pcm_dev);
        // advance every stream's state as the reference's decode_chunk does
        for (int b = 0; b < n; ++b) {
            SlotState &st = slots_[size_t(sids[b])];
            int t = frames, li = 0;
            for (int s = 0; s < kStages; ++s) {
                t *= kPatch[s];
                const int cap = kContext[s];
                for (int k = 0; k < kLayerCount[s]; ++k, ++li) {
                    const long long total = (long long)st.count[li] + t;
                    if (total > cap) {
                        st.start[li] = int((st.start[li] + (total - cap)) % cap);
                        st.count[li] = cap;
                    } else {
                        st.count[li] = int(total);
                    }
                }
                st.offset[s] += t;
            }
        }
    }

    // host buffers: codes [n][16][frames] -> pcm [n][frames * samples_per_frame]
    void decode_host(const int *sids, int n, const int32_t *codes, int frames, float *pcm, size_t cap) {
        if (n <= 0 || frames <= 0) return;
        const size_t spf = size_t(samples_per_frame());
        if (cap < size_t(n) * size_t(frames) * spf)
            throw std::runtime_error("output buffer smaller than n * frames * samples_per_frame");
        if (size_t(n) * size_t(frames) > size_t(max_frames_))
            throw std::runtime_error("a call decodes at most max_batch_frames = " + std::to_string(max_frames_) +
                                     " frames (streams x frames)");
        const size_t nc = size_t(n) * kNCb * size_t(frames);
        for (size_t i = 0; i < nc; ++i)
            if (codes[i] < 0 || codes[i] >= kCbSize)
                throw std::runtime_error("code " + std::to_string(codes[i]) + " outside [0, 1024)");
        CK(cudaMemcpyAsync(codes_, codes, nc * sizeof(int), cudaMemcpyHostToDevice, stream_));
        decode_device(sids, n, codes_, frames, pcm_);
        CK(cudaMemcpyAsync(pcm, pcm_, size_t(n) * size_t(frames) * spf * sizeof(float), cudaMemcpyDeviceToHost,
                           stream_));
        if (status() != 0)
            throw std::runtime_error("an activation left the fp16 range (|x| >= 65504 or NaN); the streams of this "
                                     "call must be reset");
    }

    // Synchronise the codec's stream and return (and clear) the range flag: 1 when a value of
    // some call since the last read could not be held in fp16.
    int status() {
        int v = 0;
        CK(cudaMemcpyAsync(&v, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        if (v) CK(cudaMemset(err_, 0, sizeof(int)));
        return v;
    }

    // AudioDecoder::decode (decoder.cpp:254-280): the whole utterance from a clean state; the
    // streaming form over pieces of at most max_batch_frames frames computes the same rows.
    void decode_whole(const int32_t *codes, int frames, float *pcm, size_t cap) {
        if (frames <= 0) return;
        const size_t spf = size_t(samples_per_frame());
        if (cap < size_t(frames) * spf) throw std::runtime_error("output buffer smaller than frames * samples_per_frame");
        const int sid = max_streams_;
        slots_[size_t(sid)] = SlotState{};
        slots_[size_t(sid)].open = true;
        std::vector<int32_t> piece;
        try {
            for (int f0 = 0; f0 < frames; f0 += max_frames_) {
                const int k = std::min(max_frames_, frames - f0);
                piece.resize(size_t(kNCb) * size_t(k));
                for (int i = 0; i < kNCb; ++i)
                    std::memcpy(piece.data() + size_t(i) * k, codes + size_t(i) * frames + f0, sizeof(int32_t) * k);
                decode_host(&sid, 1, piece.data(), k, pcm + size_t(f0) * spf, size_t(k) * spf);
            }
        } catch (...) {
            slots_[size_t(sid)].open = false;
            throw;
        }
        slots_[size_t(sid)].open = false;
    }

    int launches_per_call() const {
        int l = 2;
        for (auto &s : stages_) l += 4 + 8 * int(s.layers.size());  // patch, in.w, split, out.w + layers
        return l;
    }

private:
    // bracket the next launch with a pair of events when profiling
    void mark_begin(int kind) {
        if (!profile_) return;
        const size_t i = marks_.size();
        while (events_.size() < 2 * (i + 1)) {
            cudaEvent_t e;
            CK(cudaEventCreate(&e));
            events_.push_back(e);
        }
        marks_.push_back(kind);
        CK(cudaEventRecord(events_[2 * i], stream_));
    }
    void mark_end() {
        if (profile_) CK(cudaEventRecord(events_[2 * (marks_.size() - 1) + 1], stream_));
    }

    void check_sid(int sid) const {
        if (sid < 0 || sid >= max_streams_ || !slots_[size_t(sid)].open)
            throw std::runtime_error("codec stream " + std::to_string(sid) + " is not open");
    }

    template <class T>
    T *alloc(size_t n) {
        void *p = nullptr;
        const size_t bytes = std::max<size_t>(n, 1) * sizeof(T);
        CK(cudaMalloc(&p, bytes));
        owned_.push_back(p);
        allocated_ += bytes;
        return static_cast<T *>(p);
    }

    void gemm(const Mat &m, const Planes &x, int T, int epi, Epi ep) {
        const dim3 grid((m.rows + kTN - 1) / kTN, (T + kTM - 1) / kTM);
        ep.err = err_;
        mark_begin(KD_GEMM);
        if (epi == EPI_PLAIN)
            k_gemm_mma<EPI_PLAIN><<<grid, 256, kGemmSmem, stream_>>>(m.w, x.hi, x.lo, T, m.rows, m.cols, ep);
        else if (epi == EPI_GELU)
            k_gemm_mma<EPI_GELU><<<grid, 256, kGemmSmem, stream_>>>(m.w, x.hi, x.lo, T, m.rows, m.cols, ep);
        else if (epi == EPI_SCALED_ADD)
            k_gemm_mma<EPI_SCALED_ADD><<<grid, 256, kGemmSmem, stream_>>>(m.w, x.hi, x.lo, T, m.rows, m.cols, ep);
        else
            k_gemm_mma<EPI_QKV><<<grid, 256, kGemmSmem, stream_>>>(m.w, x.hi, x.lo, T, m.rows, m.cols, ep);
        CK(cudaGetLastError());
        mark_end();
    }
    static Epi out(float *y, const float *vec = nullptr) {
        Epi e;
        e.y = y;
        e.vec = vec;
        return e;
    }
    static int blocks_for(size_t items) { return int(std::min<size_t>((items + 255) / 256, 148 * 16)); }

    // The activation planes: p0_ and p1_ alternate so that no kernel reads the planes it writes
    // (LN1 -> p0 -> qkv; attention -> p1 -> proj; LN2 -> p0 -> f1 -> p1 -> f2).
    void run(const Meta &md, int n, const int *codes, int frames, float *pcm) {
        int rows = n * frames;  // all streams' rows of the current stage
        mark_begin(KD_FRONT);
        k_front<<<rows, 256, 0, stream_>>>(codes, frames, d_cb_, d_ow_, d_ob_, p0_, err_);
        CK(cudaGetLastError());
        mark_end();
        gemm(q_out_, p0_, rows, EPI_PLAIN, out(xa_, q_out_b_));
        int c = c0_, t = frames, li = 0;
        for (int s = 0; s < kStages; ++s) {
            Stage &st = stages_[size_t(s)];
            const int p = kPatch[s];
            mark_begin(KD_PATCH);
            k_patch<<<blocks_for(size_t(rows) * size_t(c) / 2), 256, 0, stream_>>>(xa_, size_t(rows), c, p, p0_, err_);
            CK(cudaGetLastError());
            mark_end();
            rows *= p;
            t *= p;
            c /= p;
            gemm(st.in, p0_, rows, EPI_PLAIN, out(y_));
            for (auto &l : st.layers) layer(l, md, n, rows, t, kContext[s], li++, md.offset + s * n);
            mark_begin(KD_SPLIT);
            k_split_rows<<<blocks_for(size_t(rows) * kDModel / 2), 256, 0, stream_>>>(y_, size_t(rows) * kDModel, p0_,
                                                                                        err_);
            CK(cudaGetLastError());
            mark_end();
            float *dst = s + 1 < kStages ? xa_ : pcm;  // the final patch of 240 is the identity
            gemm(st.out, p0_, rows, EPI_PLAIN, out(dst));
            c = st.out.rows;
        }
    }

    // decoder.cpp:116-196 run_layer_stream, on y_ [rows][256] in place
    void layer(Layer &l, const Meta &md, int n, int rows, int t, int window, int li, const int *offset) {
        const int lnb = (rows + 7) / 8;
        mark_begin(KD_LAYERNORM);
        k_layernorm256<<<lnb, 256, 0, stream_>>>(y_, rows, l.n1w, l.n1b, p0_, err_);
        mark_end();
        Epi qkv;
        qkv.q16 = q16_;
        qkv.kv16 = kv16_;
        qkv.offset = offset;
        qkv.t_per_stream = t;
        gemm(l.attn, p0_, rows, EPI_QKV, qkv);
        const dim3 ag((t + kQT - 1) / kQT, kHeads, n);
        mark_begin(KD_ATTN);
        k_window_attn<<<ag, 128, kAttnSmem, stream_>>>(q16_, kv16_, t, l.ring, window, li, md, n, p1_);
        mark_end();
        const size_t items = size_t(n) * size_t(std::min(t, window)) * 128;
        mark_begin(KD_RING);
        k_ring_append<<<int(std::min<size_t>((items + 255) / 256, 148 * 8)), 256, 0, stream_>>>(
            kv16_, t, n, l.ring, window, li, md);
        CK(cudaGetLastError());
        mark_end();
        gemm(l.proj, p1_, rows, EPI_SCALED_ADD, out(y_, l.ls1));
        mark_begin(KD_LAYERNORM);
        k_layernorm256<<<lnb, 256, 0, stream_>>>(y_, rows, l.n2w, l.n2b, p0_, err_);
        mark_end();
        Epi gelu;
        gelu.out = p1_;
        gemm(l.f1, p0_, rows, EPI_GELU, gelu);
        gemm(l.f2, p1_, rows, EPI_SCALED_ADD, out(y_, l.ls2));
    }

    void load(const std::string &path) {
        std::ifstream f(path, std::ios::binary | std::ios::ate);
        if (!f) throw std::runtime_error("cannot open decoder weights: " + path);
        const std::streamsize size = f.tellg();
        if (size < 16) throw std::runtime_error("short file: " + path);
        std::vector<uint8_t> file(static_cast<size_t>(size));
        f.seekg(0);
        if (!f.read(reinterpret_cast<char *>(file.data()), size)) throw std::runtime_error("short read: " + path);
        if (std::memcmp(file.data(), "MOSW", 4) != 0) throw std::runtime_error("bad magic (not a .moss file)");
        uint32_t version = 0, n = 0;
        std::memcpy(&version, file.data() + 4, 4);
        std::memcpy(&n, file.data() + 8, 4);
        if (version != 1) throw std::runtime_error("unsupported .moss version");
        if (16 + size_t(n) * 80 > file.size()) throw std::runtime_error("tensor table out of bounds");
        struct Entry {
            uint8_t dtype;
            int rows, cols;
            uint64_t off, nbytes;
        };
        std::unordered_map<std::string, Entry> ents;
        for (uint32_t i = 0; i < n; ++i) {  // the .moss table (weights.cpp:27-126)
            const uint8_t *b = file.data() + 16 + size_t(i) * 80;
            std::string name(reinterpret_cast<const char *>(b), strnlen(reinterpret_cast<const char *>(b), 48));
            Entry e{};
            e.dtype = b[48];
            uint32_t dims[3];
            std::memcpy(dims, b + 52, 12);
            std::memcpy(&e.off, b + 64, 8);
            std::memcpy(&e.nbytes, b + 72, 8);
            if (e.off > file.size() || e.nbytes > file.size() - e.off)
                throw std::runtime_error("tensor out of bounds: " + name);
            e.rows = int(dims[0]);
            e.cols = int(dims[1]);
            ents[name] = e;
        }
        auto find = [&](const std::string &name) -> const Entry & {
            auto it = ents.find(name);
            if (it == ents.end()) throw std::runtime_error("missing tensor: " + name);
            return it->second;
        };
        auto mat = [&](const std::string &name) {  // f16 matrix [rows][cols]
            const Entry &e = find(name);
            const size_t cnt = size_t(e.rows) * size_t(e.cols);
            if (e.cols % 8 || e.rows % 8)
                throw std::runtime_error("matrix " + name + " needs row and column counts that are multiples of 8");
            if (e.dtype != 0 || e.nbytes != cnt * 2) throw std::runtime_error("matrix is not f16: " + name);
            Mat m;
            m.rows = e.rows;
            m.cols = e.cols;
            m.w = alloc<__half>(cnt);
            CK(cudaMemcpy(m.w, file.data() + e.off, cnt * 2, cudaMemcpyHostToDevice));
            return m;
        };
        auto f32 = [&](const std::string &name, size_t count) {
            const Entry &e = find(name);
            if (e.dtype != 3 || e.nbytes != count * 4)
                throw std::runtime_error("tensor is not f32[" + std::to_string(count) + "]: " + name);
            float *d = alloc<float>(count);
            CK(cudaMemcpy(d, file.data() + e.off, count * 4, cudaMemcpyHostToDevice));
            return d;
        };
        q_out_ = mat("q.out.w");
        if (q_out_.cols != kZ) throw std::runtime_error("q.out.w must have 512 columns");
        c0_ = q_out_.rows;
        q_out_b_ = f32("q.out.b", size_t(c0_));
        std::vector<const float *> cb(kNCb), ow(kNCb), ob(kNCb);
        for (int i = 0; i < kNCb; ++i) {
            const std::string p = "q" + std::to_string(i) + ".";
            cb[size_t(i)] = f32(p + "cb", size_t(kCbSize) * kCbDim);
            ow[size_t(i)] = f32(p + "out.w", size_t(kZ) * kCbDim);
            ob[size_t(i)] = f32(p + "out.b", size_t(kZ));
        }
        d_cb_ = alloc<const float *>(kNCb);
        d_ow_ = alloc<const float *>(kNCb);
        d_ob_ = alloc<const float *>(kNCb);
        CK(cudaMemcpy(d_cb_, cb.data(), sizeof(float *) * kNCb, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(d_ow_, ow.data(), sizeof(float *) * kNCb, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(d_ob_, ob.data(), sizeof(float *) * kNCb, cudaMemcpyHostToDevice));
        int c = c0_;
        stages_.resize(kStages);
        const size_t nslots = slots_.size();
        for (int s = 0; s < kStages; ++s) {
            const std::string p = "d" + std::to_string(kStageIds[s]) + ".";
            Stage &st = stages_[size_t(s)];
            st.in = mat(p + "in.w");
            st.out = mat(p + "out.w");
            if (c % kPatch[s] || st.in.cols != c / kPatch[s] || st.in.rows != kDModel || st.out.cols != kDModel)
                throw std::runtime_error("stage " + p + " shapes do not chain");
            st.layers.resize(size_t(kLayerCount[s]));
            for (int k = 0; k < kLayerCount[s]; ++k) {
                const std::string lp = p + "l" + std::to_string(k) + ".";
                Layer &L = st.layers[size_t(k)];
                L.attn = mat(lp + "attn.w");
                L.proj = mat(lp + "proj.w");
                L.f1 = mat(lp + "f1.w");
                L.f2 = mat(lp + "f2.w");
                if (L.attn.rows != 3 * kDModel || L.attn.cols != kDModel || L.proj.rows != kDModel ||
                    L.proj.cols != kDModel || L.f1.cols != kDModel || L.f2.rows != kDModel || L.f2.cols != L.f1.rows)
                    throw std::runtime_error("layer " + lp + " has unexpected shapes");
                L.n1w = f32(lp + "n1.w", kDModel);
                L.n1b = f32(lp + "n1.b", kDModel);
                L.n2w = f32(lp + "n2.w", kDModel);
                L.n2b = f32(lp + "n2.b", kDModel);
                L.ls1 = f32(lp + "ls1", kDModel);
                L.ls2 = f32(lp + "ls2", kDModel);
                L.ring = alloc<__half>(nslots * size_t(kContext[s]) * 4 * kDModel);
            }
            c = st.out.rows;
        }
        if (c != kFinalPatch) throw std::runtime_error("the last stage must output 240 channels (the final patch)");
    }

    int device_ = 0, max_streams_ = 0, max_frames_ = 0, c0_ = 0;
    cudaStream_t stream_ = nullptr;  // the legacy default stream unless set
    std::vector<void *> owned_;
    size_t allocated_ = 0;
    std::vector<SlotState> slots_;
    Mat q_out_;
    float *q_out_b_ = nullptr;
    const float **d_cb_ = nullptr, **d_ow_ = nullptr, **d_ob_ = nullptr;
    std::vector<Stage> stages_;
    Planes p0_, p1_;
    float *xa_ = nullptr, *y_ = nullptr,
          *pcm_ = nullptr;
    __half *q16_ = nullptr, *kv16_ = nullptr;
    int *codes_ = nullptr, *meta_d_ = nullptr, *err_ = nullptr;
    bool profile_ = false;
    std::vector<int> marks_;            // kernel class of each bracketed launch
    std::vector<cudaEvent_t> events_;   // two per bracketed launch, reused
};

}  // namespace codec
}  // namespace mossgpu

struct mossgpu_codec {
    std::unique_ptr<mossgpu::codec::Codec> c;
    std::string error;
};

namespace {

template <class F>
int codec_guarded(mossgpu_codec *h, F &&f) {
    if (!h || !h->c) return 1;
    try {
        int d = -1;
        if (cudaGetDevice(&d) != cudaSuccess || d != h->c->device()) {
            const cudaError_t rc = cudaSetDevice(h->c->device());
            if (rc != cudaSuccess) throw std::runtime_error(std::string("cudaSetDevice: ") + cudaGetErrorString(rc));
        }
        f(*h->c);
        h->error.clear();
        return 0;
    } catch (const std::exception &ex) {
        h->error = ex.what();
        return 1;
    }
}

}  // namespace

extern "C" {

mossgpu_codec *mossgpu_codec_create(const char *decoder_path, int device_id, int max_streams, int max_batch_frames,
                                    char *err, int errlen) {
    try {
        if (!decoder_path) throw std::runtime_error("decoder_path is NULL");
        auto h = std::make_unique<mossgpu_codec>();
        h->c = std::make_unique<mossgpu::codec::Codec>(decoder_path, device_id, max_streams, max_batch_frames);
        return h.release();
    } catch (const std::exception &ex) {
        if (err && errlen > 0) {
            std::strncpy(err, ex.what(), size_t(errlen) - 1);
            err[errlen - 1] = 0;
        }
        return nullptr;
    }
}

void mossgpu_codec_destroy(mossgpu_codec *h) { delete h; }

const char *mossgpu_codec_last_error(mossgpu_codec *h) { return h ? h->error.c_str() : "null codec handle"; }

int mossgpu_codec_samples_per_frame(mossgpu_codec *h) { return h && h->c ? h->c->samples_per_frame() : 0; }

int mossgpu_codec_launches_per_call(mossgpu_codec *h) { return h && h->c ? h->c->launches_per_call() : 0; }

size_t mossgpu_codec_device_bytes(mossgpu_codec *h) { return h && h->c ? h->c->device_bytes() : 0; }

int mossgpu_codec_profile(mossgpu_codec *h, int enable) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) { c.set_profile(enable != 0); });
}

int mossgpu_codec_profile_read(mossgpu_codec *h, float *total_ms, int *launches, int max_kinds, int *n_kinds) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        using namespace mossgpu::codec;
        if (!total_ms || !launches || !n_kinds || max_kinds < KD_COUNT)
            throw std::runtime_error("profile_read needs arrays of at least " + std::to_string(KD_COUNT) + " kinds");
        c.profile_read(total_ms, launches);
        *n_kinds = KD_COUNT;
    });
}

const char *mossgpu_codec_kernel_name(int kind) {
    using namespace mossgpu::codec;
    return kind >= 0 && kind < KD_COUNT ? kKindNames[kind] : "";
}

int mossgpu_codec_status(mossgpu_codec *h, int *code) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        if (!code) throw std::runtime_error("code is NULL");
        *code = c.status();
    });
}

int mossgpu_codec_set_cuda_stream(mossgpu_codec *h, void *cuda_stream) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) { c.set_stream(static_cast<cudaStream_t>(cuda_stream)); });
}

int mossgpu_codec_open(mossgpu_codec *h, int *stream_id) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        if (!stream_id) throw std::runtime_error("stream_id is NULL");
        *stream_id = c.open();
    });
}

int mossgpu_codec_close(mossgpu_codec *h, int stream_id) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) { c.close(stream_id); });
}

int mossgpu_codec_reset(mossgpu_codec *h, int stream_id) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) { c.reset(stream_id); });
}

int mossgpu_codec_decode_chunk(mossgpu_codec *h, int stream_id, const int32_t *codes, int frames, float *out,
                               size_t out_cap, int *out_n) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        if (!out_n || (frames > 0 && (!codes || !out))) throw std::runtime_error("codes, out and out_n must not be NULL");
        if (frames < 0) throw std::runtime_error("frames must not be negative");
        c.decode_host(&stream_id, 1, codes, frames, out, out_cap);
        *out_n = frames * c.samples_per_frame();
    });
}

int mossgpu_codec_decode_batch(mossgpu_codec *h, const int32_t *stream_ids, int n, const int32_t *codes, int frames,
                               float *out, size_t out_cap) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        if (n < 0 || frames < 0) throw std::runtime_error("n and frames must not be negative");
        if (n > 0 && frames > 0 && (!stream_ids || !codes || !out))
            throw std::runtime_error("stream_ids, codes and out must not be NULL");
        c.decode_host(stream_ids, n, codes, frames, out, out_cap);
    });
}

int mossgpu_codec_decode_batch_device(mossgpu_codec *h, const int32_t *stream_ids, int n, const int32_t *codes_dev,
                                      int frames, float *out_dev) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        if (n < 0 || frames < 0) throw std::runtime_error("n and frames must not be negative");
        if (n > 0 && frames > 0 && (!stream_ids || !codes_dev || !out_dev))
            throw std::runtime_error("stream_ids, codes_dev and out_dev must not be NULL");
        c.decode_device(stream_ids, n, codes_dev, frames, out_dev);
    });
}

int mossgpu_codec_decode(mossgpu_codec *h, const int32_t *codes, int frames, float *out, size_t out_cap, int *out_n) {
    return codec_guarded(h, [&](mossgpu::codec::Codec &c) {
        if (!out_n || (frames > 0 && (!codes || !out))) throw std::runtime_error("codes, out and out_n must not be NULL");
        if (frames < 0) throw std::runtime_error("frames must not be negative");
        c.decode_whole(codes, frames, out, out_cap);
        *out_n = frames * c.samples_per_frame();
    });
}

}  // extern "C"
