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
// through each GEMM together, attention is tiled per (stream, head, 32 rows).  Activations are
// fp32 [rows][channels] with stream b's rows contiguous; matrices stay fp16 as in the file and
// are widened in shared memory, products accumulated in fp32 like the reference's gemm_par on
// f16 matrices.  The K/V rings are fp32 [slot][context][256], slot = stream id.
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

// y[t][r] = sum_k W[r][k] x[t][k] (W fp16 [R][K], x fp32 [T][K]), then the epilogue:
// EPI_PLAIN y = acc (+ vec[r] when vec is given), EPI_GELU y = gelu(acc),
// EPI_SCALED_ADD y = y + vec[r] * acc (the layer-scale residual, decoder.cpp:173-177).
enum { EPI_PLAIN = 0, EPI_GELU = 1, EPI_SCALED_ADD = 2 };
constexpr int kBM = 128, kBN = 64, kBK = 16, kGemmThreads = 256;

__device__ __forceinline__ float gelu_erf(float v) {  // audio_layer.cpp:46
    return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
}

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads) k_gemm_f16w(const __half *__restrict__ W, const float *__restrict__ x,
                                                            int T, int R, int K, const float *__restrict__ vec,
                                                            float *__restrict__ y) {
    __shared__ __align__(16) float xs[2][kBK][kBM + 4];
    __shared__ __align__(16) float ws[2][kBK][kBN + 4];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.y * kBM, r0 = blockIdx.x * kBN;
    const int tx = tid & 15, ty = tid >> 4;  // outputs r0 + 4 tx .. +3, rows t0 + 8 ty .. +7
    // loaders: x tile 128 x 16 floats = 512 float4 (2 per thread); W tile 64 x 16 halves = 128 x 8
    const int xm = tid >> 2, xk = (tid & 3) * 4;  // rows xm and xm + 64, k xk..xk+3
    const int wr = tid >> 1, wk = (tid & 1) * 8;  // threads 0..127: row wr, k wk..wk+7
    float4 px[2];
    uint4 pw = make_uint4(0, 0, 0, 0);
    auto load = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int t = t0 + xm + 64 * j, k = k0 + xk;
            px[j] = (t < T && k < K) ? *reinterpret_cast<const float4 *>(x + (size_t)t * K + k)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (tid < 128) {
            const int r = r0 + wr, k = k0 + wk;
            pw = (r < R && k < K) ? *reinterpret_cast<const uint4 *>(W + (size_t)r * K + k) : make_uint4(0, 0, 0, 0);
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            xs[buf][xk + 0][xm + 64 * j] = px[j].x;
            xs[buf][xk + 1][xm + 64 * j] = px[j].y;
            xs[buf][xk + 2][xm + 64 * j] = px[j].z;
            xs[buf][xk + 3][xm + 64 * j] = px[j].w;
        }
        if (tid < 128) {
            const __half2 *h = reinterpret_cast<const __half2 *>(&pw);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(h[j]);
                ws[buf][wk + 2 * j][wr] = f.x;
                ws[buf][wk + 2 * j + 1][wr] = f.y;
            }
        }
    };
    float acc[8][4];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
    load(0);
    store(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += kBK) {
        const bool more = k0 + kBK < K;
        if (more) load(k0 + kBK);
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            const float4 xa = *reinterpret_cast<const float4 *>(&xs[buf][kk][ty * 8]);
            const float4 xb = *reinterpret_cast<const float4 *>(&xs[buf][kk][ty * 8 + 4]);
            const float4 wv = *reinterpret_cast<const float4 *>(&ws[buf][kk][tx * 4]);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            const float wf[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(xv[a], wf[b], acc[a][b]);
        }
        if (more) {
            store(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int t = t0 + ty * 8 + a;
        if (t >= T) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int r = r0 + tx * 4 + b;
            if (r >= R) continue;
            const float v = acc[a][b];
            float *dst = y + (size_t)t * R + r;
            if (EPI == EPI_PLAIN)
                *dst = vec ? v + vec[r] : v;
            else if (EPI == EPI_GELU)
                *dst = gelu_erf(v);
            else
                *dst = *dst + vec[r] * v;
        }
    }
}

// z[row][r] = sum_i (b_i[r] + sum_k W_i[r][k] e_i[k]), e_i = codebook i's row for the row's code
// (decoder.cpp:229-244: the same per-element order).  codes [n][16][frames], row = b frames + f;
// a code outside [0, 1024) is clamped (the host entry points reject such codes first).
__global__ void k_front(const int *__restrict__ codes, int frames, const float *const *__restrict__ cb,
                        const float *const *__restrict__ ow, const float *const *__restrict__ ob,
                        float *__restrict__ z) {
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
    for (int r = threadIdx.x; r < kZ; r += blockDim.x) {
        float zi = 0.f;
        for (int i = 0; i < kNCb; ++i) {
            const float *w = ow[i] + (size_t)r * kCbDim;
            float acc = ob[i][r];
#pragma unroll
            for (int k = 0; k < kCbDim; ++k) acc += w[k] * emb[i][k];
            zi += acc;
        }
        z[(size_t)row * kZ + r] = zi;
    }
}

// x [t][c] -> out [t p][c / p]: out[t p + j][ci] = x[t][ci p + j] (decoder.cpp:73-87)
__global__ void k_patch(const float *__restrict__ x, size_t T, int c, int p, float *__restrict__ out) {
    const size_t n = T * c;
    const int d = c / p;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / d;
        const int ci = (int)(i - row * d);
        const size_t t = row / p;
        const int j = (int)(row - t * p);
        out[i] = x[t * c + (size_t)ci * p + j];
    }
}

// LayerNorm of 256-wide rows, one warp per row (audio_layer.cpp:17-29)
__global__ void k_layernorm256(const float *__restrict__ x, int T, const float *__restrict__ w,
                               const float *__restrict__ bias, float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const float *row = x + (size_t)t * kDModel;
    float v[8], s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[j] = row[lane + 32 * j];
        s += v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)kDModel;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float d = v[j] - mean;
        q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = 1.0f / sqrtf(q / (float)kDModel + 1e-5f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int k = lane + 32 * j;
        out[(size_t)t * kDModel + k] = (v[j] - mean) * inv * w[k] + bias[k];
    }
}

// Interleaved RoPE on q and k of every row, position = the stream's stage offset + the row's
// index in its chunk; frequency exp(-ln(10000) 2 i / 64) in fp32 (audio_layer.cpp:31-44).
// One row per block: thread = (q or k head hq, pair i).
__global__ void k_rope(float *__restrict__ qkv, int T, int t_per_stream, const int *__restrict__ offset) {
    const int row = blockIdx.x;
    if (row >= T) return;
    const int b = row / t_per_stream;
    const int pos = offset[b] + (row - b * t_per_stream);
    const int i = threadIdx.x & 31;   // pair within a head
    const int hq = threadIdx.x >> 5;  // 0..7: q heads 0..3, then k heads 0..3
    const float freq = expf(-logf(10000.0f) * 2.0f * (float)i / (float)kHeadDim);
    const float ang = (float)pos * freq;
    const float c = cosf(ang), s = sinf(ang);
    float *base = qkv + (size_t)row * 3 * kDModel + (hq >> 2) * kDModel + (hq & 3) * kHeadDim;
    const float x0 = base[2 * i], x1 = base[2 * i + 1];
    base[2 * i] = x0 * c - x1 * s;
    base[2 * i + 1] = x0 * s + x1 * c;
}

// Windowed causal attention of a chunk (attn_scalar.cpp:165-203 attention_window_scalar):
// chunk row i of a stream sees keys u in [max(0, i + n - window + 1), i + n], where keys
// 0..n-1 are the stream's ring (physical slot (start + u) % window) and keys n.. the chunk's
// own rows.  Block = (32 rows, head, stream), 256 threads; keys in tiles of 64 staged in
// shared memory, softmax online across tiles.  Thread (g = tid / 16, j = tid % 16): scores of
// rows 2g, 2g + 1 against keys 4j..4j+3 of a tile, then output dims 4j..4j+3 of those rows.
constexpr int kAQ = 32, kAK = 64;
constexpr size_t kAttnSmem = sizeof(float) * (kHeadDim * kAQ + kHeadDim * kAK + kAK * (kHeadDim + 4) +
                                              kAQ * (kAK + 4));  // 50,688 bytes
__global__ void __launch_bounds__(256) k_window_attn(const float *__restrict__ qkv, int t,
                                                     const float *__restrict__ ring_k,
                                                     const float *__restrict__ ring_v, int window, int layer,
                                                     Meta meta, int n_streams, float *__restrict__ out) {
    extern __shared__ __align__(16) float attn_smem[];
    auto qs = reinterpret_cast<float (*)[kAQ]>(attn_smem);                  // [64][32]
    auto ks = reinterpret_cast<float (*)[kAK]>(attn_smem + kHeadDim * kAQ);  // [64][64]
    auto vs = reinterpret_cast<float (*)[kHeadDim + 4]>(attn_smem + kHeadDim * kAQ + kHeadDim * kAK);  // [64][68]
    auto ps = reinterpret_cast<float (*)[kAK + 4]>(attn_smem + kHeadDim * kAQ + kHeadDim * kAK + kAK * (kHeadDim + 4));
    const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * kAQ;
    const int tid = threadIdx.x, g = tid >> 4, j = tid & 15;
    const int n = meta.rcount[layer * n_streams + b], start = meta.rstart[layer * n_streams + b];
    const size_t slot = (size_t)meta.sid[b];
    const float *rk = ring_k + slot * window * kDModel + h * kHeadDim;
    const float *rv = ring_v + slot * window * kDModel + h * kHeadDim;
    const float *base = qkv + (size_t)b * t * 3 * kDModel;
    const int nq = min(kAQ, t - q0);
    for (int idx = tid; idx < kAQ * 16; idx += 256) {
        const int q = idx & (kAQ - 1), d4 = idx / kAQ;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q < nq) v = *reinterpret_cast<const float4 *>(base + (size_t)(q0 + q) * 3 * kDModel + h * kHeadDim + d4 * 4);
        qs[d4 * 4 + 0][q] = v.x;
        qs[d4 * 4 + 1][q] = v.y;
        qs[d4 * 4 + 2][q] = v.z;
        qs[d4 * 4 + 3][q] = v.w;
    }
    const int ulo = max(0, q0 + n - window + 1), uhi = q0 + nq - 1 + n;
    const float scale = 1.0f / sqrtf((float)kHeadDim);
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, o[2][4] = {};
    for (int u0 = ulo; u0 <= uhi; u0 += kAK) {
        __syncthreads();  // the Q stores, and the previous tile's K and V reads, are done
        for (int idx = tid; idx < kAK * 16; idx += 256) {
            const int kk = idx & (kAK - 1), d4 = idx / kAK;
            const int u = u0 + kk;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (u <= uhi) {
                const float *kp, *vp;
                if (u < n) {
                    const size_t at = (size_t)((start + u) % window) * kDModel + d4 * 4;
                    kp = rk + at;
                    vp = rv + at;
                } else {
                    kp = base + (size_t)(u - n) * 3 * kDModel + kDModel + h * kHeadDim + d4 * 4;
                    vp = kp + kDModel;
                }
                kv = *reinterpret_cast<const float4 *>(kp);
                vv = *reinterpret_cast<const float4 *>(vp);
            }
            ks[d4 * 4 + 0][kk] = kv.x;
            ks[d4 * 4 + 1][kk] = kv.y;
            ks[d4 * 4 + 2][kk] = kv.z;
            ks[d4 * 4 + 3][kk] = kv.w;
            *reinterpret_cast<float4 *>(&vs[kk][d4 * 4]) = vv;
        }
        __syncthreads();
        float s[2][4] = {};
#pragma unroll 16
        for (int d = 0; d < kHeadDim; ++d) {
            const float2 qv = *reinterpret_cast<const float2 *>(&qs[d][2 * g]);
            const float4 kv = *reinterpret_cast<const float4 *>(&ks[d][4 * j]);
            s[0][0] = fmaf(qv.x, kv.x, s[0][0]);
            s[0][1] = fmaf(qv.x, kv.y, s[0][1]);
            s[0][2] = fmaf(qv.x, kv.z, s[0][2]);
            s[0][3] = fmaf(qv.x, kv.w, s[0][3]);
            s[1][0] = fmaf(qv.y, kv.x, s[1][0]);
            s[1][1] = fmaf(qv.y, kv.y, s[1][1]);
            s[1][2] = fmaf(qv.y, kv.z, s[1][2]);
            s[1][3] = fmaf(qv.y, kv.w, s[1][3]);
        }
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            const int i = q0 + 2 * g + a;  // chunk row
            const bool row_ok = 2 * g + a < nq;
            const int lo = i + n - window + 1, hi = i + n;
            float tmax = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int u = u0 + 4 * j + c;
                s[a][c] = (row_ok && u >= lo && u <= hi) ? s[a][c] * scale : -INFINITY;
                tmax = fmaxf(tmax, s[a][c]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float mnew = fmaxf(m[a], tmax);
            float alpha = 1.f, rs = 0.f;
            if (mnew != -INFINITY) {
                alpha = expf(m[a] - mnew);  // 0 while m is still -inf
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    s[a][c] = expf(s[a][c] - mnew);
                    rs += s[a][c];
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) s[a][c] = 0.f;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l[a] = l[a] * alpha + rs;
            m[a] = mnew;
#pragma unroll
            for (int c = 0; c < 4; ++c) o[a][c] *= alpha;
            *reinterpret_cast<float4 *>(&ps[2 * g + a][4 * j]) = make_float4(s[a][0], s[a][1], s[a][2], s[a][3]);
        }
        __syncwarp();  // rows 2g, 2g+1 are written and read by the same 16 lanes
#pragma unroll 8
        for (int kk = 0; kk < kAK; ++kk) {
            const float p0 = ps[2 * g][kk], p1 = ps[2 * g + 1][kk];
            const float4 vv = *reinterpret_cast<const float4 *>(&vs[kk][4 * j]);
            o[0][0] = fmaf(p0, vv.x, o[0][0]);
            o[0][1] = fmaf(p0, vv.y, o[0][1]);
            o[0][2] = fmaf(p0, vv.z, o[0][2]);
            o[0][3] = fmaf(p0, vv.w, o[0][3]);
            o[1][0] = fmaf(p1, vv.x, o[1][0]);
            o[1][1] = fmaf(p1, vv.y, o[1][1]);
            o[1][2] = fmaf(p1, vv.z, o[1][2]);
            o[1][3] = fmaf(p1, vv.w, o[1][3]);
        }
        __syncwarp();
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        if (2 * g + a >= nq) continue;
        const float inv = 1.0f / l[a];
        float *dst = out + ((size_t)b * t + q0 + 2 * g + a) * kDModel + h * kHeadDim + 4 * j;
        *reinterpret_cast<float4 *>(dst) = make_float4(o[a][0] * inv, o[a][1] * inv, o[a][2] * inv, o[a][3] * inv);
    }
}

// Append each stream's chunk K and V rows to its ring (decoder.cpp:150-169): chunk row i goes
// to slot (start + n + i) % window; only the last `window` rows of a chunk can survive, so only
// they are written.
__global__ void k_ring_append(const float *__restrict__ qkv, int t, int n_streams, float *__restrict__ ring_k,
                              float *__restrict__ ring_v, int window, int layer, Meta meta) {
    const int first = max(0, t - window);
    const int rows = t - first;
    const size_t total = (size_t)n_streams * rows * (kDModel / 4);
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const int d4 = (int)(idx % (kDModel / 4));
        const size_t rr = idx / (kDModel / 4);
        const int b = (int)(rr / rows), i = first + (int)(rr % rows);
        const int n = meta.rcount[layer * n_streams + b], start = meta.rstart[layer * n_streams + b];
        const size_t slot = (size_t)meta.sid[b] * window + (size_t)((start + n + i) % window);
        const float *src = qkv + ((size_t)b * t + i) * 3 * kDModel + d4 * 4;
        reinterpret_cast<float4 *>(ring_k + slot * kDModel)[d4] = *reinterpret_cast<const float4 *>(src + kDModel);
        reinterpret_cast<float4 *>(ring_v + slot * kDModel)[d4] = *reinterpret_cast<const float4 *>(src + 2 * kDModel);
    }
}

// ------------------------------------------------------------------------------- host

// kernel classes of the optional per-launch profile (mossgpu_codec_profile)
enum Kind { KD_FRONT = 0, KD_GEMM, KD_PATCH, KD_LAYERNORM, KD_ROPE, KD_ATTN, KD_RING, KD_COUNT };
const char *const kKindNames[KD_COUNT] = {"k_front", "k_gemm_f16w", "k_patch", "k_layernorm256",
                                          "k_rope", "k_window_attn", "k_ring_append"};

struct Mat {
    __half *w = nullptr;
    int rows = 0, cols = 0;
};

struct Layer {
    Mat attn, proj, f1, f2;
    float *n1w, *n1b, *n2w, *n2b, *ls1, *ls2;
    float *ring_k = nullptr, *ring_v = nullptr;  // [slots][context][256]
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
        CK(cudaFuncSetAttribute(k_window_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem)));
        slots_.resize(size_t(max_streams) + 1);  // the last slot serves decode()
        load(path);
        // activation buffers, each sized for its widest use over the stages
        const size_t F = size_t(max_frames_);
        size_t x_elems = F * size_t(std::max(c0_, kZ)), y_elems = 0, qkv_elems = 0, ffn_elems = 0;
        size_t rows = F;
        for (int s = 0; s < kStages; ++s) {
            rows *= kPatch[s];
            x_elems = std::max(x_elems, rows * size_t(stages_[size_t(s)].out.rows));
            y_elems = std::max(y_elems, rows * kDModel);
            qkv_elems = std::max(qkv_elems, rows * 3 * kDModel);
            for (auto &l : stages_[size_t(s)].layers) ffn_elems = std::max(ffn_elems, rows * size_t(l.f1.rows));
        }
        xa_ = alloc<float>(x_elems);
        xb_ = alloc<float>(x_elems);
        y_ = alloc<float>(y_elems);
        ln_ = alloc<float>(std::max(y_elems, F * kZ));
        att_ = alloc<float>(y_elems);
        qkv_ = alloc<float>(qkv_elems);
        ffn_ = alloc<float>(ffn_elems);
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
        CK(cudaStreamSynchronize(stream_));
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
        for (auto &s : stages_) l += 3 + 9 * int(s.layers.size());
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

    void gemm(const Mat &m, const float *x, int T, float *y, int epi, const float *vec) {
        const dim3 grid((m.rows + kBN - 1) / kBN, (T + kBM - 1) / kBM);
        mark_begin(KD_GEMM);
        if (epi == EPI_PLAIN)
            k_gemm_f16w<EPI_PLAIN><<<grid, kGemmThreads, 0, stream_>>>(m.w, x, T, m.rows, m.cols, vec, y);
        else if (epi == EPI_GELU)
            k_gemm_f16w<EPI_GELU><<<grid, kGemmThreads, 0, stream_>>>(m.w, x, T, m.rows, m.cols, vec, y);
        else
            k_gemm_f16w<EPI_SCALED_ADD><<<grid, kGemmThreads, 0, stream_>>>(m.w, x, T, m.rows, m.cols, vec, y);
        CK(cudaGetLastError());
        mark_end();
    }

    void run(const Meta &md, int n, const int *codes, int frames, float *pcm) {
        int rows = n * frames;  // all streams' rows of the current stage
        mark_begin(KD_FRONT);
        k_front<<<rows, 256, 0, stream_>>>(codes, frames, d_cb_, d_ow_, d_ob_, ln_);
        CK(cudaGetLastError());
        mark_end();
        gemm(q_out_, ln_, rows, xa_, EPI_PLAIN, q_out_b_);
        int c = c0_, t = frames, li = 0;
        for (int s = 0; s < kStages; ++s) {
            Stage &st = stages_[size_t(s)];
            const int p = kPatch[s];
            const size_t nel = size_t(rows) * size_t(c);
            const int pblocks = int(std::min<size_t>((nel + 255) / 256, 148 * 16));
            mark_begin(KD_PATCH);
            k_patch<<<pblocks, 256, 0, stream_>>>(xa_, size_t(rows), c, p, xb_);
            CK(cudaGetLastError());
            mark_end();
            rows *= p;
            t *= p;
            c /= p;
            gemm(st.in, xb_, rows, y_, EPI_PLAIN, nullptr);
            for (auto &l : st.layers) layer(l, md, n, rows, t, kContext[s], li++, md.offset + s * n);
            float *dst = s + 1 < kStages ? xa_ : pcm;  // the final patch of 240 is the identity
            gemm(st.out, y_, rows, dst, EPI_PLAIN, nullptr);
            c = st.out.rows;
        }
    }

    // decoder.cpp:116-196 run_layer_stream, on y_ [rows][256] in place
    void layer(Layer &l, const Meta &md, int n, int rows, int t, int window, int li, const int *offset) {
        const int lnb = (rows + 7) / 8;
        mark_begin(KD_LAYERNORM);
        k_layernorm256<<<lnb, 256, 0, stream_>>>(y_, rows, l.n1w, l.n1b, ln_);
        mark_end();
        gemm(l.attn, ln_, rows, qkv_, EPI_PLAIN, nullptr);
        mark_begin(KD_ROPE);
        k_rope<<<rows, 256, 0, stream_>>>(qkv_, rows, t, offset);
        mark_end();
        const dim3 ag((t + kAQ - 1) / kAQ, kHeads, n);
        mark_begin(KD_ATTN);
        k_window_attn<<<ag, 256, kAttnSmem, stream_>>>(qkv_, t, l.ring_k, l.ring_v, window, li, md, n, att_);
        mark_end();
        const size_t items = size_t(n) * size_t(std::min(t, window)) * (kDModel / 4);
        mark_begin(KD_RING);
        k_ring_append<<<int(std::min<size_t>((items + 255) / 256, 148 * 8)), 256, 0, stream_>>>(
            qkv_, t, n, l.ring_k, l.ring_v, window, li, md);
        CK(cudaGetLastError());
        mark_end();
        gemm(l.proj, att_, rows, y_, EPI_SCALED_ADD, l.ls1);
        mark_begin(KD_LAYERNORM);
        k_layernorm256<<<lnb, 256, 0, stream_>>>(y_, rows, l.n2w, l.n2b, ln_);
        mark_end();
        gemm(l.f1, ln_, rows, ffn_, EPI_GELU, nullptr);
        gemm(l.f2, ffn_, rows, y_, EPI_SCALED_ADD, l.ls2);
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
            if (e.cols % 8) throw std::runtime_error("matrix " + name + " needs a column count that is a multiple of 8");
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
                const size_t ring = nslots * size_t(kContext[s]) * kDModel;
                L.ring_k = alloc<float>(ring);
                L.ring_v = alloc<float>(ring);
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
    float *xa_ = nullptr, *xb_ = nullptr, *y_ = nullptr, *ln_ = nullptr, *qkv_ = nullptr, *att_ = nullptr,
          *ffn_ = nullptr, *pcm_ = nullptr;
    int *codes_ = nullptr, *meta_d_ = nullptr;
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
