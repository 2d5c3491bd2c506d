/*
 * moss_oracle.c -- CPU restatement of the MOSS-TTS-Nano per-frame LLM step.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA engine, never part of the product.
 * Each function keeps the reference's floating-point operation order; the AVX2 row dots
 * are restated lane by lane (8 fp32 lanes, fmaf for _mm256_fmadd_ps, the same horizontal
 * sum tree).  Build with -O2 -ffp-contract=off (oracle/Makefile) so that no a*b+c is fused
 * where the reference does not fuse it.  Citations are file:line in the reference
 * (litterbit/dsh-moss-tts).
 */
#include "moss_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 */

/* fp16.cpp:7-35 */
float or_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            exp = 127 - 15 + 1;
            while ((mant & 0x400u) == 0) {
                mant <<= 1;
                --exp;
            }
            mant &= 0x3FF;
            bits = sign | (exp << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

/* fp16.cpp:37-66 */
uint16_t or_float_to_half(float f) {
    uint32_t bits;
    memcpy(&bits, &f, sizeof(bits));
    const uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t exp = (int32_t)((bits >> 23) & 0xFF) - 127 + 15;
    uint32_t mant = bits & 0x7FFFFFu;
    if (((bits >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0));
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - exp;
        uint32_t half_mant = mant >> shift;
        if ((mant >> (shift - 1)) & 1u) ++half_mant;
        return (uint16_t)(sign | half_mant);
    }
    if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
    uint32_t half_mant = mant >> 13;
    if (mant & 0x1000u) ++half_mant;
    if (half_mant == 0x400u) {
        half_mant = 0;
        ++exp;
        if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | ((uint32_t)exp << 10) | half_mant);
}

void or_half_to_float_n(const uint16_t *h, int n, float *out) {
    for (int i = 0; i < n; ++i) out[i] = or_half_to_float(h[i]);
}

void or_float_to_half_n(const float *f, int n, uint16_t *out) {
    for (int i = 0; i < n; ++i) out[i] = or_float_to_half(f[i]);
}

/* ------------------------------------------------------------------ Q8_0_4X4 */

static inline float blk_scale(const uint8_t *blk, int k) {
    uint16_t dh;
    memcpy(&dh, blk + k * 2, 2);
    return or_half_to_float(dh);
}

/* quant.cpp:56-65: block b of a 4-row group = 136 B, [fp16 d0..d3][int8 q_k[32] at 8+32k] */
void or_dequant_row_q8x4(const uint8_t *group, int nb, int k, float *out) {
    for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = group + (size_t)b * 136;
        const float d = blk_scale(blk, k);
        const int8_t *qs = (const int8_t *)(blk + 8 + (size_t)k * 32);
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)qs[i];
    }
}

/* gemv_avx2.cpp:24-31: ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)) */
static inline float hsum8(const float *v) {
    float s[4];
    for (int i = 0; i < 4; ++i) s[i] = v[i] + v[i + 4];
    const float a = s[0] + s[2];
    const float c = s[1] + s[3];
    return a + c;
}

/* gemv_avx2.cpp:123-150 */
float or_row_dot_a16(const uint8_t *group, int nb, int k, const float *act) {
    float sum = 0.0f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = group + (size_t)b * 136;
        const float dw = blk_scale(blk, k);
        const int8_t *qs = (const int8_t *)(blk + 8 + (size_t)k * 32);
        const float *a = act + (size_t)b * 32;
        float acc[8];
        for (int j = 0; j < 8; ++j) acc[j] = (float)qs[j] * a[j];
        for (int s = 1; s < 4; ++s)
            for (int j = 0; j < 8; ++j) acc[j] = fmaf((float)qs[8 * s + j], a[8 * s + j], acc[j]);
        const float h = hsum8(acc);
        const float t = h * dw;
        sum = sum + t;
    }
    return sum;
}

/* quant.cpp:28-43 (scales kept in fp32, as quantize_activation uses them: quant.cpp:45-54) */
void or_quantize_act(const float *x, int n, int8_t *q, float *scales) {
    const int nb = n / 32;
    for (int b = 0; b < nb; ++b) {
        const float *src = x + b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float v = fabsf(src[i]);
            amax = (amax < v) ? v : amax; /* std::max(amax, v) */
        }
        const float d = amax / 127.0f;
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        scales[b] = d;
        for (int i = 0; i < 32; ++i) {
            int v = (int)lrintf(src[i] * id);
            v = v < -127 ? -127 : (v > 127 ? 127 : v);
            q[b * 32 + i] = (int8_t)v;
        }
    }
}

/* gemv_avx2.cpp:105-121: lane j of the int32 product = sum of bytes 4j..4j+3 */
float or_row_dot_a8(const uint8_t *group, int nb, int k, const int8_t *qa, const float *as) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = group + (size_t)b * 136;
        const float dw = blk_scale(blk, k);
        const int8_t *qs = (const int8_t *)(blk + 8 + (size_t)k * 32);
        const int8_t *a = qa + (size_t)b * 32;
        const float s = dw * as[b];
        for (int j = 0; j < 8; ++j) {
            int32_t p = 0;
            for (int i = 4 * j; i < 4 * j + 4; ++i) p += (int32_t)qs[i] * (int32_t)a[i];
            acc[j] = fmaf((float)p, s, acc[j]);
        }
    }
    return hsum8(acc);
}

/* gemv.cpp:245-274 -> gemv_avx2.cpp:173-191 (A16) or quantize_activation + row_dot (A8) */
void or_gemv(const uint8_t *w, int rows, int cols, const float *x, float *y, int a16) {
    const int nb = cols / 32;
    int8_t *qa = NULL;
    float *as = NULL;
    if (!a16) {
        qa = (int8_t *)malloc((size_t)cols);
        as = (float *)malloc(sizeof(float) * (size_t)nb);
        or_quantize_act(x, cols, qa, as);
    }
    for (int r = 0; r < rows; ++r) {
        const uint8_t *grp = w + (size_t)(r / 4) * nb * 136;
        y[r] = a16 ? or_row_dot_a16(grp, nb, r % 4, x) : or_row_dot_a8(grp, nb, r % 4, qa, as);
    }
    free(qa);
    free(as);
}

/* ------------------------------------------------------------------ small ops */

/* llm.cpp:159-171 */
void or_layernorm(const float *x, const float *w, const float *b, float *out) {
    float mean = 0.0f;
    for (int i = 0; i < OR_HIDDEN; ++i) mean += x[i];
    mean /= (float)OR_HIDDEN;
    float var = 0.0f;
    for (int i = 0; i < OR_HIDDEN; ++i) {
        const float d = x[i] - mean;
        var += d * d;
    }
    var /= (float)OR_HIDDEN;
    const float inv = 1.0f / sqrtf(var + 1e-5f);
    for (int i = 0; i < OR_HIDDEN; ++i) out[i] = (x[i] - mean) * inv * w[i] + b[i];
}

/* llm.cpp:22-25 */
static inline float gelu_new(float v) {
    const float k = 0.7978845608028654f;
    return 0.5f * v * (1.0f + tanhf(k * (v + 0.044715f * v * v * v)));
}

/* ------------------------------------------------------------------ sampler */

/* sampler.h:28-48 (xoshiro128**) */
void or_rng_seed(uint32_t *s, uint64_t v) {
    s[0] = (uint32_t)v;
    s[1] = (uint32_t)(v >> 32) ^ 0x9E3779B9u;
    s[2] = 0x243F6A88u;
    s[3] = 0xB7E15162u;
    for (int i = 0; i < 8; ++i) (void)or_rng_uniform(s);
}

static inline uint32_t rotl32(uint32_t x, int k) { return (x << k) | (x >> (32 - k)); }

static uint32_t rng_next(uint32_t *s) {
    const uint32_t result = rotl32(s[1] * 5, 7) * 9;
    const uint32_t t = s[1] << 9;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl32(s[3], 11);
    return result;
}

float or_rng_uniform(uint32_t *s) { return (float)(rng_next(s) >> 8) * (1.0f / 16777216.0f); }

static const float *g_sort_keys;
/* descending by value, then ascending by index (libstdc++'s partial_sort leaves equal
 * values in an unspecified order; ties never occur for the float logits tested) */
static int cmp_desc(const void *pa, const void *pb) {
    const int a = *(const int *)pa, b = *(const int *)pb;
    const float va = g_sort_keys[a], vb = g_sort_keys[b];
    if (va > vb) return -1;
    if (va < vb) return 1;
    return (a > b) - (a < b);
}

/* sampler.cpp:9-77 */
int or_sample_token(const float *logits, int n, const or_sample_params *p, const int *prev, int n_prev,
                    uint32_t *rng) {
    float *sc = (float *)malloc(sizeof(float) * (size_t)n);
    memcpy(sc, logits, sizeof(float) * (size_t)n);
    if (p->repetition_penalty != 1.0f && prev != NULL && n_prev > 0) {
        for (int i = 0; i < n_prev; ++i) {
            const int t = prev[i];
            if (t < 0 || t >= n) continue;
            const float v = sc[t];
            sc[t] = v < 0.0f ? v * p->repetition_penalty : v / p->repetition_penalty;
        }
    }
    if (p->greedy || p->top_k == 1) {
        int best = 0;
        for (int i = 1; i < n; ++i)
            if (sc[i] > sc[best]) best = i;
        free(sc);
        return best;
    }
    if (p->temperature > 0.0f && p->temperature != 1.0f) {
        const float inv = 1.0f / p->temperature;
        for (int i = 0; i < n; ++i) sc[i] *= inv;
    }
    int k = p->top_k > 0 ? (p->top_k < n ? p->top_k : n) : n;
    int *idx = (int *)malloc(sizeof(int) * (size_t)n);
    for (int i = 0; i < n; ++i) idx[i] = i;
    g_sort_keys = sc;
    qsort(idx, (size_t)n, sizeof(int), cmp_desc);
    int size = k;
    const float maxv = sc[idx[0]];
    float sum = 0.0f;
    for (int j = 0; j < size; ++j) {
        const int i = idx[j];
        sc[i] = expf(sc[i] - maxv);
        sum += sc[i];
    }
    if (p->top_p < 1.0f) {
        float cum = 0.0f;
        int keep = 0;
        for (; keep < size; ++keep) {
            cum += sc[idx[keep]] / sum;
            if (cum >= p->top_p) {
                ++keep;
                break;
            }
        }
        size = keep > 1 ? keep : 1;
        sum = 0.0f;
        for (int j = 0; j < size; ++j) sum += sc[idx[j]];
    }
    float r = or_rng_uniform(rng) * sum;
    int out = idx[size - 1];
    for (int j = 0; j < size; ++j) {
        r -= sc[idx[j]];
        if (r <= 0.0f) {
            out = idx[j];
            break;
        }
    }
    free(idx);
    free(sc);
    return out;
}

/* llm.cpp:30-35 */
static int end_reached(float l_slot, float l_end, const or_sample_params *p, uint32_t *rng) {
    if (p->end_greedy) return l_end > l_slot;
    double d = (double)l_end - (double)l_slot;
    d = d < -80.0 ? -80.0 : (d > 80.0 ? 80.0 : d);
    const float p_slot = (float)(1.0 / (1.0 + exp(d)));
    return or_rng_uniform(rng) >= p_slot;
}

/* ------------------------------------------------------------------ model */

typedef struct {
    const uint8_t *data; /* Q8_0_4X4 bytes, file layout */
    int rows, cols;
} or_mat;

typedef struct {
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b, *attn_b, *proj_b, *fc_in_b, *fc_out_b;
    or_mat attn_w, proj_w, fc_in_w, fc_out_w;
} or_layer;

struct or_model {
    uint8_t *file;
    size_t file_bytes;
    or_layer g[OR_LAYERS];
    or_layer local;
    const float *lnf_w, *lnf_b, *llnf_w, *llnf_b;
    or_mat wte, aemb[OR_NVQ];
    int max_ctx;
    float *g_k, *g_v; /* [12][max_ctx][768] (llm.h:132) */
    float l_k[OR_LOCAL_LEN * OR_HIDDEN], l_v[OR_LOCAL_LEN * OR_HIDDEN];
    float *cos_t, *sin_t; /* [max_ctx][384] (llm.cpp:90-102) */
    int pos, lpos;
    float hidden[OR_HIDDEN];
    int a16_decode, a16_prefill;
};

typedef struct {
    char name[49];
    int dtype, rows, cols;
    const uint8_t *ptr;
    uint64_t nbytes;
} entry_t;

static void seterr(char *err, int errlen, const char *msg, const char *name) {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s%s%s", msg, name ? ": " : "", name ? name : "");
}

static const entry_t *find_entry(const entry_t *es, int n, const char *name) {
    for (int i = 0; i < n; ++i)
        if (strcmp(es[i].name, name) == 0) return &es[i];
    return NULL;
}

static int get_mat(const entry_t *es, int n, const char *name, int rows, int cols, or_mat *out, char *err,
                   int errlen) {
    const entry_t *e = find_entry(es, n, name);
    if (!e) return seterr(err, errlen, "missing matrix", name), 0;
    if (e->dtype != 4 || e->rows != rows || e->cols != cols ||
        e->nbytes != (uint64_t)(rows / 4) * (cols / 32) * 136)
        return seterr(err, errlen, "matrix is not q8_0_4x4 of the expected shape", name), 0;
    out->data = e->ptr;
    out->rows = rows;
    out->cols = cols;
    return 1;
}

static int get_vec(const entry_t *es, int n, const char *name, int size, const float **out, char *err,
                   int errlen) {
    const entry_t *e = find_entry(es, n, name);
    if (!e) return seterr(err, errlen, "missing vector", name), 0;
    if (e->dtype != 3 || e->rows * e->cols != size || e->nbytes != (uint64_t)size * 4)
        return seterr(err, errlen, "vector is not f32 of the expected size", name), 0;
    *out = (const float *)e->ptr;
    return 1;
}

static int load_layer(const entry_t *es, int n, const char *p, or_layer *L, char *err, int errlen) {
    char nm[64];
#define VEC(field, suffix, size)                                                                   \
    snprintf(nm, sizeof(nm), "%s%s", p, suffix);                                                   \
    if (!get_vec(es, n, nm, size, &L->field, err, errlen)) return 0;
#define MAT(field, suffix, r, c)                                                                   \
    snprintf(nm, sizeof(nm), "%s%s", p, suffix);                                                   \
    if (!get_mat(es, n, nm, r, c, &L->field, err, errlen)) return 0;
    /* llm.cpp:44-57 */
    VEC(ln1_w, "ln1.w", OR_HIDDEN)
    VEC(ln1_b, "ln1.b", OR_HIDDEN)
    VEC(ln2_w, "ln2.w", OR_HIDDEN)
    VEC(ln2_b, "ln2.b", OR_HIDDEN)
    MAT(attn_w, "attn.w", 3 * OR_HIDDEN, OR_HIDDEN)
    VEC(attn_b, "attn.b", 3 * OR_HIDDEN)
    MAT(proj_w, "proj.w", OR_HIDDEN, OR_HIDDEN)
    VEC(proj_b, "proj.b", OR_HIDDEN)
    MAT(fc_in_w, "fc_in.w", OR_FF, OR_HIDDEN)
    VEC(fc_in_b, "fc_in.b", OR_FF)
    MAT(fc_out_w, "fc_out.w", OR_HIDDEN, OR_FF)
    VEC(fc_out_b, "fc_out.b", OR_HIDDEN)
#undef VEC
#undef MAT
    return 1;
}

/* weights.cpp:27-126 (container) + llm.cpp:59-110 (model) */
or_model *or_create(const char *path, int max_ctx, char *err, int errlen) {
    FILE *fh = fopen(path, "rb");
    if (!fh) return seterr(err, errlen, "cannot open weights", path), NULL;
    fseek(fh, 0, SEEK_END);
    const long size = ftell(fh);
    fseek(fh, 0, SEEK_SET);
    if (size <= 16) {
        fclose(fh);
        return seterr(err, errlen, "weights file too small", path), NULL;
    }
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->file = (uint8_t *)malloc((size_t)size);
    m->file_bytes = (size_t)size;
    const size_t got = fread(m->file, 1, (size_t)size, fh);
    fclose(fh);
    entry_t *es = NULL;
    if (got != (size_t)size) {
        seterr(err, errlen, "short read", path);
        goto fail;
    }
    if (memcmp(m->file, "MOSW", 4) != 0) {
        seterr(err, errlen, "bad magic (not a .moss file)", path);
        goto fail;
    }
    uint32_t version, n_tensors;
    memcpy(&version, m->file + 4, 4);
    memcpy(&n_tensors, m->file + 8, 4);
    if (version != 1) {
        seterr(err, errlen, "unsupported .moss version", path);
        goto fail;
    }
    if (16 + (size_t)n_tensors * 80 > (size_t)size) {
        seterr(err, errlen, "tensor table out of bounds", path);
        goto fail;
    }
    es = (entry_t *)calloc(n_tensors ? n_tensors : 1, sizeof(entry_t));
    for (uint32_t i = 0; i < n_tensors; ++i) {
        const uint8_t *base = m->file + 16 + (size_t)i * 80;
        memcpy(es[i].name, base, 48);
        es[i].name[48] = 0;
        es[i].dtype = base[48];
        uint32_t dims[3];
        uint64_t off, nbytes;
        memcpy(dims, base + 52, 12);
        memcpy(&off, base + 64, 8);
        memcpy(&nbytes, base + 72, 8);
        if (off + nbytes > (uint64_t)size) {
            seterr(err, errlen, "tensor out of bounds", es[i].name);
            goto fail;
        }
        es[i].rows = (int)dims[0];
        es[i].cols = (int)dims[1];
        es[i].ptr = m->file + off;
        es[i].nbytes = nbytes;
    }
    const int n = (int)n_tensors;
    for (int i = 0; i < OR_LAYERS; ++i) {
        char p[16];
        snprintf(p, sizeof(p), "g%d.", i);
        if (!load_layer(es, n, p, &m->g[i], err, errlen)) goto fail;
    }
    if (!load_layer(es, n, "local.", &m->local, err, errlen)) goto fail;
    if (!get_vec(es, n, "lnf.w", OR_HIDDEN, &m->lnf_w, err, errlen)) goto fail;
    if (!get_vec(es, n, "lnf.b", OR_HIDDEN, &m->lnf_b, err, errlen)) goto fail;
    if (!get_vec(es, n, "local.lnf.w", OR_HIDDEN, &m->llnf_w, err, errlen)) goto fail;
    if (!get_vec(es, n, "local.lnf.b", OR_HIDDEN, &m->llnf_b, err, errlen)) goto fail;
    if (!get_mat(es, n, "wte", OR_VOCAB, OR_HIDDEN, &m->wte, err, errlen)) goto fail;
    for (int ch = 0; ch < OR_NVQ; ++ch) {
        char nm[16];
        snprintf(nm, sizeof(nm), "aemb.%d", ch);
        if (!get_mat(es, n, nm, OR_CODEBOOK, OR_HIDDEN, &m->aemb[ch], err, errlen)) goto fail;
    }
    free(es);
    es = NULL;

    m->max_ctx = max_ctx;
    const size_t kv = (size_t)OR_LAYERS * max_ctx * OR_HIDDEN;
    m->g_k = (float *)calloc(kv, sizeof(float));
    m->g_v = (float *)calloc(kv, sizeof(float));
    m->cos_t = (float *)calloc((size_t)max_ctx * (OR_HIDDEN / 2), sizeof(float));
    m->sin_t = (float *)calloc((size_t)max_ctx * (OR_HIDDEN / 2), sizeof(float));
    const int half = OR_HEAD_DIM / 2;
    for (int pos = 0; pos < max_ctx; ++pos) {
        for (int h = 0; h < OR_HEADS; ++h) {
            for (int i = 0; i < half; ++i) {
                const double inv = 1.0 / pow(10000.0, (double)(2 * i) / OR_HEAD_DIM);
                const double angle = (double)pos * inv;
                m->cos_t[(size_t)pos * (OR_HIDDEN / 2) + h * half + i] = (float)cos(angle);
                m->sin_t[(size_t)pos * (OR_HIDDEN / 2) + h * half + i] = (float)sin(angle);
            }
        }
    }
    m->a16_decode = 1; /* MOSS_A16=decode, the product default (capi.cpp:52) */
    m->a16_prefill = 0;
    m->pos = 0;
    return m;
fail:
    free(es);
    free(m->file);
    free(m);
    return NULL;
}

void or_destroy(or_model *m) {
    if (!m) return;
    free(m->file);
    free(m->g_k);
    free(m->g_v);
    free(m->cos_t);
    free(m->sin_t);
    free(m);
}

void or_set_modes(or_model *m, int a16_decode, int a16_prefill) {
    m->a16_decode = a16_decode;
    m->a16_prefill = a16_prefill;
}

void or_reset(or_model *m) { m->pos = 0; } /* llm.cpp:112 */
int or_position(const or_model *m) { return m->pos; }
void or_get_hidden(const or_model *m, float *out) { memcpy(out, m->hidden, sizeof(m->hidden)); }

int or_set_state(or_model *m, const float *k, const float *v, int n_pos, const float *hidden) {
    if (n_pos <= 0 || n_pos > m->max_ctx) return 0;
    for (int l = 0; l < OR_LAYERS; ++l) {
        const size_t dst = (size_t)l * m->max_ctx * OR_HIDDEN;
        const size_t src = (size_t)l * n_pos * OR_HIDDEN;
        memcpy(m->g_k + dst, k + src, sizeof(float) * (size_t)n_pos * OR_HIDDEN);
        memcpy(m->g_v + dst, v + src, sizeof(float) * (size_t)n_pos * OR_HIDDEN);
    }
    if (hidden) memcpy(m->hidden, hidden, sizeof(m->hidden));
    m->pos = n_pos;
    return 1;
}

void or_get_kv(const or_model *m, int layer, int p0, int n, float *k, float *v) {
    const size_t base = ((size_t)layer * m->max_ctx + p0) * OR_HIDDEN;
    if (k) memcpy(k, m->g_k + base, sizeof(float) * (size_t)n * OR_HIDDEN);
    if (v) memcpy(v, m->g_v + base, sizeof(float) * (size_t)n * OR_HIDDEN);
}

/* llm.cpp:114-146 (Q8_0_4X4 case) */
static void lookup_row(const or_mat *mat, int row, float *out) {
    const int nb = mat->cols / 32;
    or_dequant_row_q8x4(mat->data + (size_t)(row / 4) * nb * 136, nb, row % 4, out);
}

/* llm.cpp:148-157 */
void or_embed_row(const or_model *m, const int32_t *row, float *out) {
    lookup_row(&m->wte, row[0], out);
    float tmp[OR_HIDDEN];
    for (int ch = 0; ch < OR_NVQ; ++ch) {
        const int code = row[ch + 1];
        if (code == OR_AUDIO_PAD || code < 0 || code >= OR_CODEBOOK) continue;
        lookup_row(&m->aemb[ch], code, tmp);
        for (int i = 0; i < OR_HIDDEN; ++i) out[i] += tmp[i];
    }
}

/* llm.cpp:173-187 */
static void rope(const or_model *m, float *vec, int position) {
    const float *c = m->cos_t + (size_t)position * (OR_HIDDEN / 2);
    const float *s = m->sin_t + (size_t)position * (OR_HIDDEN / 2);
    for (int h = 0; h < OR_HEADS; ++h) {
        float *base = vec + h * OR_HEAD_DIM;
        for (int i = 0; i < OR_HEAD_DIM / 2; ++i) {
            const float c0 = c[h * (OR_HEAD_DIM / 2) + i];
            const float s0 = s[h * (OR_HEAD_DIM / 2) + i];
            const float x0 = base[2 * i];
            const float x1 = base[2 * i + 1];
            base[2 * i] = x0 * c0 - x1 * s0;
            base[2 * i + 1] = x1 * c0 + x0 * s0;
        }
    }
}

/* llm.cpp:189-217 */
static void attention_core(const float *k_cache, const float *v_cache, int n_pos, const float *q, float *out,
                           float *scores) {
    const float scale = 1.0f / sqrtf((float)OR_HEAD_DIM);
    for (int h = 0; h < OR_HEADS; ++h) {
        const float *qh = q + h * OR_HEAD_DIM;
        float *oh = out + h * OR_HEAD_DIM;
        float max_score = -1e30f;
        for (int p = 0; p < n_pos; ++p) {
            const float *kh = k_cache + (size_t)p * OR_HIDDEN + h * OR_HEAD_DIM;
            float dot = 0.0f;
            for (int d = 0; d < OR_HEAD_DIM; ++d) dot += qh[d] * kh[d];
            dot *= scale;
            scores[p] = dot;
            max_score = max_score < dot ? dot : max_score;
        }
        float sum = 0.0f;
        for (int p = 0; p < n_pos; ++p) {
            scores[p] = expf(scores[p] - max_score);
            sum += scores[p];
        }
        const float inv_sum = 1.0f / sum;
        for (int d = 0; d < OR_HEAD_DIM; ++d) oh[d] = 0.0f;
        for (int p = 0; p < n_pos; ++p) {
            const float w = scores[p] * inv_sum;
            const float *vh = v_cache + (size_t)p * OR_HIDDEN + h * OR_HEAD_DIM;
            for (int d = 0; d < OR_HEAD_DIM; ++d) oh[d] += w * vh[d];
        }
    }
}

/* llm.cpp:230-246; k_cache/v_cache are the layer's [ctx][768] caches (llm.cpp:219-228) */
static void block_forward(const or_model *m, const or_layer *L, float *k_cache, float *v_cache, int ctx,
                          int position, float *x, int a16) {
    float ln[OR_HIDDEN], qkv[3 * OR_HIDDEN], att[OR_HIDDEN], res[OR_HIDDEN];
    float *mlp = (float *)malloc(sizeof(float) * OR_FF);
    float *scores = (float *)malloc(sizeof(float) * (size_t)(ctx > 0 ? ctx : 1));
    or_layernorm(x, L->ln1_w, L->ln1_b, ln);
    or_gemv(L->attn_w.data, 3 * OR_HIDDEN, OR_HIDDEN, ln, qkv, a16);
    for (int i = 0; i < 3 * OR_HIDDEN; ++i) qkv[i] += L->attn_b[i];
    rope(m, qkv, position);
    rope(m, qkv + OR_HIDDEN, position);
    memcpy(k_cache + (size_t)position * OR_HIDDEN, qkv + OR_HIDDEN, sizeof(float) * OR_HIDDEN);
    memcpy(v_cache + (size_t)position * OR_HIDDEN, qkv + 2 * OR_HIDDEN, sizeof(float) * OR_HIDDEN);
    attention_core(k_cache, v_cache, position + 1, qkv, att, scores);
    or_gemv(L->proj_w.data, OR_HIDDEN, OR_HIDDEN, att, res, a16);
    for (int i = 0; i < OR_HIDDEN; ++i) x[i] += res[i] + L->proj_b[i];
    or_layernorm(x, L->ln2_w, L->ln2_b, ln);
    or_gemv(L->fc_in_w.data, OR_FF, OR_HIDDEN, ln, mlp, a16);
    for (int i = 0; i < OR_FF; ++i) mlp[i] = gelu_new(mlp[i] + L->fc_in_b[i]);
    or_gemv(L->fc_out_w.data, OR_HIDDEN, OR_FF, mlp, res, a16);
    for (int i = 0; i < OR_HIDDEN; ++i) x[i] += res[i] + L->fc_out_b[i];
    free(mlp);
    free(scores);
}

static void global_layers(or_model *m, float *x, float *hidden_out) {
    for (int i = 0; i < OR_LAYERS; ++i) {
        float *kc = m->g_k + (size_t)i * m->max_ctx * OR_HIDDEN;
        float *vc = m->g_v + (size_t)i * m->max_ctx * OR_HIDDEN;
        block_forward(m, &m->g[i], kc, vc, m->max_ctx, m->pos, x, m->a16_decode);
    }
    or_layernorm(x, m->lnf_w, m->lnf_b, hidden_out);
    ++m->pos;
}

/* llm.cpp:248-255 */
void or_global_step_embed(or_model *m, const float *xin, float *hidden_out) {
    float x[OR_HIDDEN];
    memcpy(x, xin, sizeof(x));
    global_layers(m, x, hidden_out ? hidden_out : m->hidden);
    if (hidden_out && hidden_out != m->hidden) memcpy(m->hidden, hidden_out, sizeof(m->hidden));
}

void or_global_step_row(or_model *m, const int32_t *row, float *hidden_out) {
    float x[OR_HIDDEN];
    or_embed_row(m, row, x);
    or_global_step_embed(m, x, hidden_out);
}

/* llm.cpp:257-264 */
void or_local_step(or_model *m, int lpos, const float *input, float *out) {
    float x[OR_HIDDEN];
    memcpy(x, input, sizeof(x));
    block_forward(m, &m->local, m->l_k, m->l_v, OR_LOCAL_LEN, lpos, x, m->a16_decode);
    or_layernorm(x, m->llnf_w, m->llnf_b, out);
}

/* llm.cpp:268-270 */
void or_audio_logits(const or_model *m, int ch, const float *hidden, float *logits) {
    or_gemv(m->aemb[ch].data, OR_CODEBOOK, OR_HIDDEN, hidden, logits, m->a16_decode);
}

/* llm.cpp:274-315 (Q8_0_4X4 case): always W8A8 */
void or_assistant_logits(const or_model *m, const float *hidden, float *pair) {
    static const int rows[2] = {OR_END, OR_SLOT};
    int8_t qa[OR_HIDDEN];
    float as[OR_HIDDEN / 32];
    or_quantize_act(hidden, OR_HIDDEN, qa, as);
    const int nb = OR_HIDDEN / 32;
    for (int i = 0; i < 2; ++i) {
        const int r = rows[i];
        pair[i] = or_row_dot_a8(m->wte.data + (size_t)(r / 4) * nb * 136, nb, r % 4, qa, as);
    }
}

/* llm.cpp:327-401 */
static void prefill_impl(or_model *m, const float *x_in, const int32_t *rows, int n_rows, int start) {
    start = start < 0 ? 0 : (start > m->max_ctx ? m->max_ctx : start);
    const int n = n_rows < m->max_ctx - start ? n_rows : m->max_ctx - start;
    if (n <= 0) return;
    const int a16 = m->a16_prefill;
    float *bx = (float *)malloc(sizeof(float) * (size_t)n * OR_HIDDEN);
    float *bln = (float *)malloc(sizeof(float) * (size_t)n * OR_HIDDEN);
    float *bqkv = (float *)malloc(sizeof(float) * (size_t)n * 3 * OR_HIDDEN);
    float *batt = (float *)malloc(sizeof(float) * (size_t)n * OR_HIDDEN);
    float *bmlp = (float *)malloc(sizeof(float) * (size_t)n * OR_FF);
    float *bres = (float *)malloc(sizeof(float) * (size_t)n * OR_HIDDEN);
    float *scores = (float *)malloc(sizeof(float) * (size_t)m->max_ctx);
    for (int i = 0; i < n; ++i) {
        if (rows) or_embed_row(m, rows + (size_t)i * 17, bx + (size_t)i * OR_HIDDEN);
        else memcpy(bx + (size_t)i * OR_HIDDEN, x_in + (size_t)i * OR_HIDDEN, sizeof(float) * OR_HIDDEN);
    }
    for (int layer = 0; layer < OR_LAYERS; ++layer) {
        const or_layer *L = &m->g[layer];
        float *kc = m->g_k + (size_t)layer * m->max_ctx * OR_HIDDEN;
        float *vc = m->g_v + (size_t)layer * m->max_ctx * OR_HIDDEN;
        for (int i = 0; i < n; ++i) or_layernorm(bx + (size_t)i * OR_HIDDEN, L->ln1_w, L->ln1_b, bln + (size_t)i * OR_HIDDEN);
        for (int i = 0; i < n; ++i)
            or_gemv(L->attn_w.data, 3 * OR_HIDDEN, OR_HIDDEN, bln + (size_t)i * OR_HIDDEN, bqkv + (size_t)i * 3 * OR_HIDDEN, a16);
        for (int i = 0; i < n; ++i) {
            float *qkv = bqkv + (size_t)i * 3 * OR_HIDDEN;
            const int p = start + i;
            for (int k = 0; k < 3 * OR_HIDDEN; ++k) qkv[k] += L->attn_b[k];
            rope(m, qkv, p);
            rope(m, qkv + OR_HIDDEN, p);
            memcpy(kc + (size_t)p * OR_HIDDEN, qkv + OR_HIDDEN, sizeof(float) * OR_HIDDEN);
            memcpy(vc + (size_t)p * OR_HIDDEN, qkv + 2 * OR_HIDDEN, sizeof(float) * OR_HIDDEN);
        }
        for (int i = 0; i < n; ++i)
            attention_core(kc, vc, start + i + 1, bqkv + (size_t)i * 3 * OR_HIDDEN, batt + (size_t)i * OR_HIDDEN, scores);
        for (int i = 0; i < n; ++i) or_gemv(L->proj_w.data, OR_HIDDEN, OR_HIDDEN, batt + (size_t)i * OR_HIDDEN, bres + (size_t)i * OR_HIDDEN, a16);
        for (int i = 0; i < n; ++i) {
            float *x = bx + (size_t)i * OR_HIDDEN;
            const float *r = bres + (size_t)i * OR_HIDDEN;
            for (int k = 0; k < OR_HIDDEN; ++k) x[k] += r[k] + L->proj_b[k];
        }
        for (int i = 0; i < n; ++i) or_layernorm(bx + (size_t)i * OR_HIDDEN, L->ln2_w, L->ln2_b, bln + (size_t)i * OR_HIDDEN);
        for (int i = 0; i < n; ++i) or_gemv(L->fc_in_w.data, OR_FF, OR_HIDDEN, bln + (size_t)i * OR_HIDDEN, bmlp + (size_t)i * OR_FF, a16);
        for (int i = 0; i < n; ++i) {
            float *mlp = bmlp + (size_t)i * OR_FF;
            for (int k = 0; k < OR_FF; ++k) mlp[k] = gelu_new(mlp[k] + L->fc_in_b[k]);
        }
        for (int i = 0; i < n; ++i) or_gemv(L->fc_out_w.data, OR_HIDDEN, OR_FF, bmlp + (size_t)i * OR_FF, bres + (size_t)i * OR_HIDDEN, a16);
        for (int i = 0; i < n; ++i) {
            float *x = bx + (size_t)i * OR_HIDDEN;
            const float *r = bres + (size_t)i * OR_HIDDEN;
            for (int k = 0; k < OR_HIDDEN; ++k) x[k] += r[k] + L->fc_out_b[k];
        }
    }
    or_layernorm(bx + (size_t)(n - 1) * OR_HIDDEN, m->lnf_w, m->lnf_b, m->hidden);
    m->pos = start + n;
    free(bx);
    free(bln);
    free(bqkv);
    free(batt);
    free(bmlp);
    free(bres);
    free(scores);
}

void or_prefill_rows(or_model *m, const int32_t *rows, int n, int start) { prefill_impl(m, NULL, rows, n, start); }
void or_prefill_embeds(or_model *m, const float *x, int n, int start) { prefill_impl(m, x, NULL, n, start); }

/* n_frames whole frames = generate()'s loop body (llm.cpp:647-708) with the global step
 * always taken and greedy codes; used to time the C port per frame.  codes [n_frames][16]. */
void or_frames(or_model *m, int n_frames, float rep, int32_t *codes) {
    or_sample_params p = {1, 1.0f, 0, 1.0f, rep, 1, 0, 0};
    uint32_t rng[4];
    or_rng_seed(rng, 0);
    int *history = (int *)malloc(sizeof(int) * (size_t)OR_NVQ * (n_frames > 0 ? n_frames : 1));
    float lx[OR_HIDDEN], input[OR_HIDDEN], logits[OR_CODEBOOK], pair[2];
    for (int f = 0; f < n_frames && m->pos < m->max_ctx; ++f) {
        or_local_step(m, 0, m->hidden, lx);
        or_assistant_logits(m, lx, pair);
        lookup_row(&m->wte, OR_SLOT, input);
        int32_t next[17];
        next[0] = OR_SLOT;
        for (int ch = 0; ch < OR_NVQ; ++ch) {
            or_local_step(m, ch + 1, input, lx);
            or_audio_logits(m, ch, lx, logits);
            int *hist = history + (size_t)ch * n_frames;
            const int pred = or_sample_token(logits, OR_CODEBOOK, &p, hist, f, rng);
            hist[f] = pred;
            next[ch + 1] = pred;
            codes[(size_t)f * OR_NVQ + ch] = pred;
            lookup_row(&m->aemb[ch], pred, input);
        }
        or_global_step_row(m, next, NULL);
    }
    free(history);
}

/* llm.cpp:634-712 */
int or_generate(or_model *m, int max_frames, const or_sample_params *p, uint64_t seed, const int32_t *forced,
                int32_t *codes, float *logits_out, float *gate_out) {
    uint32_t rng[4];
    or_rng_seed(rng, seed);
    int *history = (int *)malloc(sizeof(int) * (size_t)OR_NVQ * (max_frames > 0 ? max_frames : 1));
    int n_hist = 0;
    float lx[OR_HIDDEN], input[OR_HIDDEN], logits[OR_CODEBOOK];
    int frames = 0;
    for (int f = 0; f < max_frames; ++f) {
        if (m->pos >= m->max_ctx) break;
        m->lpos = 0;
        or_local_step(m, m->lpos++, m->hidden, lx);
        float pair[2];
        or_assistant_logits(m, lx, pair);
        const float l_end = pair[0], l_slot = pair[1];
        if (gate_out) {
            gate_out[2 * f] = l_end;
            gate_out[2 * f + 1] = l_slot;
        }
        if (f >= p->min_frames && end_reached(l_slot, l_end, p, rng)) break;
        lookup_row(&m->wte, OR_SLOT, input);
        or_sample_params fp = *p;
        if (f < p->greedy_frames) fp.greedy = 1;
        int32_t frame[OR_NVQ];
        for (int ch = 0; ch < OR_NVQ; ++ch) {
            or_local_step(m, m->lpos++, input, lx);
            or_audio_logits(m, ch, lx, logits);
            if (logits_out) memcpy(logits_out + ((size_t)f * OR_NVQ + ch) * OR_CODEBOOK, logits, sizeof(logits));
            /* history[ch] holds the codes used so far on this channel, in order */
            int *hist = history + (size_t)ch * max_frames;
            const int predicted = or_sample_token(logits, OR_CODEBOOK, &fp, hist, n_hist, rng);
            const int used = forced ? forced[(size_t)f * OR_NVQ + ch] : predicted;
            frame[ch] = predicted;
            hist[n_hist] = used;
            lookup_row(&m->aemb[ch], used, input);
        }
        ++n_hist;
        memcpy(codes + (size_t)f * OR_NVQ, frame, sizeof(frame));
        frames = f + 1;
        if (f + 1 < max_frames && m->pos < m->max_ctx) {
            int32_t next[17];
            next[0] = OR_SLOT;
            for (int ch = 0; ch < OR_NVQ; ++ch) next[ch + 1] = forced ? forced[(size_t)f * OR_NVQ + ch] : frame[ch];
            or_global_step_row(m, next, NULL);
        }
    }
    free(history);
    return frames;
}
