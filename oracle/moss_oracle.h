/*
 * moss_oracle.h -- CPU restatement of the MOSS-TTS-Nano per-frame LLM step.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA engine is compared
 * against; it is never linked into, called by, or used as a fallback for the product
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.
 *
 * Every function restates one function of the reference (csrc/src/... in
 * litterbit/dsh-moss-tts) in plain C, keeping its floating-point operation order so
 * that, compiled with the same compiler and without FMA contraction, it reproduces the
 * reference bit for bit (see oracle/Makefile: the same flags the reference build uses
 * for its non-AVX2 translation units; the AVX2 kernels are restated lane by lane with
 * fmaf).  Citations are file:line in the reference.
 */
#ifndef MOSS_ORACLE_H
#define MOSS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_HIDDEN = 768, OR_HEADS = 12, OR_HEAD_DIM = 64, OR_FF = 3072, OR_VOCAB = 16384,
       OR_NVQ = 16, OR_CODEBOOK = 1024, OR_AUDIO_PAD = 1024, OR_SLOT = 9, OR_END = 7,
       OR_LOCAL_LEN = 17, OR_LAYERS = 12 };

typedef struct or_model or_model;

typedef struct {
    int greedy;             /* sampler.h:9 */
    float temperature;      /* sampler.h:10 */
    int top_k;              /* sampler.h:11 */
    float top_p;            /* sampler.h:12 */
    float repetition_penalty; /* sampler.h:13 */
    int end_greedy;         /* sampler.h:17 */
    int min_frames;         /* sampler.h:19 */
    int greedy_frames;      /* sampler.h:21 */
} or_sample_params;

/* fp16.cpp:7-35, fp16.cpp:37-66 */
float or_half_to_float(uint16_t h);
uint16_t or_float_to_half(float f);
void or_half_to_float_n(const uint16_t *h, int n, float *out);
void or_float_to_half_n(const float *f, int n, uint16_t *out);

/* quant.cpp:56-65: one row (k in 0..3 of its 4-row group) of a Q8_0_4X4 matrix */
void or_dequant_row_q8x4(const uint8_t *group, int nb, int k, float *out);
/* W8A16 row dot, AVX2 lane order: gemv_avx2.cpp:123-150 */
float or_row_dot_a16(const uint8_t *group, int nb, int k, const float *act);
/* quant.cpp:28-43 (the fp32-scale variant used by quantize_activation, quant.cpp:45-54) */
void or_quantize_act(const float *x, int n, int8_t *q, float *scales);
/* W8A8 row dot, AVX2 lane order: gemv_avx2.cpp:105-121 */
float or_row_dot_a8(const uint8_t *group, int nb, int k, const int8_t *qa, const float *as);
/* y[rows] = W x in W8A16 (a16=1) or W8A8 (a16=0): gemv.cpp:245-274 / gemv_avx2.cpp:173-191 */
void or_gemv(const uint8_t *w, int rows, int cols, const float *x, float *y, int a16);

/* llm.cpp:159-171 */
void or_layernorm(const float *x, const float *w, const float *b, float *out);
/* sampler.cpp:9-77 with Rng from sampler.h:25-48; rng_state is uint32[4], updated */
int or_sample_token(const float *logits, int n, const or_sample_params *p, const int *prev,
                    int n_prev, uint32_t *rng_state);
void or_rng_seed(uint32_t *rng_state, uint64_t seed);
float or_rng_uniform(uint32_t *rng_state);

/* Model: weights.cpp:27-126 (file parse) + llm.cpp:59-110 (load) */
or_model *or_create(const char *moss_path, int max_ctx, char *err, int errlen);
void or_destroy(or_model *m);
void or_set_modes(or_model *m, int a16_decode, int a16_prefill);
void or_reset(or_model *m);
int or_position(const or_model *m);
void or_get_hidden(const or_model *m, float *out);
/* inject a prefilled state: fp32 K,V [12][n_pos][768] and hidden[768] (llm.cpp:588-632) */
int or_set_state(or_model *m, const float *k, const float *v, int n_pos, const float *hidden);
/* read back K or V rows [n][768] of one global layer starting at position p0 */
void or_get_kv(const or_model *m, int layer, int p0, int n, float *k, float *v);
/* llm.cpp:148-157 */
void or_embed_row(const or_model *m, const int32_t *row17, float *out);
/* llm.cpp:248-255 with the embedding given directly (x_ = x) */
void or_global_step_embed(or_model *m, const float *x, float *hidden_out);
/* llm.cpp:248-255 */
void or_global_step_row(or_model *m, const int32_t *row17, float *hidden_out);
/* llm.cpp:327-401 with rows given (embed_row) or embeddings given directly */
void or_prefill_rows(or_model *m, const int32_t *rows, int n, int start);
void or_prefill_embeds(or_model *m, const float *x, int n, int start);
/* llm.cpp:257-264 on an explicit local state: one local step at local position lpos */
void or_local_step(or_model *m, int lpos, const float *input, float *out);
/* llm.cpp:268-270 */
void or_audio_logits(const or_model *m, int ch, const float *hidden, float *logits);
/* llm.cpp:274-315: pair[0] = end(7), pair[1] = slot(9) */
void or_assistant_logits(const or_model *m, const float *hidden, float *pair);
/* llm.cpp:634-712.  forced: [max_frames][16] or NULL; codes out [max_frames][16];
 * logits out [max_frames][16][1024] or NULL; gate out [max_frames][2] (end, slot) or NULL.
 * Returns the number of frames produced. */
int or_generate(or_model *m, int max_frames, const or_sample_params *p, uint64_t seed,
                const int32_t *forced, int32_t *codes, float *logits, float *gate);
/* n_frames whole frames (local decoder + greedy codes + global step each); for timing */
void or_frames(or_model *m, int n_frames, float rep, int32_t *codes);

#ifdef __cplusplus
}
#endif
#endif
