/*
 * mossgpu.h -- C ABI of the B200 engine for MOSS-TTS-Nano's per-frame LLM step.
 *
 * Drop-in boundary: these entry points replace the single-stream C++ class
 * moss::LlmModel (reference csrc/include/moss/llm.h:39-158, csrc/src/llm.cpp) with a
 * batched, device-resident engine.  A thin C++ shim with LlmModel's method names
 * (dsh-moss-tts_b200/csrc/llm_gpu.h) maps the reference's calls onto them, so the
 * reference's TtsEngine (engine.cpp) and Runtime (runtime.cpp) keep their signatures.
 *
 * Conventions (the reference's capi.cpp:16-23,109 convention): every int-returning call
 * returns 0 on success and non-zero on failure; the message is kept per engine and read
 * with mossgpu_last_error().  No call throws across the ABI.  All pointers are host
 * pointers unless a name says otherwise; sizes are element counts.
 *
 * Streams: one "stream" is one utterance's LLM state (global KV, last hidden, local
 * decoder state, repetition-penalty history).  mossgpu_step() advances any set of open
 * streams by one audio frame in one batched pass.
 *
 * Threads: calls on one engine must not overlap; any thread may make them, and each call
 * first makes the engine's device current on the calling thread.  Different engines (one
 * per GPU) may be called concurrently from different threads.
 */
#ifndef MOSSGPU_H
#define MOSSGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mossgpu_engine mossgpu_engine;

/* Mirrors moss::SampleParams (reference csrc/include/moss/sampler.h:8-22).  Sampling runs on
 * the device with the reference's arithmetic and draw order (sampler.cpp:9-77): the
 * repetition penalty, then either the first maximum or temperature -> sort by (value desc,
 * index asc) -> top-k -> exp/sum -> top-p -> one xoshiro128** draw per channel from the
 * stream's generator, seeded by mossgpu_generate_begin as generate() seeds it. */
typedef struct {
    int greedy;                /* 1: argmax (after the repetition penalty) */
    float temperature;         /* stochastic path only */
    int top_k;                 /* stochastic path only; 1 == greedy, <= 0 == all 1024 codes */
    float top_p;               /* stochastic path only */
    float repetition_penalty;  /* applied once per earlier occurrence (sampler.cpp:14-21) */
    int end_greedy;            /* 1: stop iff logit(end=7) > logit(slot=9); 0: one draw against
                                  p(slot) = 1 / (1 + e^(l_end - l_slot)) (llm.cpp:30-35) */
    int min_frames;            /* no stop before this frame index */
    int greedy_frames;         /* frames below this index are greedy */
} mossgpu_sample_params;

/* Engine lifetime.  Replaces LlmModel(threads) + LlmModel::load (llm.cpp:42-110): parses
 * the .moss file (weights.cpp:27-126 semantics), uploads it to device `device_id`,
 * repacks every Q8_0_4X4 matrix into 16-byte-aligned quant/scale planes, and allocates the
 * paged fp16 KV cache.  max_ctx caps positions per stream (reference kMaxCtx, llm.h:28);
 * kv_pages = 0 sizes the pool for max_streams * max_ctx positions.  Returns NULL on
 * failure with the reason in err (may be NULL). */
mossgpu_engine *mossgpu_create(const char *weights_path, int device_id, int max_streams, int max_ctx,
                               int kv_pages, char *err, int errlen);
/* Same, with max_rows = the rows of one pass through the layers: a prefill pass over one or
 * several streams (mossgpu_prefill_batch), or a decode batch.  0 = max(max_streams, 256).
 * A pass of thousands of rows makes every weight GEMM a dense contraction on the tensor
 * cores; device memory grows by ~33 KB per row. */
mossgpu_engine *mossgpu_create_rows(const char *weights_path, int device_id, int max_streams, int max_ctx,
                                    int kv_pages, int max_rows, char *err, int errlen);
void mossgpu_destroy(mossgpu_engine *e);
const char *mossgpu_last_error(mossgpu_engine *e);
const char *mossgpu_version(void);

/* Run all work on the caller's cudaStream_t (passed as void*); NULL = the engine's own. */
int mossgpu_set_cuda_stream(mossgpu_engine *e, void *cuda_stream);

/* Stream slots.  open = a fresh LlmModel state (reset(), llm.cpp:112). */
int mossgpu_stream_open(mossgpu_engine *e, int *stream_id);
int mossgpu_stream_close(mossgpu_engine *e, int stream_id);
int mossgpu_stream_reset(mossgpu_engine *e, int stream_id);
int mossgpu_stream_position(mossgpu_engine *e, int stream_id, int *position);

/* A new stream whose first n_pos positions are those of src_stream (n_pos <= its position),
 * for voice-prompt prefixes shared by many utterances (snapshot_prefix / restore_prefix,
 * llm.cpp:455-483, done on the device): the full 16-position KV pages are shared, not copied
 * (reference counted), the partly filled last page is copied, the hidden state is src's and
 * the position is n_pos.  Either stream writing into a shared page first copies it, so the
 * two never see each other's later positions.  Call mossgpu_generate_begin before stepping
 * the new stream. */
int mossgpu_stream_fork(mossgpu_engine *e, int src_stream, int n_pos, int *new_stream);

/* LlmModel::prefill(rows, start) (llm.cpp:327-401): rows[m][17] = [text_id, code0..15].
 * Writes the KV for positions start..start+m-1 and leaves the last row's ln_f output as
 * the stream's hidden state; position becomes start + m.  Computes in A16 (fp32
 * activations x int8 weights), the reference's MOSS_A16=all prefill mode. */
int mossgpu_prefill(mossgpu_engine *e, int stream_id, const int32_t *rows, int m, int start);
/* Same with the token embeddings given directly, x[m][768] fp32. */
int mossgpu_prefill_embeds(mossgpu_engine *e, int stream_id, const float *x, int m, int start);
/* LlmModel::prefill for n distinct streams in shared passes (the Runtime batching many
 * utterances): stream_ids[i] gets m[i] rows at positions start[i].. (clamped as the single
 * prefill clamps them), its rows taken in order from rows[.][17] (or x[.][768]), stream
 * after stream.  Each stream ends exactly as if it had been prefilled alone. */
int mossgpu_prefill_batch(mossgpu_engine *e, int n, const int32_t *stream_ids, const int32_t *m, const int32_t *start,
                          const int32_t *rows);
int mossgpu_prefill_embeds_batch(mossgpu_engine *e, int n, const int32_t *stream_ids, const int32_t *m,
                                 const int32_t *start, const float *x);

/* Start a generate() call on a stream (llm.cpp:637-641): clears the per-channel code
 * history and sets the frame counter to 0. */
int mossgpu_generate_begin(mossgpu_engine *e, int stream_id, uint64_t seed);

/* One frame of LlmModel::generate (llm.cpp:643-712) for n streams at once:
 * local decoder from the stream's hidden state, the W8A8 end gate, 16 codes (greedy with
 * repetition penalty), then -- when run_global != 0 -- the 12-layer global step on
 * [9, codes] that appends one KV position and refreshes the hidden state.
 *   forced     [n][16] teacher-forcing codes (llm.cpp:694,706) or NULL
 *   out_codes  [n][16] the model's own predictions
 *   out_stop   [n]     1 when the gate ended the stream this frame (its codes are void and
 *                      its state is unchanged, as the reference's `break`)
 *   out_logits [n][16][1024] audio logits before sampling, or NULL
 *   out_gate   [n][2]  (logit_end, logit_slot), or NULL */
int mossgpu_step(mossgpu_engine *e, const int32_t *stream_ids, int n, const mossgpu_sample_params *params,
                 const int32_t *forced, int32_t *out_codes, uint8_t *out_stop, float *out_logits, float *out_gate,
                 int run_global);

/* n_frames consecutive frames of generate() for n streams in one call, free-running (no
 * teacher forcing), with no host round trip between frames: positions, frame indices and
 * the end gate advance on the device.  out_codes [n_frames][n][16] holds -1 for frames after
 * a stream stopped; out_frames_done [n] is the number of frames each stream produced
 * (< n_frames when its gate ended it).  n_frames <= 1024. */
int mossgpu_step_frames(mossgpu_engine *e, const int32_t *stream_ids, int n, const mossgpu_sample_params *params,
                        int n_frames, int32_t *out_codes, int32_t *out_frames_done);

/* The 12-layer global step alone with the input embedding given (llm.cpp:248-255 with
 * x_ = x): x[n][768] fp32; hidden_out[n][768] or NULL.  Appends one KV position. */
int mossgpu_global_step_embed(mossgpu_engine *e, const int32_t *stream_ids, int n, const float *x, float *hidden_out);

/* State access (llm.cpp:588-632 load_state semantics and debugging):
 * set_state writes K,V fp32 [12][n_pos][768] (stored as fp16 pages) and hidden[768].
 * get_kv reads layer `layer`, positions p0..p0+n-1, back as fp32 [n][768]. */
int mossgpu_set_state(mossgpu_engine *e, int stream_id, const float *k, const float *v, int n_pos,
                      const float *hidden);
int mossgpu_get_kv(mossgpu_engine *e, int stream_id, int layer, int p0, int n, float *k, float *v);
int mossgpu_get_hidden(mossgpu_engine *e, int stream_id, float *hidden);

/* Read back one repacked matrix (by .moss tensor name) as the original Q8_0_4X4 bytes,
 * rows/4 * cols/32 * 136 bytes, to prove the device repack is a byte permutation. */
int mossgpu_debug_matrix_bytes(mossgpu_engine *e, const char *name, uint8_t *out, size_t out_bytes);

/* Kernel launches issued by the last mossgpu_step / mossgpu_global_step_embed call. */
int mossgpu_last_launch_count(mossgpu_engine *e);

/* Synthetic prefilled state (benchmarks and tests; the reference's nearest counterpart is
 * load_state, llm.cpp:588-632): K, V ~ N(0,1) rounded to fp16 for positions 0..n_pos-1 of
 * every layer and hidden ~ N(0,1), generated on the device from `seed`. */
int mossgpu_fill_state_random(mossgpu_engine *e, int stream_id, int n_pos, uint64_t seed);

/* Execution options: graphs = 1 (default) replays each frame as a CUDA graph captured on
 * first use per batch size; 0 launches kernels one by one.
 * gemm_path: 0 = automatic (CUDA-core GEMV up to 8 rows, tcgen05 tensor-core GEMM for 9..256
 * rows), 1 = always the CUDA-core GEMV, 2 = tensor cores whenever rows <= 256, 3 = as 2 but
 * with single fp16 operands instead of the default hi/lo fp16 split (faster, ~5e-4 relative
 * rounding on weights and activations; the default split keeps fp32-level accuracy). */
int mossgpu_set_graphs(mossgpu_engine *e, int enable);
/* Local decoder (the 17 one-layer steps, the audio heads and the codes of a frame):
 * 0 = for greedy frames (params.greedy, or top_k == 1), one fused kernel per frame segment --
 *   step 0, then steps 1..16 after the end gate -- in which thread-block clusters of 8 rows keep
 *   the activations on chip and stream the local weights from L2; other frames take the
 *   per-step kernels;
 * 1 (default) = the per-step kernels for every frame (about 10 launches per step).  Measured
 *   on one B200: 1.97 ms per 64-stream frame either way, and at 512 streams the fused form is
 *   slower (5.1 against 2.5 ms for the local decoder), so it is not the default. */
int mossgpu_set_local_path(mossgpu_engine *e, int mode);
/* Global layers of decode batches of at most 8 rows on the CUDA-core path:
 * 1 (default) = two launches per layer: an attention half in which a thread-block cluster of
 *   8 CTAs per head runs LN1, QKV, RoPE, the KV append, attention and the head's share of proj,
 *   and an MLP half (LN2, fc_in, GELU, fc_out over 32 features per CTA); the residual stream
 *   between them is an int64 accumulator (2^-32 units, atomic adds, so the result is the same
 *   on every run); limit |activation| < 2^31;
 * 0 = five launches per layer (QKV, attention, proj, fc_in, fc_out GEMV kernels).
 * Prefill passes always take the five-launch form. */
int mossgpu_set_small_layers(mossgpu_engine *e, int mode);
/* Profiling aid for the two-launch layers: in a library built with -DMOSSGPU_PHASE_STAMPS
 * (`bench.py --phase-stamps` builds one beside the product library), thread 0 of every CTA
 * stamps %globaltimer (ns) at each phase boundary of the last step's small-layer launches;
 * copies them as [24 launches][96 CTAs][12 phases] (n >= 27,648 entries).  Other builds return
 * non-zero ("built without phase stamps").  No counterpart in the reference. */
int mossgpu_debug_small_layer_stamps(mossgpu_engine *e, unsigned long long *out, size_t n);
int mossgpu_set_gemm_path(mossgpu_engine *e, int mode);
/* Tensor-core GEMM form by batch size: batches of at least direct_min_rows padded rows run
 * one CTA per (128 weight rows, slice of direct_rows batch rows) over the whole K with the
 * accumulators read straight from tensor memory; smaller batches split K over thread-block
 * clusters.  direct_min_rows = 0 disables the direct form; direct_rows = 0 sizes the slices
 * per matrix (the fewest rows whose tiles fit one wave of the SMs; split-K for a matrix with
 * too few tiles) below 1024 rows and takes 256-row slices from there on.  Default (256, 0),
 * measured on one B200: 9.75 ms per 512-stream decode frame against 10.70 with split-K
 * throughout; 5.80 against 5.87 ms at 256 streams; at 128 streams split-K is faster. */
int mossgpu_set_tc_policy(mossgpu_engine *e, int direct_min_rows, int direct_rows);

/* Fault injection for testing the bounded-wait error path: while enabled, the first global
 * layer's split-K decode attention (batches above 96 rows on the tensor-core path, above 8 on
 * the CUDA-core path) leaves one stage of its page ring unfilled -- no copy is issued for it --
 * so the consumer warps' bounded wait runs out after about a second.  The frame's kernels all
 * finish, the step returns non-zero with "wait timed out (code 7)", and the streams in that
 * frame keep their host-side positions but hold undefined device state (re-initialise them).
 * Off by default; the engine keeps stepping normally once it is disabled again. */
int mossgpu_debug_inject_wait_timeout(mossgpu_engine *e, int enable);

/* Same as mossgpu_debug_matrix_bytes for the tensor-core tile copy of the matrix. */
int mossgpu_debug_matrix_tile_bytes(mossgpu_engine *e, const char *name, uint8_t *out, size_t out_bytes);

/* Per-kernel device timing, measured with CUDA events recorded between the kernels of the
 * captured frame.  enable = 1 clears the totals and starts accumulating; read returns, per
 * kernel class, the summed milliseconds and launch counts (n_kinds = number of classes). */
int mossgpu_kernel_profile(mossgpu_engine *e, int enable);
int mossgpu_kernel_profile_read(mossgpu_engine *e, float *total_ms, int *launches, int max_kinds, int *n_kinds);
const char *mossgpu_kernel_name(int kind);

/* ---- standalone kernel-level ops (no engine handle; all pointers are DEVICE pointers) ----
 *
 * mossgpu_attention_decode_paged: decode attention of one layer over an fp16 paged KV cache
 * -- the engine's split-K flash-decode, with the reference's attention semantics
 * (llm.cpp:189-228: scores q.k / 8, max-subtracted softmax, weighted sum of v):
 *   q          [R][768] fp32 queries (RoPE already applied)
 *   kv_layer   one layer's pages, fp16 [n_pages][2 (k, v)][12 heads][16 positions][64]
 *   page_table [slots][pages_per_stream] int32; row r reads pages of slot row_slot[r]
 *   row_pos    [R] int32; row r attends to positions 0..row_pos[r]
 *   out        [R][768] fp32
 *   workspace  >= mossgpu_attention_workspace_bytes(R) bytes, 16-byte aligned, any contents
 * cuda_stream is a cudaStream_t (NULL = legacy default stream); the call only enqueues work.
 * Errors: non-zero return, message from mossgpu_op_last_error() (per thread). */
size_t mossgpu_attention_workspace_bytes(int R);
int mossgpu_attention_decode_paged(const float *q, const void *kv_layer, const int32_t *page_table,
                                   int pages_per_stream, const int32_t *row_slot, const int32_t *row_pos, int R,
                                   float *out, void *workspace, size_t workspace_bytes, void *cuda_stream);
const char *mossgpu_op_last_error(void);

/* Device status of the standalone ops on the calling thread's current device.  Every kernel
 * wait in these ops is bounded (about a second); a wait that runs out ends its kernel early,
 * leaves `out` incomplete, and records a code here instead of hanging the GPU: 7 = a consumer
 * warp waited for a KV page, 8 = the page producer waited for a free ring stage.  The op's
 * own return value cannot report it, because the call only enqueues work.  Call this after
 * the op's stream has been synchronised: *code = 0 when no wait ran out, else the first code
 * recorded since the last read (the status is then cleared).  Returns non-zero on a CUDA
 * error.  No counterpart in the reference (its CPU attention has no waits). */
int mossgpu_op_device_status(int *code);

/* mossgpu_attention_decode_paged_noalloc: the same attention for callers that cannot
 * allocate device memory when they run it -- for example a real-time audio callback in a
 * plugin host, where cudaMalloc/cudaFree may block for milliseconds (cudaFree synchronises
 * the device), or a program whose device memory belongs to another allocator.  It takes no
 * workspace and allocates nothing: its scratch (1,120,960 bytes, about 1.07 MiB) is a fixed
 * array that the library places on every GPU that loads it, kept until the process exits.
 *   - R must be <= 256 rows; larger batches are rejected with an error (use the workspace
 *     entry point above).
 *   - The first call on each device does a one-time set-up with the device current: it looks
 *     up that array's device address and opts the kernel into its shared memory.  Under CUDA
 *     lazy loading that set-up may also load the library's kernels onto the device, which can
 *     block and allocate.  So make the first call on each device a warm-up call outside the
 *     real-time or no-allocation context, and before any CUDA stream capture.
 *   - All calls on a device share the one array.  Each call clears the parts that must start
 *     at zero, but two calls whose kernels overlap on the GPU (different streams, or other
 *     host threads) race on it: serialise them on one stream.
 * Arguments, results and errors are those of mossgpu_attention_decode_paged.  This entry
 * point has no counterpart in the reference (its CPU attention needs no scratch). */
int mossgpu_attention_decode_paged_noalloc(const float *q, const void *kv_layer, const int32_t *page_table,
                                           int pages_per_stream, const int32_t *row_slot, const int32_t *row_pos,
                                           int R, float *out, void *cuda_stream);

/* ---- the audio codec decoder (codes -> 48 kHz interleaved stereo samples) ----
 *
 * Replaces moss::AudioDecoder (reference csrc/include/moss/decoder.h:16-79,
 * csrc/src/decoder.cpp) with a batched device decoder.  One codec holds up to max_streams
 * "codec streams"; each is one utterance's streaming state as AudioDecoder keeps it (the
 * RoPE offset of each of the 4 stages and the last 500 / 800 / 1200 / 1600 K and V rows of
 * each of their 12 layers).  Codes are laid out [16][frames] per stream (decoder.h:23, the
 * codebook index major), each in [0, 1024); samples are fp32, frames * 7680 per stream
 * (samples_per_frame: 32 rows x 240 of the last stage, interleaved L, R at 48 kHz).
 * The decoder file is the reference's .moss export with f16 matrices (decoder_f16.moss,
 * tools/export_decoder.py --dtype f16); other matrix types are rejected at create.
 * Arithmetic: the reference computes in fp32 with fp16 matrices; here the products run on
 * the tensor cores with each fp32 operand split into fp16 hi + lo (~22 significant bits)
 * and fp32 accumulation, so results agree with the reference's to float rounding, not bit for
 * bit.  The split needs every activation below 65504 in magnitude: a larger one (or a NaN)
 * makes the host entry points fail and is reported by mossgpu_codec_status; the streams of
 * that call must then be reset.  Conventions as above: 0 on success, the message from
 * mossgpu_codec_last_error. */
typedef struct mossgpu_codec mossgpu_codec;

/* AudioDecoder(threads) + load (decoder.cpp:26-71).  max_batch_frames bounds the frames one
 * call decodes over all its streams (streams x frames); it sizes the activation buffers. */
mossgpu_codec *mossgpu_codec_create(const char *decoder_path, int device_id, int max_streams, int max_batch_frames,
                                    char *err, int errlen);
void mossgpu_codec_destroy(mossgpu_codec *c);
const char *mossgpu_codec_last_error(mossgpu_codec *c);
int mossgpu_codec_samples_per_frame(mossgpu_codec *c);
/* Kernel launches one decode call enqueues (whatever its batch). */
int mossgpu_codec_launches_per_call(mossgpu_codec *c);
size_t mossgpu_codec_device_bytes(mossgpu_codec *c);
/* The CUDA stream (cudaStream_t; NULL = legacy default) every later call enqueues on. */
int mossgpu_codec_set_cuda_stream(mossgpu_codec *c, void *cuda_stream);
/* Per-kernel-class device time: while enabled, each launch is bracketed by CUDA events (which
 * add a gap per launch); profile_read synchronises, writes the milliseconds and launch count of
 * each class since the last read (max_kinds >= 7) and the class count to *n_kinds.  Class
 * names: mossgpu_codec_kernel_name. */
int mossgpu_codec_profile(mossgpu_codec *c, int enable);
int mossgpu_codec_profile_read(mossgpu_codec *c, float *total_ms, int *launches, int max_kinds, int *n_kinds);
const char *mossgpu_codec_kernel_name(int kind);
/* A codec stream in the clean state; close frees its slot. */
int mossgpu_codec_open(mossgpu_codec *c, int *stream_id);
int mossgpu_codec_close(mossgpu_codec *c, int stream_id);
/* AudioDecoder::reset_stream (decoder.cpp:105-114): back to the clean state. */
int mossgpu_codec_reset(mossgpu_codec *c, int stream_id);
/* AudioDecoder::decode_chunk (decoder.cpp:211-225): codes [16][frames] -> out
 * [frames * samples_per_frame]; *out_n = samples written.  Chunks of one stream must come in
 * order; the call returns when the samples are in `out`. */
int mossgpu_codec_decode_chunk(mossgpu_codec *c, int stream_id, const int32_t *codes, int frames, float *out,
                               size_t out_cap, int *out_n);
/* decode_chunk for n distinct streams at once, each `frames` frames: codes [n][16][frames],
 * out [n][frames * samples_per_frame]; each stream ends as after its own decode_chunk. */
int mossgpu_codec_decode_batch(mossgpu_codec *c, const int32_t *stream_ids, int n, const int32_t *codes, int frames,
                               float *out, size_t out_cap);
/* The same with DEVICE codes and output; only enqueues work on the codec's stream.  A code
 * outside [0, 1024) is clamped here (the host entry points reject it). */
int mossgpu_codec_decode_batch_device(mossgpu_codec *c, const int32_t *stream_ids, int n, const int32_t *codes_dev,
                                      int frames, float *out_dev);
/* AudioDecoder::decode (decoder.cpp:254-280): a whole utterance, codes [16][frames], from a
 * clean state, leaving every codec stream untouched. */
int mossgpu_codec_decode(mossgpu_codec *c, const int32_t *codes, int frames, float *out, size_t out_cap, int *out_n);
/* Synchronise the codec's stream; *code = 1 when an activation of a call since the last read
 * left the fp16 range (then cleared), else 0.  The device entry point's only error report. */
int mossgpu_codec_status(mossgpu_codec *c, int *code);

#ifdef __cplusplus
}
#endif
#endif
