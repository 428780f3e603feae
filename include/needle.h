/*
 * needle.h — C ABI of the B200 Needle-3 engine (libneedle_b200.so).
 *
 * Part 1 mirrors the Needle-3 surface of bynds/needle-rs
 * (crates/needle-c/include/needle.h:360-487, crates/needle-c/src/v3.rs:63-382,
 * crates/needle-c/src/lib.rs:27-40, :118): same symbol names, argument meaning,
 * ownership and error behaviour, so a caller of the reference's C library can
 * link this one instead. Every call clears the thread-local last error first;
 * failures return NULL / false / 0 and set it.
 *
 * Part 2 is an extension with no counterpart in the reference: token-level
 * sessions and batches (what the reference exposes only inside Rust as
 * V3Model::prefill / decode_step and V3Cache), used for multi-session serving.
 *
 * Part 3 exposes single kernels with device pointers for callers that manage
 * their own memory and streams (tests, benchmarks, other runtimes).
 *
 * Device: a handle binds to the CUDA device that is current when it is loaded.
 * One handle may be used from several threads; calls on one handle are
 * serialised internally.
 */
#ifndef NEEDLE_B200_H
#define NEEDLE_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── Part 1: the reference's Needle 3 surface ─────────────────────────── */

typedef struct NeedleV3Handle NeedleV3Handle;

/* needle.h:370 / v3.rs:63-77. NULL on failure; free with needle_v3_free(). */
NeedleV3Handle *needle_v3_load(const char *cact_path);

/* needle.h:382 / v3.rs:109-128. The `layers`-block rung of the intelligence
 * ladder, sliced at load (v3.rs:656-745); the container's own depth loads it
 * unchanged. NULL for a depth outside 2..num_layers. */
NeedleV3Handle *needle_v3_load_with_depth(const char *cact_path, size_t layers);

/* needle.h:385 / v3.rs:135-138. 0 for NULL. */
size_t needle_v3_num_layers(NeedleV3Handle *handle);

/* needle.h:388 / v3.rs:85-100. */
NeedleV3Handle *needle_v3_load_bytes(const unsigned char *data, size_t len);

/* needle.h:396 / v3.rs:153-164; needle.h:405 / v3.rs:176-187;
 * needle.h:411 / v3.rs:198-211; needle.h:417 / v3.rs:219-250;
 * needle.h:431 / v3.rs:259-281. Text-level calls (V3Engine::generate_with,
 * v3_engine.rs:193-305): chat prompt, the container's SentencePiece tokenizer,
 * greedy or temperature sampling on the GPU engine until </s> or <|im_end|>.
 * run / run_json / run_stream use the defaults (256 new tokens, greedy, f32
 * KV); run_json returns the trimmed <tool_call> payload, "" when there is
 * none. generate with constrain = true masks the logits inside <tool_call>
 * spans to the declared tool names and argument keys (constrained.rs). When
 * the container has no tokenizer record they return NULL and set the last
 * error. */
char *needle_v3_run(NeedleV3Handle *handle, const char *query, const char *tools_json);
char *needle_v3_run_json(NeedleV3Handle *handle, const char *query, const char *tools_json);
char *needle_v3_reasoning(NeedleV3Handle *handle, const char *text);
char *needle_v3_generate(NeedleV3Handle *handle, const char *query, const char *tools_json,
                         size_t max_new_tokens, float temperature, uint64_t seed,
                         bool constrain, bool kv_int8);
char *needle_v3_run_stream(NeedleV3Handle *handle, const char *query, const char *tools_json,
                           void (*cb)(const char *piece, void *userdata), void *userdata);

/* needle.h:438 / v3.rs:287-291. */
bool needle_v3_has_confidence(NeedleV3Handle *handle);

/* needle.h:452 / v3.rs:307-334. The confidence head over the chat prompt
 * plus `completion` (v3_engine.rs:351-368): a prefill on the GPU engine that
 * captures the per-layer cells, the head's two poolings and projection on the
 * GPU, the sigmoid of its logit in *out. False with the last error set when
 * the container exports no confidence head (or no tokenizer). */
bool needle_v3_confidence_for(NeedleV3Handle *handle, const char *query, const char *tools_json,
                              const char *completion, float *out);

/* needle.h:464 / v3.rs:350-362 (config.rs:234-272). */
size_t needle_v3_kv_bytes(NeedleV3Handle *handle, size_t seq_len, bool kv_int8);

/* needle.h:467 / v3.rs:369-373. */
size_t needle_v3_max_seq_len(NeedleV3Handle *handle);

/* needle.h:470 / v3.rs:378-382. Safe with NULL. */
void needle_v3_free(NeedleV3Handle *handle);

/* lib.rs:118. Safe with NULL. */
void needle_free_str(char *s);

/* needle.h:479-487 / lib.rs:27-40. Borrowed; valid until the next needle_*
 * call on this thread. */
const char *needle_last_error(void);

/* ── Part 2: token-level sessions and batches (extension) ─────────────── */

typedef struct NeedleV3Session NeedleV3Session;
typedef struct NeedleV3Batch NeedleV3Batch;

/* needle_v3_load_with_depth from a container already in memory
 * (V3Engine::from_bytes_with_depth, v3_engine.rs:140-143). */
NeedleV3Handle *needle_v3_load_bytes_with_depth(const unsigned char *data, size_t len, size_t layers);

/* A per-generation KV cache on the device (V3Cache::with_precision,
 * cache.rs:177-238): `hint` sizes the first allocation, rings grow on demand. */
NeedleV3Session *needle_v3_session_new(NeedleV3Handle *handle, size_t hint, bool kv_int8);
void needle_v3_session_free(NeedleV3Session *session);
size_t needle_v3_session_pos(NeedleV3Session *session);
/* Device bytes the session's cache holds (V3Cache::bytes, cache.rs:255-268). */
size_t needle_v3_session_bytes(NeedleV3Session *session);
size_t needle_v3_session_slots(NeedleV3Session *session, size_t layer);

/* Host copy of one layer's KV ring, in the reference's layout (V3Cache::kv,
 * cache.rs:382-393; ring slot of position p is p % slots): k [slots][kv_heads]
 * [qk] and v [slots][kv_heads][v_head] as floats (f32 session) or int8 codes
 * (int8 session), plus for int8 the f32 scales k_scale / v_scale
 * [slots][kv_heads]; slots no position has reached yet read as zero codes
 * with scale 1, the reference's initial state. Any of k, v may be NULL (with
 * its scale for int8). Synchronous. */
bool needle_v3_session_kv(NeedleV3Session *session, size_t layer, void *k, void *v, float *k_scale,
                          float *v_scale);

/* Prefill a fresh session with `n` token ids (V3Model::prefill, model.rs:512).
 * Writes the last position's logits (logit_rows floats) when `logits` is not
 * NULL. Host buffers. */
bool needle_v3_prefill(NeedleV3Handle *handle, NeedleV3Session *session, const uint32_t *ids,
                       size_t n, float *logits);

/* One decode step (V3Model::decode_step, model.rs:150). Host buffers. */
bool needle_v3_decode_step(NeedleV3Handle *handle, NeedleV3Session *session, uint32_t token,
                           float *logits);

/* Batched forms over `n` distinct sessions that share one KV precision.
 * prefill: ids concatenated, lens[i] tokens for session i; last_logits
 * [n][logit_rows] and picks [n] (greedy argmax, v3_engine.rs:410-420) may be
 * NULL. decode: one token per session. Host buffers. */
bool needle_v3_prefill_batch(NeedleV3Handle *handle, NeedleV3Session *const *sessions,
                             const uint32_t *ids, const size_t *lens, size_t n,
                             float *last_logits, uint32_t *picks);
bool needle_v3_decode_batch(NeedleV3Handle *handle, NeedleV3Session *const *sessions,
                            const uint32_t *tokens, size_t n, float *logits, uint32_t *picks);

/* Greedy or sampled generation from token ids (V3Engine::generate_with loop,
 * v3_engine.rs:193-315, without the text layers): prefill, then up to
 * max_new_tokens steps; temperature <= 0 is greedy, else SplitMix64 sampling
 * (v3_engine.rs:422-464). Stops at `eos_id` unless it is UINT32_MAX. Writes the
 * generated ids to out_ids (capacity max_new_tokens) and returns their count;
 * (size_t)-1 on failure. */
size_t needle_v3_generate_ids(NeedleV3Handle *handle, const uint32_t *prompt, size_t n,
                              size_t max_new_tokens, float temperature, uint64_t seed,
                              bool kv_int8, uint32_t eos_id, uint32_t *out_ids);

/* One temperature draw from `n` logits (host) as generate_with takes it
 * (sample, v3_engine.rs:422-443): softmax(logits / temperature) weights summed
 * in f64, target = next_f64() * sum from the SplitMix64 generator whose state
 * is *rng_state (v3_engine.rs:446-464; seed it with the generation seed), which
 * advances by one draw. For callers that sample the logits of the batched
 * calls themselves. UINT32_MAX with the last error set for NULL arguments,
 * n == 0 or temperature <= 0. Host only. */
uint32_t needle_v3_sample(const float *logits, size_t n, float temperature, uint64_t *rng_state);

/* A fixed set of sessions decoded together with device-resident tokens; one
 * step is captured once as a CUDA graph and replayed. */
NeedleV3Batch *needle_v3_batch_new(NeedleV3Handle *handle, NeedleV3Session *const *sessions,
                                   size_t n);
void needle_v3_batch_free(NeedleV3Batch *batch);
/* Device pointers to the batch's token buffers: `tokens` [n] is read by the
 * next step, `next` [n] receives its greedy picks. */
uint32_t *needle_v3_batch_tokens(NeedleV3Batch *batch);
uint32_t *needle_v3_batch_next(NeedleV3Batch *batch);
/* One step on `stream` (a cudaStream_t, NULL = the handle's stream).
 * d_logits (device, [n][logit_rows]) may be NULL. Asynchronous. */
bool needle_v3_batch_step(NeedleV3Batch *batch, float *d_logits, void *stream, bool use_graph);
/* Copy `next` into `tokens` on `stream` (feed the greedy picks back). */
bool needle_v3_batch_feed_next(NeedleV3Batch *batch, void *stream);
/* Synchronous host copies: set the tokens of the next step from host memory,
 * or read the picks of the last step into host memory ([n] each). */
bool needle_v3_batch_set_tokens(NeedleV3Batch *batch, const uint32_t *tokens);
bool needle_v3_batch_get_next(NeedleV3Batch *batch, uint32_t *next);

/* One eager decode step of the batch with CUDA events between kernel groups
 * (advances every session by one position like needle_v3_batch_step). Writes
 * milliseconds per group to ms[12] — engram, embed, layer_pre, qkvg
 * projection, qkv_post, attention, attention finish, out projection,
 * layer_post, final norm, LM head, bookkeeping — and this library's kernel
 * launch count for the step to *launches. Synchronous. */
bool needle_v3_batch_profile(NeedleV3Batch *batch, float *ms, int *launches);

/* The container tokenizer on its own, from a RAW tokenizer blob
 * (sp_tokenizer.rs:116-414); host only, needs no GPU. encode writes
 * min(count, cap) ids and returns the count ((size_t)-1 on error); decode
 * returns a string to free with needle_free_str. */
typedef struct NeedleTokenizer NeedleTokenizer;
NeedleTokenizer *needle_tokenizer_new(const unsigned char *blob, size_t len);
void needle_tokenizer_free(NeedleTokenizer *tokenizer);
size_t needle_tokenizer_encode(NeedleTokenizer *tokenizer, const char *text, uint32_t *out, size_t cap);
char *needle_tokenizer_decode(NeedleTokenizer *tokenizer, const uint32_t *ids, size_t n);
/* The grammar mask (0 or -1e9 per id, `vocab` entries) that constrained
 * decoding adds after the tool-call bytes out_bytes[0..n) have been written,
 * for the tools declared in tools_json (ConstrainedDecoder::logit_mask,
 * constrained.rs:431-461; unique_keys as with_unique_arg_keys). */
bool needle_tokenizer_tool_mask(NeedleTokenizer *tokenizer, const char *tools_json,
                                const unsigned char *out_bytes, size_t n, bool unique_keys,
                                float *mask, size_t vocab);

/* Geometry: vocab, out_vocab, d_model, heads, kv_heads, layers, qk, v_head,
 * max_seq, hada_n, lanes, window, conv_taps, logit_rows (14 int64). */
bool needle_v3_geometry(NeedleV3Handle *handle, int64_t *out14);
/* CUDA device a handle is bound to; -1 for NULL. */
int needle_v3_device(NeedleV3Handle *handle);

/* ── Part 3: single kernels on device pointers ─────────────────────────── */

/* CQ projection y[m, row0 + r] = W[row0 + r] . xh[m] for m < M, r < nrows,
 * reading one `.cact` CQ blob in place: `packed` = rows*in_pad*bits/8 bytes,
 * `norms` = rows*(in_pad/128) FP16 (cq.rs:181-238). `levels` = the 2^bits
 * codebook entries (host). xh is the rotated input (prepare_input, cq.rs:264),
 * [M][ldx] f32. path: 0 auto, 1 GEMV (M <= 8), 2 tiled SIMT GEMM, 3 tensor-core
 * GEMM (tcgen05; chosen by path 0 for M > 8; uses stream-ordered scratch of
 * 4*(M + nrows)*in_pad + 4*M*in_pad/128 bytes); for M <= 8, 4 the SIMT GEMV kernels and 5
 * the tensor-core GEMV (mma.sync; codebooks whose levels are f16 values). Replaces
 * CqWeight::matvec_rows_prepared / matmul_rows_prepared (cq.rs:301, :446). */
int nd_cq_project(const void *packed, const void *norms, int rows, int in_feat, int bits,
                  const float *levels, const float *xh, int ldx, int M, float *y, int ldy,
                  int row0, int nrows, int path, void *stream);

/* Several CQ projections of the same input as one: matrix i (packed[i],
 * norms[i], rows[i] rows, laid out as for nd_cq_project; every matrix with the
 * same in_feat, bits and levels; 1 <= count <= 4) fills columns [r_i, r_i +
 * rows[i]) of y [M][ldy], r_i the rows of the matrices before it: one tensor-
 * core launch for all of them (path 0 or 3 with M > 8), as the engine runs a
 * block's q, k, v and gate projections (v3/model.rs:260-262, :309). Other
 * paths and the scratch are those of nd_cq_project over all the rows. */
int nd_cq_project_grouped(int count, const void *const *packed, const void *const *norms, const int *rows,
                          int in_feat, int bits, const float *levels, const float *xh, int ldx, int M,
                          float *y, int ldy, int path, void *stream);

/* prepare_input (cq.rs:264-274): zero-pad x [M][in_feat] to in_pad and apply
 * the normalised Walsh-Hadamard transform to every group of 128. */
int nd_cq_prepare(const float *x, int M, int in_feat, float *xh, int ld_out, void *stream);

/* quant_into (cache.rs:100-106) over `rows` vectors of `dim` <= 64 floats:
 * int8 codes and one f32 scale per vector, bit-exact with the reference. */
int nd_kv_quant(const float *x, int rows, int dim, int8_t *q, float *scales, void *stream);

/* attend_step (attention.rs:300-377) for B independent sessions. Rings use the
 * reference layout k [slots][kv_heads][qk], v [slots][kv_heads][vh], scales
 * [slots][kv_heads] (int8 only), session b at b*slots*...; lo/hi are device
 * int arrays [B] of the inclusive logical range; q [B][heads][qk] (already
 * fake-quantised for int8), out [B][heads][vh]. */
int nd_attend_step(const float *q, const void *k, const void *v, const float *ks, const float *vs,
                   int int8, int slots, const int *lo, const int *hi, int B, int heads, int kv_heads,
                   int qk, int vh, float *out, void *stream);

/* Allocation-free nd_attend_step. No counterpart in the reference (its CPU
 * code never allocates device memory). For callers that cannot allocate device
 * memory — a runtime that reserved the GPU's memory for its own pool, or a
 * latency-critical path that must not make an allocation call — the split
 * partials use a fixed 4 MiB device array compiled into this library (held by
 * every GPU that loads the library until exit) instead of per-call scratch.
 * Requests needing more than 1048576 floats of partials even with a single
 * position split (B * heads * (vh + 2) floats) fail with cudaErrorInvalidValue
 * and a message in nd_last_error(). The first call on each device (and the
 * first after that device's context was reset) looks up the array's device
 * address; make that call before any stream capture.
 * All calls on a device share the array and keep the last call's contents:
 * calls whose kernels overlap on the GPU race and must be serialised.
 * Arguments and result as nd_attend_step. */
int nd_attend_step_noalloc(const float *q, const void *k, const void *v, const float *ks,
                           const float *vs, int int8, int slots, const int *lo, const int *hi,
                           int B, int heads, int kv_heads, int qk, int vh, float *out, void *stream);

/* Returns the cudaError_t of the last nd_* failure on this thread as text. */
const char *nd_last_error(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* NEEDLE_B200_H */
