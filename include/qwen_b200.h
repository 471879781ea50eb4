/*
 * qwen_b200.h -- C ABI of the B200 (sm_100a) Qwen2 token-loop library.
 *
 * The library replaces the hot path of the reference crate `llm_inference`
 * (pshevskiy/llm_inference_edu): the linear kernels, INT8 scheme, RoPE,
 * elementwise ops, KV-cached decode step, prefill and the greedy generation
 * loop.  Each entry point below names the reference interface it replaces
 * (path:line within that project).
 *
 * Conventions, following the reference's native bridge
 * (apple/cpu_bridge/include/llm_cpu_bridge.h:8-13):
 *   - every function returns a uint32_t status (QB_OK = 0);
 *   - the caller owns every buffer; no foreign pointer is retained after a
 *     call returns (model tensors are copied to the device);
 *   - validate-before-write: an admission error leaves every output
 *     untouched (src/lib.rs:46-50);
 *   - models, sessions and generation states are opaque uint64_t handles,
 *     never reused.
 * Pointers documented as DEVICE must be device memory on the current CUDA
 * device; HOST pointers are ordinary host memory.  `stream` is a
 * cudaStream_t (NULL = the legacy default stream).
 * Token ids are uint32_t (the bridge's id type, llm_cpu_bridge.h:32).
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define QB_ABI_VERSION 1u

/* Status codes.  1..25 mirror the reference error enums LinearError
 * (src/lib.rs:22-30), QuantError (src/quantization.rs:3-25), OpError
 * (src/ops.rs:5-33), RopeError (src/rope.rs:3-20) and CacheError
 * (src/kv_cache.rs:46-62); 26.. are the generation/bridge states
 * (src/generation.rs:83-92, llm_cpu_bridge.h:14-18) and device errors. */
enum {
    QB_OK = 0,
    QB_ZERO_DIMENSION = 1,
    QB_DIMENSION_OVERFLOW = 2,
    QB_INVALID_LENGTH = 3,
    QB_INVALID_GROUP_SIZE = 4,
    QB_INVALID_SHAPE = 5,
    QB_NONFINITE_WEIGHT = 6,
    QB_UNREPRESENTABLE_SCALE = 7,
    QB_ALLOCATION = 8,
    QB_INVALID_TOKEN = 9,
    QB_INVALID_EPSILON = 10,
    QB_NONFINITE = 11,
    QB_ALL_MASKED = 12,
    QB_ODD_HEAD_DIMENSION = 13,
    QB_POSITION_OVERFLOW = 14,
    QB_POSITION_OUT_OF_RANGE = 15,
    QB_INVALID_BASE = 16,
    QB_INVALID_ANGLE = 17,
    QB_INVALID_CAPACITY = 18,
    QB_RESOURCE_BUDGET = 19,
    QB_INVALID_OUTPUT_LENGTH = 20,
    QB_EMPTY_INPUT = 21,
    QB_NOT_EMPTY = 22,
    QB_FULL = 23,
    QB_INVALID_STATE = 24,
    QB_INVALID_CONFIG = 25,
    QB_INVALID_HANDLE = 26,
    QB_INVALID_PARAMETERS = 27,
    QB_NOT_STARTED = 28,
    QB_ALREADY_STARTED = 29,
    QB_CANCELLED = 30,
    QB_EMPTY_LOGITS = 31,
    QB_CUDA_ERROR = 32,
    QB_DEVICE_TIMEOUT = 33,
    QB_CONTEXT_LIMIT = 34,
    QB_TRACE_LIMIT = 35,
    QB_EMPTY_PROMPT = 36,
    QB_OUTPUT_LIMIT = 37,
    QB_INVALID_LAYER_COUNT = 38,
    QB_UNSUPPORTED = 39,
    /* LoadError (src/weights.rs:72-88) variants without an earlier code;
     * its InvalidShape, NonFinite, DimensionOverflow, ResourceBudget and
     * Allocation map to 5, 11, 2, 19 and 8. */
    QB_LOAD_FORMAT = 40,
    QB_LOAD_UNSUPPORTED_CONFIG = 41,
    QB_LOAD_MISSING_TENSOR = 42,
    QB_LOAD_UNEXPECTED_TENSOR = 43,
    QB_LOAD_INVALID_DTYPE = 44,
    /* TokenizerError (src/tokenizer.rs:27-35) */
    QB_TOKENIZER_JSON = 45,
    QB_TOKENIZER_ENCODING = 46,
    QB_TOKENIZER_UNSUPPORTED_ASSETS = 47,
    QB_TOKENIZER_EMPTY_MESSAGES = 48,
    QB_TOKENIZER_INVALID_TOKEN = 49,
    QB_TOKENIZER_INVALID_STREAM = 50
};

/* Detail of the calling thread's last error: which buffer (argument order),
 * expected and actual lengths, and the offending index or id -- the payload
 * of the reference's InvalidLength/InvalidToken/NonFinite variants. */
typedef struct {
    size_t buffer;
    size_t expected;
    size_t actual;
    size_t index;
} qb_detail;

uint32_t qb_abi_version(void);
const char *qb_status_name(uint32_t status);
void qb_last_detail(qb_detail *out);
/* The last CUDA runtime error number seen by this thread (0 if none). */
int qb_last_cuda_error(void);

/* ------------------------------------------------------------------ */
/* Linear kernels (DEVICE buffers; lengths are element counts)         */
/* ------------------------------------------------------------------ */

/* Y[t,o] = sum_i X[t,i] * W[o,i], all row-major FP32, FP32 accumulation in
 * increasing i (bit-identical to the crate).  Replaces `linear`,
 * src/lib.rs:51-73 (admission src/lib.rs:76-111: zero dimension, product
 * overflow, then exact lengths of x, w, y). */
uint32_t qb_linear_f32(const float *x, size_t x_len, const float *w, size_t w_len, float *y,
                       size_t y_len, size_t tokens, size_t input_dim, size_t output_dim,
                       void *stream);
/* Same contract as qb_linear_f32, in the four-lane order of dot_lanes4
 * (lanes i % 4, ((s0 + s1) + s2) + s3, then the tail; bit-identical to the
 * crate).  Replaces `linear_lanes4`, src/kernels.rs:10-46 (the tied LM-head
 * kernel). */
uint32_t qb_linear_lanes4_f32(const float *x, size_t x_len, const float *w, size_t w_len,
                              float *y, size_t y_len, size_t tokens, size_t input_dim,
                              size_t output_dim, void *stream);
/* BF16 weights (uint16 bit patterns, value = bits << 16 as in
 * src/weights.rs:250-251), FP32 activations and accumulation in `linear`'s
 * order. */
uint32_t qb_linear_bf16(const float *x, size_t x_len, const uint16_t *w, size_t w_len, float *y,
                        size_t y_len, size_t tokens, size_t input_dim, size_t output_dim,
                        void *stream);

/* ------------------------------------------------------------------ */
/* INT8 weight-only scheme                                             */
/* ------------------------------------------------------------------ */

/* Quantizes W[output_dim, input_dim] (DEVICE FP32) into `values`
 * [output_dim, input_dim] int8 and `scales` [output_dim, groups_per_row]
 * FP32, groups_per_row = ceil(input_dim / group_size), bit-exact with
 * GroupwiseInt8::quantize, src/quantization.rs:55-116 (encode :36-40).
 * group_size is 1..=256 (the reference's range) or equal to input_dim
 * (one scale per output row).  Synchronizes `stream`: non-finite weights
 * and unrepresentable scales are found before any output is written. */
uint32_t qb_quantize_int8(const float *w, size_t w_len, size_t output_dim, size_t input_dim,
                          size_t group_size, int8_t *values, float *scales, void *stream);
/* y = f32(q) * scale; replaces GroupwiseInt8::dequantize,
 * src/quantization.rs:141-166. */
uint32_t qb_dequantize_int8(const int8_t *values, const float *scales, size_t output_dim,
                            size_t input_dim, size_t group_size, float *y, size_t y_len,
                            void *stream);
/* Fused dequantizing linear: y[t,o] = sum_i x[t,i] * (f32(q[o,i]) * s[o,g(i)]),
 * summed in increasing i (bit-identical to the crate).  Replaces
 * linear_int8, src/quantization.rs:168-215. */
uint32_t qb_linear_int8(const float *x, size_t x_len, const int8_t *values, const float *scales,
                        size_t output_dim, size_t input_dim, size_t group_size, float *y,
                        size_t y_len, size_t tokens, void *stream);
/* The same product in the four-lane order (lanes i % 4 over the first
 * input_dim - input_dim % 4 elements, ((s0 + s1) + s2) + s3, then the tail
 * in order; bit-identical to the crate).  Replaces linear_int8_lanes4,
 * src/quantization.rs:218-281. */
uint32_t qb_linear_int8_lanes4(const float *x, size_t x_len, const int8_t *values,
                               const float *scales, size_t output_dim, size_t input_dim,
                               size_t group_size, float *y, size_t y_len, size_t tokens,
                               void *stream);

/* ------------------------------------------------------------------ */
/* Elementwise ops (DEVICE buffers; ids are HOST)                      */
/* Checks that read values (finiteness, masks) synchronize `stream`    */
/* before any output is written.                                       */
/* ------------------------------------------------------------------ */

/* Replaces `embedding`, src/ops.rs:67-91. */
uint32_t qb_embedding(const uint32_t *ids, size_t count, const float *table, size_t table_len,
                      float *y, size_t y_len, size_t vocab_size, size_t width, void *stream);
/* Replaces `residual_add`, src/ops.rs:97-107. */
uint32_t qb_residual_add(const float *x, size_t x_len, const float *residual, size_t residual_len,
                         float *y, size_t y_len, void *stream);
/* Scaled RMSNorm; replaces `rmsnorm`, src/ops.rs:119-152. */
uint32_t qb_rmsnorm(const float *x, size_t x_len, const float *weight, size_t weight_len, float *y,
                    size_t y_len, size_t rows, size_t width, float epsilon, void *stream);
/* Replaces `silu`, src/ops.rs:158-173. */
uint32_t qb_silu(const float *x, size_t x_len, float *y, size_t y_len, void *stream);
/* Row softmax; `mask` (DEVICE uint8, nullable) selects masked_softmax.
 * Replaces `softmax` / `masked_softmax`, src/ops.rs:179-257. */
uint32_t qb_softmax(const float *logits, size_t logits_len, const uint8_t *mask, size_t mask_len,
                    float *y, size_t y_len, size_t rows, size_t width, void *stream);
/* Split-half RoPE at absolute positions; replaces `rope`,
 * src/rope.rs:38-105.  Angles come from a host table computed with the
 * C library's powf/sinf/cosf, the functions the reference calls. */
uint32_t qb_rope(const float *x, size_t x_len, float *y, size_t y_len, size_t tokens,
                 size_t heads, size_t head_dim, size_t start_position, float base, void *stream);

/* qb_rope without any allocation.  No counterpart in the reference: it is
 * qb_rope (same arguments, checks, results and error codes) for callers
 * that must not allocate -- a serving process that has already divided
 * device memory between weights and KV pages, where a late cudaMalloc can
 * fail or fragment memory another allocator owns, and latency-bound code
 * with work in flight on other streams, which cudaFree would wait for.
 * It uses no cudaMalloc/cudaFree, no heap and no allocating library call:
 * its device scratch (a flag word and the angle table) is one fixed static
 * array of QB_ROPE_STATIC_SCRATCH_BYTES per device inside this library, and
 * the host stages the table through a 16 KiB stack buffer.
 *  - Limit: tokens * head_dim <= QB_ROPE_STATIC_MAX_TABLE.  A larger call
 *    returns QB_RESOURCE_BUDGET before any device work, with qb_last_detail
 *    expected = the limit and actual = tokens * head_dim.
 *  - Like qb_rope, the call synchronizes `stream` before it returns.
 *  - The first call on each device looks up the array's address with
 *    cudaGetSymbolAddress (not a stream operation); make that first call
 *    before any stream capture begins on that device.
 *  - Each call resets the flag word itself; the angle table needs no
 *    starting value (each call writes all of it before the kernel reads it).
 *  - All calls on one device share the one array, so calls that overlap in
 *    time (several host threads) race and can return wrong results:
 *    serialize them.  As with qb_rope, `stream` is synchronized before the
 *    call returns, so consecutive calls from one thread never overlap. */
#define QB_ROPE_STATIC_SCRATCH_BYTES 262144u
#define QB_ROPE_STATIC_MAX_TABLE 65472u /* (262144 - 256) / 4 floats */
uint32_t qb_rope_static(const float *x, size_t x_len, float *y, size_t y_len, size_t tokens,
                        size_t heads, size_t head_dim, size_t start_position, float base,
                        void *stream);

/* ------------------------------------------------------------------ */
/* Model: ModelConfig / Decoder (src/model.rs:12-25,191-273)           */
/* ------------------------------------------------------------------ */

typedef struct {
    size_t vocab_size, layers, hidden_dim, query_heads, kv_heads, head_dim, ff_dim, max_tokens;
    float rope_base, norm_epsilon;
} qb_model_config;

/* Storage of the seven per-layer linears on the device. */
enum {
    QB_LINEAR_F32 = 0,       /* FP32, the reference's WeightMatrix::Float */
    QB_LINEAR_BF16 = 1,      /* BF16 values */
    QB_LINEAR_INT8_ROW = 2   /* int8 with one FP32 absmax scale per output row */
};
/* Storage of the embedding table (tied LM head) and an untied head. */
enum { QB_TABLE_F32 = 0, QB_TABLE_BF16 = 1 };
/* Host source element type passed to qb_model_set_tensor. */
enum { QB_HOST_F32 = 0, QB_HOST_BF16 = 1 };
/* Tensor ids; HF Qwen2 names in comments (src/model.rs:296-316). */
enum {
    QB_T_EMBEDDING = 0,   /* model.embed_tokens.weight [V,h] */
    QB_T_LM_HEAD = 1,     /* lm_head.weight [V,h]; absent = tied */
    QB_T_FINAL_NORM = 2,  /* model.norm.weight [h] */
    QB_T_ATTN_NORM = 3,   /* input_layernorm.weight [h] */
    QB_T_Q = 4,           /* self_attn.q_proj.weight [h,h] */
    QB_T_K = 5,           /* self_attn.k_proj.weight [kv,h] */
    QB_T_V = 6,           /* self_attn.v_proj.weight [kv,h] */
    QB_T_O = 7,           /* self_attn.o_proj.weight [h,h] */
    QB_T_Q_BIAS = 8,      /* self_attn.q_proj.bias [h] (optional) */
    QB_T_K_BIAS = 9,      /* self_attn.k_proj.bias [kv] (optional) */
    QB_T_V_BIAS = 10,     /* self_attn.v_proj.bias [kv] (optional) */
    QB_T_FFN_NORM = 11,   /* post_attention_layernorm.weight [h] */
    QB_T_GATE = 12,       /* mlp.gate_proj.weight [ff,h] */
    QB_T_UP = 13,         /* mlp.up_proj.weight [ff,h] */
    QB_T_DOWN = 14        /* mlp.down_proj.weight [h,ff] */
};

/* Starts a model on `device` (config admission as Decoder::new,
 * src/model.rs:191-230). */
uint32_t qb_model_create(const qb_model_config *config, uint32_t linear_format,
                         uint32_t table_format, int device, uint64_t *out_model);
/* Copies one HOST tensor to the device (layer = -1 for embedding,
 * lm_head and final_norm).  Lengths and finiteness are checked as in
 * Decoder::new, src/model.rs:232-272. */
uint32_t qb_model_set_tensor(uint64_t model, int64_t layer, uint32_t tensor, uint32_t host_dtype,
                             const void *data, size_t elements);
/* Checks completeness, quantizes INT8 linears on the device and builds the
 * decode layout.  No tensor may be set afterwards. */
uint32_t qb_model_finalize(uint64_t model);
/* Logical stored payload in bytes; replaces Decoder::logical_weight_bytes,
 * src/model.rs:347-385. */
uint32_t qb_model_logical_weight_bytes(uint64_t model, size_t *out);
/* Device copy of one quantized linear (int8 values and scales); for
 * bit-exact checks of the on-device quantization. */
uint32_t qb_model_read_int8(uint64_t model, int64_t layer, uint32_t tensor, int8_t *values,
                            size_t values_len, float *scales, size_t scales_len);
uint32_t qb_model_free(uint64_t model);

/* ------------------------------------------------------------------ */
/* CachedSession (src/kv_cache.rs:156-475)                              */
/* ------------------------------------------------------------------ */

enum { QB_KV_F32 = 0, QB_KV_BF16 = 1 };

typedef struct {
    size_t processed, capacity, logical_bytes, workspace_bytes;
    int32_t valid;
} qb_session_info;

/* CachedSession::new, src/kv_cache.rs:167-200.  `budget_bytes` bounds the
 * logical KV bytes plus workspace (the reference fixes 128 MiB,
 * src/kv_cache.rs:184-190); 0 means unbounded.  The device cache is paged:
 * per layer a K and a V pool of 16-position pages, each page
 * [kv_heads][16][head_dim] (FP32 or BF16), allocated for the whole
 * capacity at creation and reached through the session's page table; the
 * reported byte counts stay the reference's (FP32, unpaged). */
uint32_t qb_session_create(uint64_t model, size_t capacity, uint32_t kv_dtype,
                           size_t budget_bytes, uint64_t *out_session);
/* step_into, src/kv_cache.rs:306-346.  `logits` (HOST, nullable) receives
 * the vocabulary-width logits; `argmax` (HOST, nullable) the greedy id
 * (lowest id on ties, src/sampling.rs:65-70).  Admission errors leave the
 * state and outputs unchanged; execution errors invalidate the session. */
uint32_t qb_session_step(uint64_t session, uint32_t token, float *logits, size_t logits_len,
                         uint32_t *argmax);
/* append_into / prefill_into (require_empty = 1), src/kv_cache.rs:249-294:
 * the whole chunk is admitted first; only the last position's logits are
 * returned. */
uint32_t qb_session_append(uint64_t session, const uint32_t *tokens, size_t count, float *logits,
                           size_t logits_len, uint32_t *argmax, int32_t require_empty);
/* step_profiled, src/kv_cache.rs:309-316: one step as qb_session_step that
 * also records device timestamps (ns, %globaltimer) into `stamps`:
 * [B][grid] times at which each CTA finished each phase, then [B][grid]
 * times at which each CTA held that phase's outputs as the inputs of its
 * next phase (0 where the CTA had no work in it), then the step's start and
 * end, where B = 4 * layers (QKV, attention, gate/up and down phases of
 * every layer).  `*needed` receives the count;
 * a short `stamps` buffer is an admission error (QB_INVALID_LENGTH). */
uint32_t qb_session_step_profiled(uint64_t session, uint32_t token, float *logits,
                                  size_t logits_len, uint32_t *argmax, uint64_t *stamps,
                                  size_t stamps_len, size_t *needed);
/* Fault-path test hook with no counterpart in the reference: one decode
 * step in which CTA 0 withholds its first-layer QKV outputs, so the polls
 * that wait for them run out after `timeout_ns` (1 ns .. 2 s; outside that
 * range: QB_INVALID_PARAMETERS, with qb_last_detail expected = 2e9 and
 * actual = timeout_ns, and nothing runs).  Expected result:
 * QB_DEVICE_TIMEOUT, the session invalidated (as after any execution
 * error) until qb_session_reset; the device stays usable. */
uint32_t qb_session_step_withheld(uint64_t session, uint32_t token, uint64_t timeout_ns);
/* reset, src/kv_cache.rs:225-229. */
uint32_t qb_session_reset(uint64_t session);
uint32_t qb_session_info_get(uint64_t session, qb_session_info *out);
/* Runs `steps` greedy decode steps back to back on the device, each feeding
 * its own argmax to the next, starting from `token`; writes the emitted ids
 * (HOST, `steps` entries).  Equivalent to `steps` rounds of step_into +
 * greedy sample with no stop tokens. */
uint32_t qb_session_decode_greedy(uint64_t session, uint32_t token, size_t steps, uint32_t *ids);
/* The CUDA stream the session launches on (for event timing). */
uint32_t qb_session_stream(uint64_t session, void **stream);
uint32_t qb_session_free(uint64_t session);

/* ------------------------------------------------------------------ */
/* Sampling (src/sampling.rs:5-110)                                     */
/* ------------------------------------------------------------------ */

enum { QB_SAMPLING_GREEDY = 0, QB_SAMPLING_TEMPERATURE = 1 };

/* Sampling::{Greedy, Temperature { temperature, top_k, seed }}
 * (src/sampling.rs:5-12); temperature, top_k and seed are ignored for
 * QB_SAMPLING_GREEDY. */
typedef struct {
    uint32_t kind;
    float temperature;
    uint64_t top_k;
    uint64_t seed;
} qb_sampling;

/* Sampler::new, src/sampling.rs:24-42: QB_INVALID_PARAMETERS for a
 * temperature that is not finite and positive, or top_k = 0.  The
 * generator (ChaCha8, seeded from `seed`) lives on the host; the selection
 * runs on CUDA device `device`. */
uint32_t qb_sampler_create(const qb_sampling *policy, int device, uint64_t *out_sampler);
/* Sampler::validate_vocab, src/sampling.rs:43-49. */
uint32_t qb_sampler_validate_vocab(uint64_t sampler, size_t vocab);
/* Sampler::reset, src/sampling.rs:51-56: the stream restarts from the seed. */
uint32_t qb_sampler_reset(uint64_t sampler);
/* Sampler::sample, src/sampling.rs:57-110, over `count` HOST logits (copied
 * to the device): QB_EMPTY_LOGITS, QB_NONFINITE, QB_INVALID_PARAMETERS
 * (top_k > count) leave the stream where it was. */
uint32_t qb_sampler_sample(uint64_t sampler, const float *logits, size_t count, uint32_t *out_id);
/* The same over DEVICE logits on the sampler's device. */
uint32_t qb_sampler_sample_device(uint64_t sampler, const float *device_logits, size_t count,
                                  uint32_t *out_id);
uint32_t qb_sampler_free(uint64_t sampler);

/* ------------------------------------------------------------------ */
/* GenerationSession (src/generation.rs:98-338)                         */
/* ------------------------------------------------------------------ */

enum { QB_STOP_NONE = 0, QB_STOP_TOKEN = 1, QB_STOP_OUTPUT_LIMIT = 2 };

typedef struct {
    size_t processed, history_len, generated, max_new;
    int32_t stop_reason, valid, logits_ready;
} qb_generation_info;

/* GenerationSession::new, src/generation.rs:111-138. */
uint32_t qb_generation_create(uint64_t model, size_t capacity, const uint32_t *stops,
                              size_t stop_count, size_t max_new, uint32_t kv_dtype,
                              size_t budget_bytes, uint64_t *out_generation);
/* GenerationSession::new with a sampling policy (NULL = greedy): the
 * policy's errors (Sampler::new, validate_vocab against the model's vocab)
 * are QB_INVALID_PARAMETERS.  next_token samples the device logits of the
 * last evaluated token; reset and replay_history restart the stream. */
uint32_t qb_generation_create_sampled(uint64_t model, size_t capacity, const qb_sampling *policy,
                                      const uint32_t *stops, size_t stop_count, size_t max_new,
                                      uint32_t kv_dtype, size_t budget_bytes,
                                      uint64_t *out_generation);
/* start_with_cancel, src/generation.rs:145-170; `cancel` (HOST, nullable)
 * is polled at token boundaries (nonzero = cancelled). */
uint32_t qb_generation_start(uint64_t generation, const uint32_t *prompt, size_t count,
                             const volatile int32_t *cancel);
/* next_token, src/generation.rs:307-337: *has_token = 0 once stopped. */
uint32_t qb_generation_next_token(uint64_t generation, const volatile int32_t *cancel,
                                  uint32_t *token, int32_t *has_token);
/* append_context, src/generation.rs:177-218. */
uint32_t qb_generation_append_context(uint64_t generation, const uint32_t *suffix, size_t count,
                                      size_t max_new, const volatile int32_t *cancel);
/* replay_history, src/generation.rs:222-257. */
uint32_t qb_generation_replay_history(uint64_t generation, const uint32_t *history, size_t count,
                                      size_t max_new, const volatile int32_t *cancel);
/* reset, src/generation.rs:294-301. */
uint32_t qb_generation_reset(uint64_t generation);
uint32_t qb_generation_info_get(uint64_t generation, qb_generation_info *out);
/* history, src/generation.rs:275-277: copies min(len, capacity) ids. */
uint32_t qb_generation_history(uint64_t generation, uint32_t *ids, size_t capacity, size_t *len);
/* prefix_logits, src/generation.rs:281-283: QB_NOT_STARTED when None. */
uint32_t qb_generation_prefix_logits(uint64_t generation, float *logits, size_t logits_len);
uint32_t qb_generation_free(uint64_t generation);

/* ------------------------------------------------------------------ */
/* Batched greedy decode of independent sequences                      */
/* ------------------------------------------------------------------ */
/* No counterpart in the reference, which decodes one sequence per session
 * (src/kv_cache.rs:186-215 is the per-token step each row here repeats).
 * `sequences` rows advance in lockstep, each with its own KV cache of
 * `capacity` positions; every row equals what a CachedSession fed the same
 * tokens would compute (within FP32 reassociation).  The sequences' caches
 * share one page pool per layer (16-position pages; sequence s's page j is
 * pool page j * sequences + s).  Created on the model's device; the model
 * must outlive it. */
typedef struct {
    size_t sequences, capacity, processed;
    int32_t valid;
} qb_batch_info;

uint32_t qb_batch_create(uint64_t model, size_t sequences, size_t capacity, uint32_t kv_dtype,
                         uint64_t *out_batch);
/* prompts [sequences][prompt_len] (HOST); next_ids [sequences] (HOST,
 * nullable) receives each row's greedy id after its last prompt token.
 * QB_NOT_EMPTY unless the batch is empty. */
uint32_t qb_batch_prefill(uint64_t batch, const uint32_t *prompts, size_t prompt_len,
                          uint32_t *next_ids);
/* Feeds tokens [sequences] (HOST), then each row's greedy id, for `steps`
 * steps; ids [steps][sequences] (HOST, nullable) receives the greedy ids. */
uint32_t qb_batch_decode_greedy(uint64_t batch, const uint32_t *tokens, size_t steps,
                                uint32_t *ids);
/* Logits of the last step, [sequences][vocab]. */
uint32_t qb_batch_logits(uint64_t batch, float *logits, size_t logits_len);
uint32_t qb_batch_info_get(uint64_t batch, qb_batch_info *out);
uint32_t qb_batch_reset(uint64_t batch);
uint32_t qb_batch_stream(uint64_t batch, void **stream);
uint32_t qb_batch_free(uint64_t batch);

/* ------------------------------------------------------------------ */
/* Checkpoint loading: safetensors (src/weights.rs:89-264)             */
/* ------------------------------------------------------------------ */
/* The HF config.json fields the reference validates (QwenConfig,
 * src/weights.rs:9-28), parsed by the caller.  `architectures` holds
 * `architectures_count` strings (the reference requires exactly
 * ["Qwen2ForCausalLM"]); has_rope_scaling = a rope_scaling key present and
 * not null. */
typedef struct {
    const char *model_type, *hidden_act, *torch_dtype;
    const char *const *architectures;
    size_t architectures_count;
    size_t vocab_size, hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
        num_key_value_heads, max_position_embeddings;
    float rms_norm_eps, rope_theta;
    int32_t tie_word_embeddings, use_sliding_window, has_rope_scaling;
} qb_qwen_config;

/* tensor_shapes (src/weights.rs:96-187): validates the config (supported
 * architecture, positive dimensions, head divisibility, even head width,
 * finite positive epsilon and base; QB_LOAD_UNSUPPORTED_CONFIG), checks
 * every dimension product (QB_DIMENSION_OVERFLOW) and the 6 GiB planning
 * budget of raw BF16 plus FP32 payload (QB_RESOURCE_BUDGET); *count = the
 * number of expected tensors (12 per layer plus the embedding and final
 * norm; the tied head has no tensor).  Host only. */
uint32_t qb_qwen_tensor_count(const qb_qwen_config *config, size_t *count);
/* inspect_qwen (src/weights.rs:189-221) over a whole safetensors file in
 * HOST memory: the file format (header length and JSON, known dtypes,
 * contiguous data offsets covering exactly the data section, sizes that
 * match the shapes: QB_LOAD_FORMAT), then no unexpected name
 * (QB_LOAD_UNEXPECTED_TENSOR, detail.index = its position in the header),
 * then, in sorted-name order, every expected tensor present
 * (QB_LOAD_MISSING_TENSOR), of its shape (QB_INVALID_SHAPE) and BF16
 * (QB_LOAD_INVALID_DTYPE), detail.index = its position in the sorted
 * expected names.  Host only. */
uint32_t qb_safetensors_inspect(const uint8_t *data, size_t len, const qb_qwen_config *config,
                                size_t *tensor_count);
/* decode_qwen (src/weights.rs:226-264) and Decoder creation: inspects,
 * checks the 6 GiB budget of the decoded payload plus the file
 * (QB_RESOURCE_BUDGET), rejects any non-finite BF16 value before any
 * device work (QB_NONFINITE, detail.index = the tensor's sorted position,
 * detail.actual = the element), then creates and finalizes a device model
 * (qb_model_create with max_tokens = max_position_embeddings, heads of
 * hidden_size / num_attention_heads) from the BF16 payload: no partially
 * loaded model is returned.  The reference's file integrity checks
 * (inventory sizes and SHA-256, src/weights.rs:266-288) stay with the
 * caller, which owns the files. */
uint32_t qb_model_load_safetensors(const uint8_t *data, size_t len, const qb_qwen_config *config,
                                   uint32_t linear_format, uint32_t table_format, int device,
                                   uint64_t *out_model);

/* ------------------------------------------------------------------ */
/* Tokenizer and chat template (src/tokenizer.rs), host only           */
/* ------------------------------------------------------------------ */
/* The Qwen2 byte-level BPE of a tokenizer.json (NFC, the Qwen2 split
 * pattern, ByteLevel pre-tokenizer and decoder, unnormalized added tokens);
 * other configurations are QB_TOKENIZER_UNSUPPORTED_ASSETS, malformed JSON
 * QB_TOKENIZER_JSON.  Text is UTF-8 (QB_TOKENIZER_ENCODING otherwise).
 * Outputs: counts/lengths are always written; QB_INVALID_OUTPUT_LENGTH when
 * the capacity is short (nothing copied). */
enum { QB_ROLE_SYSTEM = 0, QB_ROLE_USER = 1, QB_ROLE_ASSISTANT = 2 };

/* Tokenizer::from_bytes of a tokenizer.json (no chat checks). */
uint32_t qb_tokenizer_from_json(const uint8_t *json, size_t len, uint64_t *out_tokenizer);
/* ChatTokenizer::load, src/tokenizer.rs:68-124, from the three files'
 * contents: tokenizer_config.json (Qwen2Tokenizer, no BOS, <|im_end|> EOS),
 * generation_config.json (stop ids [151645, 151643]) and tokenizer.json
 * (<|im_start|> 151644, <|im_end|> 151645, <|endoftext|> 151643).  The
 * reference's inventory hash check of the files stays with the caller. */
uint32_t qb_tokenizer_load_chat(const uint8_t *tokenizer_json, size_t tokenizer_len,
                                const uint8_t *tokenizer_config_json, size_t config_len,
                                const uint8_t *generation_config_json, size_t generation_len,
                                uint64_t *out_tokenizer);
/* ChatTokenizer::encode, src/tokenizer.rs:125-131 (no special tokens added). */
uint32_t qb_tokenizer_encode(uint64_t tokenizer, const uint8_t *text, size_t len, uint32_t *ids,
                             size_t capacity, size_t *count);
/* ChatTokenizer::decode, src/tokenizer.rs:139-154: QB_TOKENIZER_INVALID_TOKEN
 * (detail.actual = the id) for an id with no token. */
uint32_t qb_tokenizer_decode(uint64_t tokenizer, const uint32_t *ids, size_t count,
                             int32_t skip_special, char *text, size_t capacity, size_t *len);
/* ChatTokenizer::stop_tokens (empty for qb_tokenizer_from_json). */
uint32_t qb_tokenizer_stop_tokens(uint64_t tokenizer, uint32_t *ids, size_t capacity, size_t *count);
uint32_t qb_tokenizer_free(uint64_t tokenizer);
/* TextStream (src/tokenizer.rs:168-214): push writes the newly completed
 * text (*has_text = 1) or nothing while a UTF-8 sequence is incomplete;
 * special tokens print nothing; an unknown id is QB_TOKENIZER_INVALID_TOKEN
 * and leaves the stream as it was. */
uint32_t qb_tokenizer_stream_create(uint64_t tokenizer, uint64_t *out_stream);
uint32_t qb_tokenizer_stream_push(uint64_t stream, uint32_t id, char *text, size_t capacity,
                                  size_t *len, int32_t *has_text);
uint32_t qb_tokenizer_stream_pending(uint64_t stream, size_t *pending);
uint32_t qb_tokenizer_stream_free(uint64_t stream);
/* render_chat, src/tokenizer.rs:40-63: messages as (role, UTF-8 content)
 * triples; QB_TOKENIZER_EMPTY_MESSAGES for none. */
uint32_t qb_render_chat(const uint32_t *roles, const uint8_t *const *contents, const size_t *lengths,
                        size_t count, int32_t generation_prompt, char *text, size_t capacity,
                        size_t *len);

/* ------------------------------------------------------------------ */
/* Tensor parallelism across the GPUs of one box                       */
/* ------------------------------------------------------------------ */
/* No counterpart in the reference (one CPU thread, src/kernels.rs:8); these
 * replace its two full-width reductions per layer -- o_proj
 * (src/kv_cache.rs:581-585) and down (src/kv_cache.rs:437-443) -- with a
 * sum over ranks, and its argmax over the vocabulary
 * (src/sampling.rs:65-70) with one over ranks.  One process per GPU; every
 * rank makes the same calls in the same order.
 *
 * A shard (qb_model_create_tp) of rank r of `size` holds: for size <=
 * kv_heads, kv_heads / size whole KV groups (their query heads and KV
 * heads); for larger sizes (a multiple of kv_heads), one KV head replicated
 * on size / kv_heads ranks that split its group's query heads (e.g. 4 and
 * 3 of 7); ff_dim / size FFN columns; whole 128-row tiles of the LM-head
 * rows; the whole embedding table and norms.  qb_model_set_tensor takes
 * the FULL tensors on every rank (INT8 row scales are those of the whole
 * rows).  Finiteness of the rows a rank does not keep is checked by the
 * rank that keeps them.  A shard decodes only through qb_batch_create_tp
 * (qb_session_create returns QB_UNSUPPORTED). */
typedef struct {
    int32_t rank, size;
    size_t head0, heads;        /* query heads [head0, head0 + heads) */
    size_t kv_head0, kv_heads;  /* KV heads */
    size_t ff0, ff;             /* FFN columns */
    size_t vocab0, vocab;       /* LM-head rows (global ids) */
} qb_tp_shard;

uint32_t qb_model_create_tp(const qb_model_config *config, uint32_t linear_format,
                            uint32_t table_format, int device, int tp_rank, int tp_size,
                            uint64_t *out_model);
uint32_t qb_model_tp_info(uint64_t model, qb_tp_shard *out);
/* The shard rank `tp_rank` of `tp_size` would hold (host only, no device
 * needed); QB_UNSUPPORTED when the shape does not split that way. */
uint32_t qb_tp_shard_of(const qb_model_config *config, int tp_rank, int tp_size, qb_tp_shard *out);

/* The communicator: one exchange buffer per rank in device memory (flags,
 * two slots of partial sums [rows][hidden], two slots of argmax pairs),
 * shared with the other ranks through CUDA IPC.  Create it on the rank's
 * device for at least the batch's workspace rows (max(sequences, 256)),
 * export its 64-byte handle, exchange the handles (any host channel), then
 * connect with all `size` handles in rank order.  Each exchange raises this
 * rank's flag in every rank's buffer and waits (bounded, 2 s; then
 * QB_DEVICE_TIMEOUT) for all flags, then reads every rank's data with peer
 * loads and sums in rank order: every rank gets the same values. */
uint32_t qb_tp_comm_create(int device, size_t rows, size_t hidden, uint64_t *out_comm);
uint32_t qb_tp_comm_handle(uint64_t comm, void *out, size_t len /* 64 */);
uint32_t qb_tp_comm_connect(uint64_t comm, int rank, int size, const void *handles,
                            size_t len /* size * 64 */);
uint32_t qb_tp_comm_free(uint64_t comm);
/* A batch over a shard: as qb_batch_create; greedy ids are global, and
 * qb_batch_logits returns this rank's rows, [sequences][vocab] of its
 * qb_tp_shard. */
uint32_t qb_batch_create_tp(uint64_t model, uint64_t comm, size_t sequences, size_t capacity,
                            uint32_t kv_dtype, uint64_t *out_batch);

/* ------------------------------------------------------------------ */
/* Synthetic inputs (host only; no GPU needed)                         */
/* ------------------------------------------------------------------ */

/* Fills `out` with n normal(0, stddev) draws of the documented counter-based
 * generator (splitmix64 + Box-Muller) for (seed, stream).  out_dtype:
 * QB_HOST_F32 (FP32) or QB_HOST_BF16 (FP32 rounded to BF16, nearest-even). */
uint32_t qb_synthetic_normal(uint64_t seed, uint64_t stream, size_t n, double stddev,
                             uint32_t out_dtype, void *out);
/* n token ids uniform over [0, vocab) for (seed, stream). */
uint32_t qb_synthetic_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab,
                             uint32_t *out);

#ifdef __cplusplus
}
#endif
#endif
