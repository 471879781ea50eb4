/*
 * CPU oracle for the Qwen2 token loop -- TEST INFRASTRUCTURE ONLY.
 * A C restatement of the reference crate's FP32 arithmetic; only the tests,
 * the smoke check and the benchmark's CPU-baseline leg may load it.
 */
#ifndef QWEN_ORACLE_H
#define QWEN_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; numerically identical to the product's QB_* codes. */
enum {
    OR_OK = 0,
    OR_ZERO_DIMENSION = 1,
    OR_DIMENSION_OVERFLOW = 2,
    OR_INVALID_LENGTH = 3,
    OR_INVALID_GROUP_SIZE = 4,
    OR_INVALID_SHAPE = 5,
    OR_NONFINITE_WEIGHT = 6,
    OR_UNREPRESENTABLE_SCALE = 7,
    OR_ALLOCATION = 8,
    OR_INVALID_TOKEN = 9,
    OR_INVALID_EPSILON = 10,
    OR_NONFINITE = 11,
    OR_ALL_MASKED = 12,
    OR_ODD_HEAD_DIMENSION = 13,
    OR_POSITION_OVERFLOW = 14,
    OR_POSITION_OUT_OF_RANGE = 15,
    OR_INVALID_BASE = 16,
    OR_INVALID_ANGLE = 17,
    OR_INVALID_CAPACITY = 18,
    OR_RESOURCE_BUDGET = 19,
    OR_INVALID_OUTPUT_LENGTH = 20,
    OR_EMPTY_INPUT = 21,
    OR_NOT_EMPTY = 22,
    OR_FULL = 23,
    OR_INVALID_STATE = 24,
    OR_INVALID_CONFIG = 25,
    OR_INVALID_PARAMETERS = 27,
    OR_EMPTY_LOGITS = 31,
    OR_CONTEXT_LIMIT = 34,
    OR_TRACE_LIMIT = 35,
    OR_EMPTY_PROMPT = 36,
    OR_OUTPUT_LIMIT = 37,
};

typedef struct {
    size_t buffer;   /* which buffer (argument order) */
    size_t expected; /* expected length */
    size_t actual;   /* actual length, or an offending id */
    size_t index;    /* offending element index */
} or_detail;

typedef struct {
    size_t vocab, layers, hidden, query_heads, kv_heads, head_dim, ff, max_tokens;
    float rope_base, norm_eps;
} or_config;

enum { OR_MAT_NONE = -1, OR_MAT_F32 = 0, OR_MAT_BF16 = 1, OR_MAT_INT8 = 2 };
typedef struct {
    int kind;
    const float *f32;      /* OR_MAT_F32: [rows, cols] */
    const uint16_t *bf16;  /* OR_MAT_BF16: [rows, cols] BF16 bit patterns */
    const int8_t *q;       /* OR_MAT_INT8: [rows, cols] */
    const float *scales;   /* OR_MAT_INT8: [rows, ceil(cols/group)] */
    size_t group;
} or_matrix;

typedef struct {
    const float *attn_norm, *ffn_norm;
    or_matrix q, k, v, o, gate, up, down;
    const float *qb, *kb, *vb;
} or_layer;

enum { OR_W_EMBEDDING = 0, OR_W_LM_HEAD = 1, OR_W_Q = 2, OR_W_K, OR_W_V, OR_W_O, OR_W_GATE, OR_W_UP, OR_W_DOWN };
enum { OR_V_FINAL_NORM = 0, OR_V_ATTN_NORM = 1, OR_V_FFN_NORM, OR_V_Q_BIAS, OR_V_K_BIAS, OR_V_V_BIAS };

typedef struct or_model or_model;
typedef struct or_session or_session;

void or_set_threads(int n);
int or_get_threads(void);
float or_round_bf16(float x);

int or_linear(const float *x, size_t xl, const float *w, size_t wl, float *y, size_t yl,
              size_t t, size_t in, size_t out, or_detail *d);
int or_linear_lanes4(const float *x, size_t xl, const float *w, size_t wl, float *y, size_t yl,
                     size_t t, size_t in, size_t out, or_detail *d);
int8_t or_encode(float weight, float scale);
int or_quantize(const float *w, size_t wl, size_t out, size_t in, size_t group, int8_t *values,
                float *scales, or_detail *d);
void or_dequantize(const int8_t *values, const float *scales, size_t out, size_t in, size_t group,
                   float *y);
int or_linear_int8(const float *x, size_t xl, const int8_t *values, const float *scales,
                   float *y, size_t yl, size_t t, size_t in, size_t out, size_t group,
                   int lanes4, or_detail *d);
int or_embedding(const size_t *ids, size_t n, const float *table, size_t tl, float *y, size_t yl,
                 size_t vocab, size_t width, or_detail *d);
int or_residual_add(const float *x, size_t xl, const float *r, size_t rl, float *y, size_t yl,
                    or_detail *d);
int or_rmsnorm(const float *x, size_t xl, const float *g, size_t gl, float *y, size_t yl,
               size_t rows, size_t width, float eps, or_detail *d);
int or_silu(const float *x, size_t xl, float *y, size_t yl, or_detail *d);
int or_softmax(const float *logits, size_t ll, const uint8_t *mask, size_t ml, float *y, size_t yl,
               size_t rows, size_t width, or_detail *d);
void or_rope_table(float base, size_t hd, size_t start, size_t count, float *cos_out,
                   float *sin_out);
int or_rope(const float *x, size_t xl, float *y, size_t yl, size_t tokens, size_t heads,
            size_t hd, size_t start, float base, or_detail *d);

or_model *or_model_new(const or_config *c);
void or_model_free(or_model *m);
void or_model_set_matrix(or_model *m, long layer, int which, const or_matrix *mat);
void or_model_set_vector(or_model *m, long layer, int which, const float *v);
size_t or_trace_len(const or_config *c, size_t T);
int or_forward(const or_model *m, const size_t *ids, size_t T, float *logits, float *trace);

size_t or_workspace_bytes(const or_config *c, size_t capacity);
int or_session_new(const or_model *m, size_t capacity, int kv_bf16, size_t budget,
                   or_session **out);
void or_session_free(or_session *s);
size_t or_session_processed(const or_session *s);
int or_session_is_valid(const or_session *s);
size_t or_session_logical_bytes(const or_session *s);
size_t or_session_workspace_bytes(const or_session *s);
void or_session_reset(or_session *s);
int or_session_step(or_session *s, size_t token, float *logits, size_t logits_len);
int or_session_append(or_session *s, const size_t *tokens, size_t n, float *logits,
                      size_t logits_len, int require_empty);
int or_session_append_chunked(or_session *s, const size_t *tokens, size_t n, float *logits,
                              size_t logits_len, int require_empty, size_t chunk);
void or_set_fast(int on);
size_t or_argmax(const float *logits, size_t n);
long or_greedy(or_session *s, const size_t *prompt, size_t n, const size_t *stops, size_t nstops,
               size_t max_new, size_t *out);
long or_uncached_greedy(const or_model *m, const size_t *prompt, size_t n, const size_t *stops,
                        size_t nstops, size_t max_new, size_t *out);

/* Seeded synthetic inputs for the benchmark workloads: the documented
 * counter-based generator (splitmix64 finalizer + Box-Muller) that the
 * library's qb_synthetic_normal / qb_synthetic_tokens also implement, so the
 * oracle can build the same weights and prompts without loading the
 * library.  out_dtype 0 = FP32, 1 = BF16 bits (nearest-even). */
int or_synthetic_normal(uint64_t seed, uint64_t stream, size_t n, double stddev, int out_dtype,
                        void *out);
/* Seeded temperature / top-k sampling (src/sampling.rs): ChaCha8 stream of
 * rand_chacha 0.9 seeded through rand_core 0.9's seed_from_u64. */
typedef struct {
    uint32_t key[8];
    uint64_t counter;  /* next block number */
    uint32_t buf[64];  /* four blocks of keystream */
    size_t index;      /* next unread word of buf; 64 = empty */
} or_rng;
typedef struct {
    int greedy;
    float temperature;
    size_t top_k;
    uint64_t seed;
    or_rng rng;
} or_sampler;
void or_chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]);
void or_rng_from_seed(or_rng *g, const uint8_t seed[32]);
void or_rng_seed(or_rng *g, uint64_t seed);
uint64_t or_rng_next_u64(or_rng *g);
double or_rng_next_f64(or_rng *g);
int or_sampler_init(or_sampler *s, int greedy, float temperature, size_t top_k, uint64_t seed);
void or_sampler_reset(or_sampler *s);
int or_sampler_validate_vocab(const or_sampler *s, size_t vocab);
int or_sampler_sample(or_sampler *s, const float *logits, size_t n, size_t *out);

int or_synthetic_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab, uint32_t *out);

#ifdef __cplusplus
}
#endif
#endif
