/*
 * CPU oracle for the Qwen2 token loop -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the scalar FP32 arithmetic of the reference
 * crate `llm_inference` (pshevskiy/llm_inference_edu, Rust).  It exists so the
 * tests and the benchmark's CPU baseline can check the CUDA product path; the
 * product never links, loads or calls it.
 *
 * Every function names the reference lines it follows.  Arithmetic rules:
 *   - compiled with -ffp-contract=off and no fast-math, so `a*b+c` is two
 *     roundings exactly like Rust's f32 operators;
 *   - transcendental calls are glibc's expf/powf/sinf/cosf/roundf, which is
 *     what Rust's f32::{exp,powf,sin_cos,round} lower to on Linux;
 *   - every reduction keeps the reference's order (increasing index, or the
 *     four-lane order of `dot_lanes4`).
 * Independent output rows may be computed by several OpenMP threads; that
 * never changes a result because each row's reduction order is fixed.
 *
 * Extensions beyond the reference (each documented where it appears):
 *   - a per-row INT8 scheme (group size equal to the row width, which the
 *     reference's 1..=256 admission rejects but whose per-group arithmetic is
 *     identical, src/quantization.rs:91-101);
 *   - BF16-valued matrices read directly (value = bits << 16, exactly the
 *     expansion of src/weights.rs:250-251);
 *   - an optional BF16 KV cache (K after RoPE and V rounded to BF16 with
 *     round-to-nearest-even at write);
 *   - an untied output head (7B shape), which the reference cannot express.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#include "qwen_oracle.h"

/* ------------------------------------------------------------------ */
/* helpers                                                             */
/* ------------------------------------------------------------------ */

static int mul_ovf(size_t a, size_t b, size_t *out) {
    if (a != 0 && b > SIZE_MAX / a) return 1;
    *out = a * b;
    return 0;
}

static int finite_all(const float *v, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(v[i])) return 0;
    return 1;
}

static float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round-to-nearest-even FP32 -> BF16 -> FP32 (NaN kept quiet). */
float or_round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
        u = (u | 0x00400000u) & 0xffff0000u;
    } else {
        uint32_t lsb = (u >> 16) & 1u;
        u = (u + 0x7fffu + lsb) & 0xffff0000u;
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static int g_threads = 0;
void or_set_threads(int n) { g_threads = n; }
int or_get_threads(void) { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

/* Rust's f32::max: returns the other operand when one is NaN. */
static float rmax(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* ------------------------------------------------------------------ */
/* linear  (src/lib.rs:51-111)                                          */
/* ------------------------------------------------------------------ */

/* validate_linear, src/lib.rs:76-111: zero dimensions, then product
 * overflow (x, w, y), then exact lengths x, w, y; nothing is written. */
static int validate_linear(size_t xl, size_t wl, size_t yl, size_t t, size_t in, size_t out,
                           or_detail *d) {
    if (t == 0 || in == 0 || out == 0) return OR_ZERO_DIMENSION;
    size_t xn, wn, yn;
    if (mul_ovf(t, in, &xn) || mul_ovf(out, in, &wn) || mul_ovf(t, out, &yn))
        return OR_DIMENSION_OVERFLOW;
    const size_t exp_[3] = {xn, wn, yn}, act[3] = {xl, wl, yl};
    for (int i = 0; i < 3; ++i) {
        if (act[i] != exp_[i]) {
            if (d) { d->buffer = i; d->expected = exp_[i]; d->actual = act[i]; }
            return OR_INVALID_LENGTH;
        }
    }
    return OR_OK;
}

/* The scalar dot of src/lib.rs:63-70: one FP32 sum in increasing index order. */
static float dot_scalar(const float *x, const float *w, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += x[i] * w[i];
    return sum;
}

/* dot_lanes4, src/kernels.rs:31-46: four strided lanes, ((s0+s1)+s2)+s3,
 * then the tail in order. */
static float dot_lanes4(const float *x, const float *w, size_t n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    size_t bulk = n - n % 4;
    for (size_t i = 0; i < bulk; i += 4) {
        s0 += x[i] * w[i];
        s1 += x[i + 1] * w[i + 1];
        s2 += x[i + 2] * w[i + 2];
        s3 += x[i + 3] * w[i + 3];
    }
    float sum = ((s0 + s1) + s2) + s3;
    for (size_t i = bulk; i < n; ++i) sum += x[i] * w[i];
    return sum;
}

int or_linear(const float *x, size_t xl, const float *w, size_t wl, float *y, size_t yl,
              size_t t, size_t in, size_t out, or_detail *d) {
    int s = validate_linear(xl, wl, yl, t, in, out, d);
    if (s) return s;
    long long n = (long long)(t * out);
#pragma omp parallel for schedule(static) num_threads(or_get_threads()) if (n * (long long)in > 65536)
    for (long long k = 0; k < n; ++k) {
        size_t tt = (size_t)k / out, o = (size_t)k % out;
        y[tt * out + o] = dot_scalar(x + tt * in, w + o * in, in);
    }
    return OR_OK;
}

/* linear_lanes4, src/kernels.rs:10-28. */
int or_linear_lanes4(const float *x, size_t xl, const float *w, size_t wl, float *y, size_t yl,
                     size_t t, size_t in, size_t out, or_detail *d) {
    int s = validate_linear(xl, wl, yl, t, in, out, d);
    if (s) return s;
    long long n = (long long)(t * out);
#pragma omp parallel for schedule(static) num_threads(or_get_threads()) if (n * (long long)in > 65536)
    for (long long k = 0; k < n; ++k) {
        size_t tt = (size_t)k / out, o = (size_t)k % out;
        y[tt * out + o] = dot_lanes4(x + tt * in, w + o * in, in);
    }
    return OR_OK;
}

/* ------------------------------------------------------------------ */
/* groupwise INT8 (src/quantization.rs)                                */
/* ------------------------------------------------------------------ */

/* encode, src/quantization.rs:36-40: f32 quotient, round half away from
 * zero, clamp to [-127, 127]. */
int8_t or_encode(float weight, float scale) {
    float r = roundf(weight / scale);
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)r;
}

/* GroupwiseInt8::quantize, src/quantization.rs:55-116.  Admission order:
 * group size, zero dimension, overflow, length, non-finite weight; then per
 * group max|w| folded from 0, scale = max/127 (zero group -> 1), reject a
 * non-positive/non-finite scale or an unrepresentable reconstruction.
 * Extension: group == input_dim is also admitted (one scale per row). */
int or_quantize(const float *w, size_t wl, size_t out, size_t in, size_t group,
                int8_t *values, float *scales, or_detail *d) {
    if (!((group >= 1 && group <= 256) || (group == in && in > 0))) return OR_INVALID_GROUP_SIZE;
    if (out == 0 || in == 0) return OR_ZERO_DIMENSION;
    size_t len, sc;
    if (mul_ovf(out, in, &len)) return OR_DIMENSION_OVERFLOW;
    size_t gpr = in / group + (in % group != 0);
    if (mul_ovf(out, gpr, &sc)) return OR_DIMENSION_OVERFLOW;
    size_t sb;
    if (mul_ovf(sc, 4, &sb) || sb > SIZE_MAX - len) return OR_DIMENSION_OVERFLOW;
    if (wl != len) {
        if (d) { d->buffer = 0; d->expected = len; d->actual = wl; }
        return OR_INVALID_LENGTH;
    }
    for (size_t i = 0; i < len; ++i)
        if (!isfinite(w[i])) {
            if (d) d->index = i;
            return OR_NONFINITE_WEIGHT;
        }
    int status = OR_OK;
#pragma omp parallel for schedule(static) num_threads(or_get_threads()) if (len > 65536)
    for (long long o = 0; o < (long long)out; ++o) {
        for (size_t g = 0; g < gpr; ++g) {
            size_t start = g * group, end = start + group < in ? start + group : in;
            const float *row = w + (size_t)o * in;
            float m = 0.0f;
            for (size_t i = start; i < end; ++i) m = rmax(m, fabsf(row[i]));
            float scale = m == 0.0f ? 1.0f : m / 127.0f;
            if (!isfinite(scale) || scale <= 0.0f) {
#pragma omp atomic write
                status = OR_UNREPRESENTABLE_SCALE;
                continue;
            }
            scales[(size_t)o * gpr + g] = scale;
            for (size_t i = start; i < end; ++i) {
                int8_t q = or_encode(row[i], scale);
                if (!isfinite((float)q * scale)) {
#pragma omp atomic write
                    status = OR_UNREPRESENTABLE_SCALE;
                }
                values[(size_t)o * in + i] = q;
            }
        }
    }
    return status;
}

/* dequantize, src/quantization.rs:141-166: value = f32(q) * scale. */
void or_dequantize(const int8_t *values, const float *scales, size_t out, size_t in, size_t group,
                   float *y) {
    size_t gpr = in / group + (in % group != 0);
    for (size_t o = 0; o < out; ++o)
        for (size_t i = 0; i < in; ++i)
            y[o * in + i] = (float)values[o * in + i] * scales[o * gpr + i / group];
}

/* The fused dot of linear_int8, src/quantization.rs:200-212:
 * sum += x[i] * (f32(q) * scale), increasing i. */
static float dot_int8(const float *x, const int8_t *q, const float *s, size_t in, size_t group) {
    float sum = 0.0f;
    size_t gpr = in / group + (in % group != 0);
    for (size_t g = 0; g < gpr; ++g) {
        float scale = s[g];
        size_t start = g * group, end = start + group < in ? start + group : in;
        for (size_t i = start; i < end; ++i) sum += x[i] * ((float)q[i] * scale);
    }
    return sum;
}

/* The four-lane fused dot of linear_int8_lanes4, src/quantization.rs:248-276. */
static float dot_int8_lanes4(const float *x, const int8_t *q, const float *s, size_t in,
                             size_t group) {
    float sums[4] = {0, 0, 0, 0};
    size_t bulk = in - in % 4;
    if (group % 4 == 0) {
        size_t gpr = in / group + (in % group != 0);
        for (size_t g = 0; g < gpr; ++g) {
            float scale = s[g];
            size_t start = g * group, end = start + group < in ? start + group : in;
            size_t n4 = (end - start) / 4;
            for (size_t c = 0; c < n4; ++c) {
                size_t b = start + c * 4;
                sums[0] += x[b] * ((float)q[b] * scale);
                sums[1] += x[b + 1] * ((float)q[b + 1] * scale);
                sums[2] += x[b + 2] * ((float)q[b + 2] * scale);
                sums[3] += x[b + 3] * ((float)q[b + 3] * scale);
            }
        }
    } else {
        for (size_t i = 0; i < bulk; ++i) sums[i % 4] += x[i] * ((float)q[i] * s[i / group]);
    }
    float sum = ((sums[0] + sums[1]) + sums[2]) + sums[3];
    for (size_t i = bulk; i < in; ++i) sum += x[i] * ((float)q[i] * s[i / group]);
    return sum;
}

static int validate_int8_linear(size_t xl, size_t yl, size_t t, size_t in, size_t out,
                                or_detail *d) {
    if (t == 0) return OR_ZERO_DIMENSION;
    size_t xn, yn;
    if (mul_ovf(t, in, &xn) || mul_ovf(t, out, &yn)) return OR_DIMENSION_OVERFLOW;
    if (xl != xn) {
        if (d) { d->buffer = 0; d->expected = xn; d->actual = xl; }
        return OR_INVALID_LENGTH;
    }
    if (yl != yn) {
        if (d) { d->buffer = 2; d->expected = yn; d->actual = yl; }
        return OR_INVALID_LENGTH;
    }
    return OR_OK;
}

/* linear_int8, src/quantization.rs:168-215. */
int or_linear_int8(const float *x, size_t xl, const int8_t *values, const float *scales,
                   float *y, size_t yl, size_t t, size_t in, size_t out, size_t group,
                   int lanes4, or_detail *d) {
    int s = validate_int8_linear(xl, yl, t, in, out, d);
    if (s) return s;
    size_t gpr = in / group + (in % group != 0);
    long long n = (long long)(t * out);
#pragma omp parallel for schedule(static) num_threads(or_get_threads()) if (n * (long long)in > 65536)
    for (long long k = 0; k < n; ++k) {
        size_t tt = (size_t)k / out, o = (size_t)k % out;
        const int8_t *q = values + o * in;
        const float *sc = scales + o * gpr;
        y[tt * out + o] = lanes4 ? dot_int8_lanes4(x + tt * in, q, sc, in, group)
                                 : dot_int8(x + tt * in, q, sc, in, group);
    }
    return OR_OK;
}

/* ------------------------------------------------------------------ */
/* elementwise ops (src/ops.rs)                                        */
/* ------------------------------------------------------------------ */

/* embedding, src/ops.rs:67-91. */
int or_embedding(const size_t *ids, size_t n, const float *table, size_t tl, float *y, size_t yl,
                 size_t vocab, size_t width, or_detail *d) {
    size_t tn, yn;
    if (vocab == 0 || width == 0) return OR_ZERO_DIMENSION;
    if (mul_ovf(vocab, width, &tn)) return OR_DIMENSION_OVERFLOW;
    if (n == 0) return OR_ZERO_DIMENSION;
    if (mul_ovf(n, width, &yn)) return OR_DIMENSION_OVERFLOW;
    if (tl != tn) { if (d) { d->buffer = 0; d->expected = tn; d->actual = tl; } return OR_INVALID_LENGTH; }
    if (yl != yn) { if (d) { d->buffer = 1; d->expected = yn; d->actual = yl; } return OR_INVALID_LENGTH; }
    for (size_t p = 0; p < n; ++p)
        if (ids[p] >= vocab) { if (d) { d->index = p; d->actual = ids[p]; } return OR_INVALID_TOKEN; }
    for (size_t p = 0; p < n; ++p) memcpy(y + p * width, table + ids[p] * width, width * 4);
    return OR_OK;
}

/* residual_add, src/ops.rs:97-107. */
int or_residual_add(const float *x, size_t xl, const float *r, size_t rl, float *y, size_t yl,
                    or_detail *d) {
    if (xl == 0) return OR_ZERO_DIMENSION;
    if (rl != xl) { if (d) { d->buffer = 1; d->expected = xl; d->actual = rl; } return OR_INVALID_LENGTH; }
    if (yl != xl) { if (d) { d->buffer = 2; d->expected = xl; d->actual = yl; } return OR_INVALID_LENGTH; }
    for (size_t i = 0; i < xl; ++i) y[i] = x[i] + r[i];
    return OR_OK;
}

/* The per-row body of rmsnorm, src/ops.rs:137-149: row scale
 * s = fold(sqrt(eps), max|x|); sum((x/s)^2) in order;
 * d = sqrt(sum/width + (sqrt(eps)/s)^2); y = (x/s)/d*gain. */
static void rms_row(const float *x, const float *g, float *y, size_t width, float eps) {
    float se = sqrtf(eps);
    float scale = se;
    for (size_t i = 0; i < width; ++i) scale = rmax(scale, fabsf(x[i]));
    float ss = 0.0f;
    for (size_t i = 0; i < width; ++i) {
        float v = x[i] / scale;
        ss += v * v;
    }
    float seps = se / scale;
    float den = sqrtf(ss / (float)width + seps * seps);
    for (size_t i = 0; i < width; ++i) y[i] = (x[i] / scale) / den * g[i];
}

/* rmsnorm, src/ops.rs:119-152. */
int or_rmsnorm(const float *x, size_t xl, const float *g, size_t gl, float *y, size_t yl,
               size_t rows, size_t width, float eps, or_detail *d) {
    if (rows == 0 || width == 0) return OR_ZERO_DIMENSION;
    size_t len;
    if (mul_ovf(rows, width, &len)) return OR_DIMENSION_OVERFLOW;
    if (xl != len) { if (d) { d->buffer = 0; d->expected = len; d->actual = xl; } return OR_INVALID_LENGTH; }
    if (gl != width) { if (d) { d->buffer = 1; d->expected = width; d->actual = gl; } return OR_INVALID_LENGTH; }
    if (yl != len) { if (d) { d->buffer = 2; d->expected = len; d->actual = yl; } return OR_INVALID_LENGTH; }
    if (!isfinite(eps) || eps <= 0.0f) return OR_INVALID_EPSILON;
    for (size_t i = 0; i < xl; ++i) if (!isfinite(x[i])) { if (d) { d->buffer = 0; d->index = i; } return OR_NONFINITE; }
    for (size_t i = 0; i < gl; ++i) if (!isfinite(g[i])) { if (d) { d->buffer = 1; d->index = i; } return OR_NONFINITE; }
    for (size_t r = 0; r < rows; ++r) rms_row(x + r * width, g, y + r * width, width, eps);
    return OR_OK;
}

/* silu, src/ops.rs:158-173: the sign branch avoids exp overflow. */
static float silu1(float v) {
    if (v >= 0.0f) return v / (1.0f + expf(-v));
    float e = expf(v);
    return v * e / (1.0f + e);
}

int or_silu(const float *x, size_t xl, float *y, size_t yl, or_detail *d) {
    if (xl == 0) return OR_ZERO_DIMENSION;
    if (yl != xl) { if (d) { d->buffer = 1; d->expected = xl; d->actual = yl; } return OR_INVALID_LENGTH; }
    for (size_t i = 0; i < xl; ++i) if (!isfinite(x[i])) { if (d) { d->buffer = 0; d->index = i; } return OR_NONFINITE; }
    for (size_t i = 0; i < xl; ++i) y[i] = silu1(x[i]);
    return OR_OK;
}

/* softmax_impl, src/ops.rs:198-257: every row is admitted before any write;
 * max over allowed entries, exp(v - max) summed in order, then divided. */
int or_softmax(const float *logits, size_t ll, const uint8_t *mask, size_t ml, float *y, size_t yl,
               size_t rows, size_t width, or_detail *d) {
    if (rows == 0 || width == 0) return OR_ZERO_DIMENSION;
    size_t len;
    if (mul_ovf(rows, width, &len)) return OR_DIMENSION_OVERFLOW;
    if (ll != len) { if (d) { d->buffer = 0; d->expected = len; d->actual = ll; } return OR_INVALID_LENGTH; }
    if (yl != len) { if (d) { d->buffer = 1; d->expected = len; d->actual = yl; } return OR_INVALID_LENGTH; }
    if (mask && ml != len) { if (d) { d->buffer = 2; d->expected = len; d->actual = ml; } return OR_INVALID_LENGTH; }
    for (size_t r = 0; r < rows; ++r) {
        int any = 0;
        for (size_t i = 0; i < width; ++i) {
            size_t k = r * width + i;
            if (!mask || mask[k]) {
                any = 1;
                if (!isfinite(logits[k])) { if (d) { d->buffer = 0; d->index = k; } return OR_NONFINITE; }
            }
        }
        if (!any) { if (d) d->index = r; return OR_ALL_MASKED; }
    }
    for (size_t r = 0; r < rows; ++r) {
        const float *row = logits + r * width;
        float *out = y + r * width;
        float m = -INFINITY;
        for (size_t i = 0; i < width; ++i)
            if (!mask || mask[r * width + i]) m = rmax(m, row[i]);
        float sum = 0.0f;
        for (size_t i = 0; i < width; ++i) {
            out[i] = (!mask || mask[r * width + i]) ? expf(row[i] - m) : 0.0f;
            sum += out[i];
        }
        for (size_t i = 0; i < width; ++i) out[i] /= sum;
    }
    return OR_OK;
}

/* ------------------------------------------------------------------ */
/* rope  (src/rope.rs:38-105)                                          */
/* ------------------------------------------------------------------ */

/* frequency_j = base.powf(-(2j as f32) / head_dim as f32), src/rope.rs:86. */
static float rope_frequency(float base, size_t j, size_t hd) {
    return powf(base, -((float)(2 * j)) / (float)hd);
}

/* Fills cos/sin for positions [start, start+count) and j < hd/2, row-major
 * [count][hd/2]; the same values the reference computes per call. */
void or_rope_table(float base, size_t hd, size_t start, size_t count, float *cos_out,
                   float *sin_out) {
    size_t half = hd / 2;
    for (size_t t = 0; t < count; ++t) {
        float pos = (float)(start + t);
        for (size_t j = 0; j < half; ++j) {
            float a = pos * rope_frequency(base, j, hd);
            cos_out[t * half + j] = cosf(a);
            sin_out[t * half + j] = sinf(a);
        }
    }
}

int or_rope(const float *x, size_t xl, float *y, size_t yl, size_t tokens, size_t heads,
            size_t hd, size_t start, float base, or_detail *d) {
    if (tokens == 0 || heads == 0 || hd == 0) return OR_ZERO_DIMENSION;
    if (hd % 2) return OR_ODD_HEAD_DIMENSION;
    size_t row, len;
    if (mul_ovf(heads, hd, &row) || mul_ovf(tokens, row, &len)) return OR_DIMENSION_OVERFLOW;
    if (start > SIZE_MAX - (tokens - 1)) return OR_POSITION_OVERFLOW;
    size_t last = start + tokens - 1;
    if (last > ((size_t)1 << 24)) return OR_POSITION_OUT_OF_RANGE;
    if (!isfinite(base) || base <= 0.0f) return OR_INVALID_BASE;
    if (xl != len) { if (d) { d->buffer = 0; d->expected = len; d->actual = xl; } return OR_INVALID_LENGTH; }
    if (yl != len) { if (d) { d->buffer = 1; d->expected = len; d->actual = yl; } return OR_INVALID_LENGTH; }
    for (size_t i = 0; i < xl; ++i) if (!isfinite(x[i])) { if (d) d->index = i; return OR_NONFINITE; }
    size_t half = hd / 2;
    for (size_t j = 0; j < half; ++j) {
        float f = rope_frequency(base, j, hd);
        if (!isfinite(f) || !isfinite((float)last * f)) return OR_INVALID_ANGLE;
    }
    for (size_t t = 0; t < tokens; ++t) {
        float pos = (float)(start + t);
        for (size_t j = 0; j < half; ++j) {
            float a = pos * rope_frequency(base, j, hd);
            float s = sinf(a), c = cosf(a);
            for (size_t h = 0; h < heads; ++h) {
                size_t off = t * row + h * hd;
                float av = x[off + j], bv = x[off + j + half];
                y[off + j] = av * c - bv * s;
                y[off + j + half] = bv * c + av * s;
            }
        }
    }
    return OR_OK;
}

/* ------------------------------------------------------------------ */
/* weight matrices (src/matrix.rs)                                      */
/* ------------------------------------------------------------------ */

/* Interleaved evaluation (test speed only): OR_IL output rows are summed
 * side by side, each in its own accumulator and in increasing index order,
 * so every output is bit-identical to the one-row-at-a-time dot; the CPU
 * overlaps the independent chains.  Off by default (the timed CPU baseline
 * keeps the reference's one-row-at-a-time loop); or_set_fast turns it on. */
static int g_fast = 0;
void or_set_fast(int on) { g_fast = on; }
#define OR_IL 8

static void project_il(const or_matrix *m, const float *x, float *y, size_t t, size_t in, size_t out) {
    long long nb = (long long)(out / OR_IL);
#pragma omp parallel for schedule(static) num_threads(or_get_threads()) if (nb * (long long)t * (long long)in > 65536)
    for (long long b = 0; b < nb; ++b) {
        size_t o0 = (size_t)b * OR_IL;
        for (size_t tt = 0; tt < t; ++tt) {
            const float *xr = x + tt * in;
            float acc[OR_IL];
#pragma GCC unroll 8
            for (int r = 0; r < OR_IL; ++r) acc[r] = 0.0f;
            if (m->kind == OR_MAT_F32) {
                const float *w = m->f32 + o0 * in;
                for (size_t i = 0; i < in; ++i) {
                    float xi = xr[i];
#pragma GCC unroll 8
                    for (int r = 0; r < OR_IL; ++r) acc[r] += xi * w[r * in + i];
                }
            } else if (m->kind == OR_MAT_BF16) {
                const uint16_t *w = m->bf16 + o0 * in;
                for (size_t i = 0; i < in; ++i) {
                    float xi = xr[i];
#pragma GCC unroll 8
                    for (int r = 0; r < OR_IL; ++r) acc[r] += xi * bf16_to_f32(w[r * in + i]);
                }
            } else {
                size_t group = m->group, gpr = in / group + (in % group != 0);
                const int8_t *q = m->q + o0 * in;
                const float *sc = m->scales + o0 * gpr;
                for (size_t g = 0; g < gpr; ++g) {
                    float scale[OR_IL];
                    for (int r = 0; r < OR_IL; ++r) scale[r] = sc[r * gpr + g];
                    size_t start = g * group, end = start + group < in ? start + group : in;
                    for (size_t i = start; i < end; ++i) {
                        float xi = xr[i];
#pragma GCC unroll 8
                        for (int r = 0; r < OR_IL; ++r) acc[r] += xi * ((float)q[r * in + i] * scale[r]);
                    }
                }
            }
            for (int r = 0; r < OR_IL; ++r) y[tt * out + o0 + r] = acc[r];
        }
    }
}

/* Token-vectorised evaluation (test speed only, several tokens): for each
 * output row, OR_IL tokens are summed side by side from a transposed copy
 * of their inputs, each token's sum in increasing index order, so every
 * output is bit-identical to the one-row-at-a-time dot. */
static void project_tv(const or_matrix *m, const float *x, float *y, size_t t, size_t in, size_t out) {
    enum { RB = 4, KB = 512 };
    size_t nb = (t + OR_IL - 1) / OR_IL, nrb = (out + RB - 1) / RB;
    float *xt = (float *)calloc(nb * in * OR_IL, sizeof(float));
    for (size_t tt = 0; tt < t; ++tt)
        for (size_t i = 0; i < in; ++i) xt[((tt / OR_IL) * in + i) * OR_IL + tt % OR_IL] = x[tt * in + i];
    size_t group = m->kind == OR_MAT_INT8 ? m->group : in, gpr = in / group + (in % group != 0);
    /* Tiles: RB rows x OR_IL tokens, the reduction in KB-element pieces, so
     * the inputs and weights of a piece stay in L1; each accumulator still
     * runs over its row in increasing index order. */
#pragma omp parallel for schedule(dynamic, 4) num_threads(or_get_threads()) if ((long long)out * (long long)t * (long long)in > 65536)
    for (long long rbb = 0; rbb < (long long)(nrb * nb); ++rbb) {
        size_t rb = (size_t)rbb / nb, b = (size_t)rbb % nb;
        size_t o0 = rb * RB, nr = out - o0 < RB ? out - o0 : RB;
        const float *xb = xt + b * in * OR_IL;
        float acc[RB][OR_IL];
        for (int r = 0; r < RB; ++r)
            for (int j = 0; j < OR_IL; ++j) acc[r][j] = 0.0f;
        for (size_t i0 = 0; i0 < in; i0 += KB) {
            size_t i1 = i0 + KB < in ? i0 + KB : in;
            for (size_t r = 0; r < nr; ++r) {
                size_t o = o0 + r;
                float *a = acc[r];
                if (m->kind == OR_MAT_F32) {
                    const float *w = m->f32 + o * in;
                    for (size_t i = i0; i < i1; ++i) {
                        float wi = w[i];
#pragma GCC unroll 8
                        for (int j = 0; j < OR_IL; ++j) a[j] += xb[i * OR_IL + j] * wi;
                    }
                } else if (m->kind == OR_MAT_BF16) {
                    const uint16_t *w = m->bf16 + o * in;
                    for (size_t i = i0; i < i1; ++i) {
                        float wi = bf16_to_f32(w[i]);
#pragma GCC unroll 8
                        for (int j = 0; j < OR_IL; ++j) a[j] += xb[i * OR_IL + j] * wi;
                    }
                } else {
                    const int8_t *q = m->q + o * in;
                    const float *sc = m->scales + o * gpr;
                    for (size_t i = i0; i < i1;) {
                        size_t g = i / group, ge = (g + 1) * group < i1 ? (g + 1) * group : i1;
                        float scale = sc[g];
                        for (; i < ge; ++i) {
                            float wi = (float)q[i] * scale;
#pragma GCC unroll 8
                            for (int j = 0; j < OR_IL; ++j) a[j] += xb[i * OR_IL + j] * wi;
                        }
                    }
                }
            }
        }
        for (size_t r = 0; r < nr; ++r)
            for (int j = 0; j < OR_IL; ++j)
                if (b * OR_IL + j < t) y[(b * OR_IL + j) * out + o0 + r] = acc[r][j];
    }
    free(xt);
}

/* MatrixRef::project, src/matrix.rs:153-187, extended with a BF16 kind. */
static void project(const or_matrix *m, const float *x, float *y, size_t t, size_t in,
                    size_t out, int lanes) {
    if (g_fast && !lanes && t >= 4) {
        project_tv(m, x, y, t, in, out);
        return;
    }
    if (g_fast && !lanes && out >= OR_IL) {
        /* whole blocks interleaved, the tail rows below one at a time */
        project_il(m, x, y, t, in, out);
        size_t done = out / OR_IL * OR_IL;
        if (done == out) return;
        for (size_t tt = 0; tt < t; ++tt) {
            const float *xr = x + tt * in;
            for (size_t o = done; o < out; ++o) {
                float r;
                if (m->kind == OR_MAT_F32) {
                    r = dot_scalar(xr, m->f32 + o * in, in);
                } else if (m->kind == OR_MAT_BF16) {
                    const uint16_t *w = m->bf16 + o * in;
                    r = 0.0f;
                    for (size_t i = 0; i < in; ++i) r += xr[i] * bf16_to_f32(w[i]);
                } else {
                    size_t gpr = in / m->group + (in % m->group != 0);
                    r = dot_int8(xr, m->q + o * in, m->scales + o * gpr, in, m->group);
                }
                y[tt * out + o] = r;
            }
        }
        return;
    }
    long long n = (long long)(t * out);
#pragma omp parallel for schedule(static) num_threads(or_get_threads()) if (n * (long long)in > 65536)
    for (long long k = 0; k < n; ++k) {
        size_t tt = (size_t)k / out, o = (size_t)k % out;
        const float *xr = x + tt * in;
        float r;
        if (m->kind == OR_MAT_F32) {
            r = lanes ? dot_lanes4(xr, m->f32 + o * in, in) : dot_scalar(xr, m->f32 + o * in, in);
        } else if (m->kind == OR_MAT_BF16) {
            const uint16_t *w = m->bf16 + o * in;
            if (lanes) {
                float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
                size_t bulk = in - in % 4;
                for (size_t i = 0; i < bulk; i += 4) {
                    s0 += xr[i] * bf16_to_f32(w[i]);
                    s1 += xr[i + 1] * bf16_to_f32(w[i + 1]);
                    s2 += xr[i + 2] * bf16_to_f32(w[i + 2]);
                    s3 += xr[i + 3] * bf16_to_f32(w[i + 3]);
                }
                r = ((s0 + s1) + s2) + s3;
                for (size_t i = bulk; i < in; ++i) r += xr[i] * bf16_to_f32(w[i]);
            } else {
                r = 0.0f;
                for (size_t i = 0; i < in; ++i) r += xr[i] * bf16_to_f32(w[i]);
            }
        } else {
            size_t gpr = in / m->group + (in % m->group != 0);
            const int8_t *q = m->q + o * in;
            const float *s = m->scales + o * gpr;
            r = lanes ? dot_int8_lanes4(xr, q, s, in, m->group) : dot_int8(xr, q, s, in, m->group);
        }
        y[tt * out + o] = r;
    }
}

/* MatrixRef::gather, src/matrix.rs:188-241 (the INT8 row is dequantized). */
static void gather_row(const or_matrix *m, size_t id, size_t width, float *y) {
    if (m->kind == OR_MAT_F32) {
        memcpy(y, m->f32 + id * width, width * 4);
    } else if (m->kind == OR_MAT_BF16) {
        for (size_t i = 0; i < width; ++i) y[i] = bf16_to_f32(m->bf16[id * width + i]);
    } else {
        size_t gpr = width / m->group + (width % m->group != 0);
        for (size_t i = 0; i < width; ++i)
            y[i] = (float)m->q[id * width + i] * m->scales[id * gpr + i / m->group];
    }
}

/* ------------------------------------------------------------------ */
/* model                                                               */
/* ------------------------------------------------------------------ */

typedef struct or_model {
    or_config c;
    or_matrix embedding;
    or_matrix lm_head; /* kind OR_MAT_NONE = tied to the embedding */
    const float *final_norm;
    or_layer *layers;
} or_model;

or_model *or_model_new(const or_config *c) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->c = *c;
    m->layers = (or_layer *)calloc(c->layers, sizeof(or_layer));
    m->lm_head.kind = OR_MAT_NONE;
    return m;
}

void or_model_free(or_model *m) {
    if (!m) return;
    free(m->layers);
    free(m);
}

/* Stores pointers only; the caller keeps the arrays alive. */
void or_model_set_matrix(or_model *m, long layer, int which, const or_matrix *mat) {
    if (layer < 0) {
        if (which == OR_W_EMBEDDING) m->embedding = *mat;
        else if (which == OR_W_LM_HEAD) m->lm_head = *mat;
        return;
    }
    or_layer *l = &m->layers[layer];
    or_matrix *dst[] = {&l->q, &l->k, &l->v, &l->o, &l->gate, &l->up, &l->down};
    if (which >= OR_W_Q && which <= OR_W_DOWN) *dst[which - OR_W_Q] = *mat;
}

void or_model_set_vector(or_model *m, long layer, int which, const float *v) {
    if (layer < 0) {
        if (which == OR_V_FINAL_NORM) m->final_norm = v;
        return;
    }
    or_layer *l = &m->layers[layer];
    switch (which) {
    case OR_V_ATTN_NORM: l->attn_norm = v; break;
    case OR_V_FFN_NORM: l->ffn_norm = v; break;
    case OR_V_Q_BIAS: l->qb = v; break;
    case OR_V_K_BIAS: l->kb = v; break;
    case OR_V_V_BIAS: l->vb = v; break;
    }
}

static const or_matrix *head_matrix(const or_model *m) {
    return m->lm_head.kind == OR_MAT_NONE ? &m->embedding : &m->lm_head;
}

/* ------------------------------------------------------------------ */
/* uncached forward (src/model.rs:441-591, src/attention.rs:89-276)    */
/* ------------------------------------------------------------------ */

/* Trace layout for `or_forward` when `trace` is non-null (all row-major):
 *   embedding [T,h], then per layer the 16 named activations of
 *   src/model.rs:66-77 / src/attention.rs:33-41 in this order:
 *   attention_norm[T,h] query[T,h] key[T,kv] value[T,kv] rotated_query[T,h]
 *   rotated_key[T,kv] context[T,h] attention_output[T,h] after_attention[T,h]
 *   ffn_norm[T,h] gate[T,ff] up[T,ff] activated_gate[T,ff] product[T,ff]
 *   ffn_output[T,h] output[T,h]; then final_norm[T,h] and logits[T,V]. */
size_t or_trace_len(const or_config *c, size_t T) {
    size_t h = c->hidden, kv = c->kv_heads * c->head_dim, ff = c->ff;
    size_t per = T * (h * 10 + kv * 3 + ff * 4);
    return T * h + c->layers * per + T * h + T * c->vocab;
}

int or_forward(const or_model *m, const size_t *ids, size_t T, float *logits, float *trace) {
    const or_config *c = &m->c;
    size_t h = c->hidden, d = c->head_dim, kv = c->kv_heads * d, ff = c->ff, V = c->vocab;
    if (T == 0 || T > c->max_tokens) return OR_CONTEXT_LIMIT;
    if (trace && T > 32) return OR_TRACE_LIMIT;
    for (size_t t = 0; t < T; ++t) if (ids[t] >= V) return OR_INVALID_TOKEN;
    float *hidden = (float *)calloc(T * h, 4);
    float *an = (float *)calloc(T * h, 4), *q = (float *)calloc(T * h, 4);
    float *k = (float *)calloc(T * kv, 4), *v = (float *)calloc(T * kv, 4);
    float *qr = (float *)calloc(T * h, 4), *kr = (float *)calloc(T * kv, 4);
    float *ctx = (float *)calloc(T * h, 4), *ao = (float *)calloc(T * h, 4);
    float *after = (float *)calloc(T * h, 4), *fn = (float *)calloc(T * h, 4);
    float *gate = (float *)calloc(T * ff, 4), *up = (float *)calloc(T * ff, 4);
    float *act = (float *)calloc(T * ff, 4), *prod = (float *)calloc(T * ff, 4);
    float *fo = (float *)calloc(T * h, 4), *next = (float *)calloc(T * h, 4);
    float *scores = (float *)calloc(T, 4), *probs = (float *)calloc(T, 4);
    int status = OR_OK;
    float *tp = trace;
#define TRACE(buf, n)                         \
    do {                                      \
        if (tp) { memcpy(tp, buf, (n) * 4); tp += (n); } \
    } while (0)
    for (size_t t = 0; t < T; ++t) gather_row(&m->embedding, ids[t], h, hidden + t * h);
    TRACE(hidden, T * h);
    size_t group = c->query_heads / c->kv_heads;
    float scale = sqrtf((float)d);
    for (size_t li = 0; li < c->layers && !status; ++li) {
        const or_layer *l = &m->layers[li];
        for (size_t t = 0; t < T; ++t) rms_row(hidden + t * h, l->attn_norm, an + t * h, h, c->norm_eps);
        /* causal_attention, src/attention.rs:196-276 */
        project(&l->q, an, q, T, h, h, 0);
        project(&l->k, an, k, T, h, kv, 0);
        project(&l->v, an, v, T, h, kv, 0);
        for (size_t t = 0; t < T; ++t) {
            if (l->qb) for (size_t i = 0; i < h; ++i) q[t * h + i] += l->qb[i];
            if (l->kb) for (size_t i = 0; i < kv; ++i) k[t * kv + i] += l->kb[i];
            if (l->vb) for (size_t i = 0; i < kv; ++i) v[t * kv + i] += l->vb[i];
        }
        if (!finite_all(q, T * h) || !finite_all(k, T * kv) || !finite_all(v, T * kv)) { status = OR_NONFINITE; break; }
        if ((status = or_rope(q, T * h, qr, T * h, T, c->query_heads, d, 0, c->rope_base, NULL))) break;
        if ((status = or_rope(k, T * kv, kr, T * kv, T, c->kv_heads, d, 0, c->rope_base, NULL))) break;
        memset(ctx, 0, T * h * 4);
        for (size_t t = 0; t < T; ++t) {
            for (size_t qh = 0; qh < c->query_heads; ++qh) {
                size_t kvh = qh / group, qo = t * h + qh * d;
                for (size_t p = 0; p <= t; ++p) {
                    size_t ko = p * kv + kvh * d;
                    float dot = 0.0f;
                    for (size_t i = 0; i < d; ++i) dot += qr[qo + i] * kr[ko + i];
                    scores[p] = dot / scale;
                }
                if ((status = or_softmax(scores, t + 1, NULL, 0, probs, t + 1, 1, t + 1, NULL))) break;
                for (size_t p = 0; p <= t; ++p) {
                    size_t vo = p * kv + kvh * d;
                    for (size_t i = 0; i < d; ++i) ctx[qo + i] += probs[p] * v[vo + i];
                }
            }
            if (status) break;
        }
        if (status) break;
        if (!finite_all(ctx, T * h)) { status = OR_NONFINITE; break; }
        project(&l->o, ctx, ao, T, h, h, 0);
        if (!finite_all(ao, T * h)) { status = OR_NONFINITE; break; }
        for (size_t i = 0; i < T * h; ++i) after[i] = hidden[i] + ao[i];
        for (size_t t = 0; t < T; ++t) {
            if (!finite_all(after + t * h, h)) { status = OR_NONFINITE; break; }
            rms_row(after + t * h, l->ffn_norm, fn + t * h, h, c->norm_eps);
        }
        if (status) break;
        project(&l->gate, fn, gate, T, h, ff, 0);
        project(&l->up, fn, up, T, h, ff, 0);
        if (!finite_all(gate, T * ff)) { status = OR_NONFINITE; break; }
        for (size_t i = 0; i < T * ff; ++i) act[i] = silu1(gate[i]);
        for (size_t i = 0; i < T * ff; ++i) prod[i] = act[i] * up[i];
        if (!finite_all(prod, T * ff)) { status = OR_NONFINITE; break; }
        project(&l->down, prod, fo, T, ff, h, 0);
        for (size_t i = 0; i < T * h; ++i) next[i] = after[i] + fo[i];
        if (!finite_all(next, T * h)) { status = OR_NONFINITE; break; }
        TRACE(an, T * h); TRACE(q, T * h); TRACE(k, T * kv); TRACE(v, T * kv);
        TRACE(qr, T * h); TRACE(kr, T * kv); TRACE(ctx, T * h); TRACE(ao, T * h);
        TRACE(after, T * h); TRACE(fn, T * h); TRACE(gate, T * ff); TRACE(up, T * ff);
        TRACE(act, T * ff); TRACE(prod, T * ff); TRACE(fo, T * h); TRACE(next, T * h);
        memcpy(hidden, next, T * h * 4);
    }
    if (!status) {
        for (size_t t = 0; t < T; ++t) {
            if (!finite_all(hidden + t * h, h)) { status = OR_NONFINITE; break; }
            rms_row(hidden + t * h, m->final_norm, fn + t * h, h, c->norm_eps);
        }
    }
    if (!status) {
        TRACE(fn, T * h);
        if (tp) {
            project(head_matrix(m), fn, tp, T, h, V, 1);
            if (!finite_all(tp, T * V)) status = OR_NONFINITE;
            if (logits) memcpy(logits, tp + (T - 1) * V, V * 4);
        } else {
            project(head_matrix(m), fn + (T - 1) * h, logits, 1, h, V, 1);
            if (!finite_all(logits, V)) status = OR_NONFINITE;
        }
    }
#undef TRACE
    free(hidden); free(an); free(q); free(k); free(v); free(qr); free(kr); free(ctx); free(ao);
    free(after); free(fn); free(gate); free(up); free(act); free(prod); free(fo); free(next);
    free(scores); free(probs);
    return status;
}

/* ------------------------------------------------------------------ */
/* cached session (src/kv_cache.rs)                                    */
/* ------------------------------------------------------------------ */

typedef struct or_session {
    const or_model *m;
    size_t capacity, processed;
    int valid, kv_bf16;
    float *key, *value; /* [layer][kv_head][capacity][head_dim] */
    float *hidden, *norm, *resid, *ffn, *gate, *up, *act;
    float *q, *k, *v, *qr, *kr, *ctx, *out, *scores, *probs;
    size_t logical_bytes, workspace_bytes;
} or_session;

/* workspace_bytes, src/kv_cache.rs:114-127. */
size_t or_workspace_bytes(const or_config *c, size_t capacity) {
    return (c->hidden * 8 + c->kv_heads * c->head_dim * 3 + c->ff * 3 + capacity * 2) * 4;
}

/* CachedSession::new, src/kv_cache.rs:167-200; `budget` = 0 disables the
 * 128 MiB KV-plus-workspace bound (the reference always applies it). */
int or_session_new(const or_model *m, size_t capacity, int kv_bf16, size_t budget,
                   or_session **out) {
    const or_config *c = &m->c;
    if (capacity == 0 || capacity > c->max_tokens) return OR_INVALID_CAPACITY;
    size_t per = c->kv_heads * capacity * c->head_dim;
    size_t logical = per * 2 * c->layers * 4;
    size_t ws = or_workspace_bytes(c, capacity);
    if (budget && logical + ws > budget) return OR_RESOURCE_BUDGET;
    or_session *s = (or_session *)calloc(1, sizeof(or_session));
    s->m = m;
    s->capacity = capacity;
    s->valid = 1;
    s->kv_bf16 = kv_bf16;
    s->key = (float *)calloc(per * c->layers, 4);
    s->value = (float *)calloc(per * c->layers, 4);
    size_t h = c->hidden, kv = c->kv_heads * c->head_dim, ff = c->ff;
    s->hidden = (float *)calloc(h, 4); s->norm = (float *)calloc(h, 4);
    s->resid = (float *)calloc(h, 4); s->ffn = (float *)calloc(h, 4);
    s->gate = (float *)calloc(ff, 4); s->up = (float *)calloc(ff, 4); s->act = (float *)calloc(ff, 4);
    s->q = (float *)calloc(h, 4); s->k = (float *)calloc(kv, 4); s->v = (float *)calloc(kv, 4);
    s->qr = (float *)calloc(h, 4); s->kr = (float *)calloc(kv, 4);
    s->ctx = (float *)calloc(h, 4); s->out = (float *)calloc(h, 4);
    s->scores = (float *)calloc(capacity, 4); s->probs = (float *)calloc(capacity, 4);
    s->logical_bytes = logical;
    s->workspace_bytes = ws;
    *out = s;
    return OR_OK;
}

void or_session_free(or_session *s) {
    if (!s) return;
    free(s->key); free(s->value); free(s->hidden); free(s->norm); free(s->resid); free(s->ffn);
    free(s->gate); free(s->up); free(s->act); free(s->q); free(s->k); free(s->v); free(s->qr);
    free(s->kr); free(s->ctx); free(s->out); free(s->scores); free(s->probs);
    free(s);
}

size_t or_session_processed(const or_session *s) { return s->processed; }
int or_session_is_valid(const or_session *s) { return s->valid; }
size_t or_session_logical_bytes(const or_session *s) { return s->logical_bytes; }
size_t or_session_workspace_bytes(const or_session *s) { return s->workspace_bytes; }
/* CachedSession::reset, src/kv_cache.rs:225-229. */
void or_session_reset(or_session *s) { s->processed = 0; s->valid = 1; }

/* The per-token body of attend_one after the q/k/v projections
 * (src/kv_cache.rs:505-576): biases, RoPE at `pos`, the cache write at
 * `pos`, then scores, softmax and context over positions 0..pos.  q, k, v
 * hold this token's projections (biases added in place); qr, kr are
 * scratch; the context lands in ctx [h]. */
static int attend_core(or_session *s, size_t li, size_t pos, float *q, float *k, float *v, float *qr,
                       float *kr, float *ctx) {
    const or_model *m = s->m;
    const or_config *c = &m->c;
    const or_layer *l = &m->layers[li];
    size_t h = c->hidden, d = c->head_dim, kv = c->kv_heads * d, cap = s->capacity;
    if (l->qb) for (size_t i = 0; i < h; ++i) q[i] += l->qb[i];
    if (!finite_all(q, h)) return OR_NONFINITE;
    if (l->kb) for (size_t i = 0; i < kv; ++i) k[i] += l->kb[i];
    if (!finite_all(k, kv)) return OR_NONFINITE;
    if (l->vb) for (size_t i = 0; i < kv; ++i) v[i] += l->vb[i];
    if (!finite_all(v, kv)) return OR_NONFINITE;
    int st;
    if ((st = or_rope(q, h, qr, h, 1, c->query_heads, d, pos, c->rope_base, NULL))) return st;
    if ((st = or_rope(k, kv, kr, kv, 1, c->kv_heads, d, pos, c->rope_base, NULL))) return st;
    if (!finite_all(qr, h) || !finite_all(kr, kv)) return OR_NONFINITE;
    float *K = s->key + li * c->kv_heads * cap * d, *Vc = s->value + li * c->kv_heads * cap * d;
    for (size_t hh = 0; hh < c->kv_heads; ++hh) {
        size_t off = (hh * cap + pos) * d;
        for (size_t i = 0; i < d; ++i) {
            float kk = kr[hh * d + i], vv = v[hh * d + i];
            K[off + i] = s->kv_bf16 ? or_round_bf16(kk) : kk;
            Vc[off + i] = s->kv_bf16 ? or_round_bf16(vv) : vv;
        }
    }
    memset(ctx, 0, h * 4);
    size_t group = c->query_heads / c->kv_heads;
    float scale = sqrtf((float)d);
    if (g_fast && pos >= 256) {
        /* heads in parallel (each head's sums unchanged), own score buffers */
        int bad = 0;
        float *buf = (float *)malloc(2 * (pos + 1) * c->query_heads * sizeof(float));
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
        for (long long qi = 0; qi < (long long)c->query_heads; ++qi) {
            size_t qh = (size_t)qi, kvh = qh / group;
            float *sc = buf + 2 * (pos + 1) * qh, *pr = sc + (pos + 1);
            for (size_t p = 0; p <= pos; ++p) {
                size_t off = (kvh * cap + p) * d;
                float sum = 0.0f;
                for (size_t i = 0; i < d; ++i) sum += qr[qh * d + i] * K[off + i];
                sc[p] = sum / scale;
            }
            if (or_softmax(sc, pos + 1, NULL, 0, pr, pos + 1, 1, pos + 1, NULL)) {
#pragma omp atomic write
                bad = 1;
                continue;
            }
            for (size_t p = 0; p <= pos; ++p) {
                size_t off = (kvh * cap + p) * d;
                for (size_t i = 0; i < d; ++i) ctx[qh * d + i] += pr[p] * Vc[off + i];
            }
        }
        free(buf);
        if (bad) return OR_NONFINITE;
    } else {
        for (size_t qh = 0; qh < c->query_heads; ++qh) {
            size_t kvh = qh / group;
            for (size_t p = 0; p <= pos; ++p) {
                size_t off = (kvh * cap + p) * d;
                float sum = 0.0f;
                for (size_t i = 0; i < d; ++i) sum += qr[qh * d + i] * K[off + i];
                s->scores[p] = sum / scale;
            }
            if ((st = or_softmax(s->scores, pos + 1, NULL, 0, s->probs, pos + 1, 1, pos + 1, NULL))) return st;
            for (size_t p = 0; p <= pos; ++p) {
                size_t off = (kvh * cap + p) * d;
                for (size_t i = 0; i < d; ++i) ctx[qh * d + i] += s->probs[p] * Vc[off + i];
            }
        }
    }
    if (!finite_all(ctx, h)) return OR_NONFINITE;
    return OR_OK;
}

/* attend_one, src/kv_cache.rs:479-590. */
static int attend_one(or_session *s, size_t li, const float *x) {
    const or_model *m = s->m;
    const or_config *c = &m->c;
    const or_layer *l = &m->layers[li];
    size_t h = c->hidden, kv = c->kv_heads * c->head_dim;
    project(&l->q, x, s->q, 1, h, h, 0);
    project(&l->k, x, s->k, 1, h, kv, 0);
    project(&l->v, x, s->v, 1, h, kv, 0);
    int st = attend_core(s, li, s->processed, s->q, s->k, s->v, s->qr, s->kr, s->ctx);
    if (st) return st;
    project(&l->o, s->ctx, s->out, 1, h, h, 0);
    if (!finite_all(s->out, h)) return OR_NONFINITE;
    return OR_OK;
}

/* CachedSession::forward, src/kv_cache.rs:347-475. */
static int session_forward(or_session *s, size_t token, float *logits) {
    const or_model *m = s->m;
    const or_config *c = &m->c;
    size_t h = c->hidden, ff = c->ff;
    gather_row(&m->embedding, token, h, s->hidden);
    for (size_t li = 0; li < c->layers; ++li) {
        const or_layer *l = &m->layers[li];
        if (!finite_all(s->hidden, h)) return OR_NONFINITE;
        rms_row(s->hidden, l->attn_norm, s->norm, h, c->norm_eps);
        int st = attend_one(s, li, s->norm);
        if (st) return st;
        for (size_t i = 0; i < h; ++i) s->resid[i] = s->hidden[i] + s->out[i];
        if (!finite_all(s->resid, h)) return OR_NONFINITE;
        rms_row(s->resid, l->ffn_norm, s->norm, h, c->norm_eps);
        project(&l->gate, s->norm, s->gate, 1, h, ff, 0);
        project(&l->up, s->norm, s->up, 1, h, ff, 0);
        if (!finite_all(s->gate, ff)) return OR_NONFINITE;
        for (size_t i = 0; i < ff; ++i) s->act[i] = silu1(s->gate[i]);
        for (size_t i = 0; i < ff; ++i) s->act[i] *= s->up[i];
        if (!finite_all(s->act, ff)) return OR_NONFINITE;
        project(&l->down, s->act, s->ffn, 1, ff, h, 0);
        for (size_t i = 0; i < h; ++i) s->hidden[i] = s->resid[i] + s->ffn[i];
        if (!finite_all(s->hidden, h)) return OR_NONFINITE;
    }
    rms_row(s->hidden, m->final_norm, s->norm, h, c->norm_eps);
    project(head_matrix(m), s->norm, logits, 1, h, c->vocab, 1);
    if (!finite_all(logits, c->vocab)) return OR_NONFINITE;
    return OR_OK;
}

/* step_inner, src/kv_cache.rs:317-346: admission leaves state unchanged;
 * an execution error invalidates the session and zeroes `processed`. */
int or_session_step(or_session *s, size_t token, float *logits, size_t logits_len) {
    if (!s->valid) return OR_INVALID_STATE;
    if (logits_len != s->m->c.vocab) return OR_INVALID_OUTPUT_LENGTH;
    if (token >= s->m->c.vocab) return OR_INVALID_TOKEN;
    if (s->processed == s->capacity) return OR_FULL;
    int st = session_forward(s, token, logits);
    if (st) {
        s->valid = 0;
        s->processed = 0;
        return st;
    }
    s->processed += 1;
    return OR_OK;
}

/* append_into, src/kv_cache.rs:249-280 (prefill_into adds the empty check). */
int or_session_append(or_session *s, const size_t *tokens, size_t n, float *logits,
                      size_t logits_len, int require_empty) {
    if (!s->valid) return OR_INVALID_STATE;
    if (require_empty && s->processed != 0) return OR_NOT_EMPTY;
    if (n == 0) return OR_EMPTY_INPUT;
    if (logits_len != s->m->c.vocab) return OR_INVALID_OUTPUT_LENGTH;
    for (size_t i = 0; i < n; ++i) if (tokens[i] >= s->m->c.vocab) return OR_INVALID_TOKEN;
    if (s->processed + n > s->capacity) return OR_FULL;
    for (size_t i = 0; i < n; ++i) {
        int st = or_session_step(s, tokens[i], logits, logits_len);
        if (st) return st;
    }
    return OR_OK;
}

/* The same evaluation as or_session_append (every per-token value
 * bit-identical: the same dots, norms and attention in the same order),
 * organised layer-major over chunks of up to `chunk` tokens so each weight
 * row is read once per chunk, for the long prompts of the parity tests.
 * Differences: intermediate tokens' logits are not computed (only the last
 * token's), and any non-finite value makes the chunk run again token by
 * token through or_session_step, whose error semantics then apply. */
int or_session_append_chunked(or_session *s, const size_t *tokens, size_t n, float *logits,
                              size_t logits_len, int require_empty, size_t chunk) {
    if (!s->valid) return OR_INVALID_STATE;
    if (require_empty && s->processed != 0) return OR_NOT_EMPTY;
    if (n == 0) return OR_EMPTY_INPUT;
    if (logits_len != s->m->c.vocab) return OR_INVALID_OUTPUT_LENGTH;
    for (size_t i = 0; i < n; ++i) if (tokens[i] >= s->m->c.vocab) return OR_INVALID_TOKEN;
    if (s->processed + n > s->capacity) return OR_FULL;
    if (chunk == 0) chunk = 64;
    const or_model *m = s->m;
    const or_config *c = &m->c;
    size_t h = c->hidden, kv = c->kv_heads * c->head_dim, ff = c->ff, T = chunk < n ? chunk : n;
    float *H = (float *)malloc(T * h * 4), *N = (float *)malloc(T * h * 4), *R = (float *)malloc(T * h * 4);
    float *Q = (float *)malloc(T * h * 4), *K = (float *)malloc(T * kv * 4), *Vv = (float *)malloc(T * kv * 4);
    float *X = (float *)malloc(T * h * 4), *O = (float *)malloc(T * h * 4);
    float *G = (float *)malloc(T * ff * 4), *U = (float *)malloc(T * ff * 4), *A = (float *)malloc(T * ff * 4);
    int status = OR_OK;
    for (size_t c0 = 0; c0 < n && !status; c0 += T) {
        size_t nt = n - c0 < T ? n - c0 : T, pos0 = s->processed;
        int bad = 0;
        for (size_t t = 0; t < nt; ++t) gather_row(&m->embedding, tokens[c0 + t], h, H + t * h);
        for (size_t li = 0; li < c->layers && !bad; ++li) {
            const or_layer *l = &m->layers[li];
            if (!finite_all(H, nt * h)) { bad = 1; break; }
            for (size_t t = 0; t < nt; ++t) rms_row(H + t * h, l->attn_norm, N + t * h, h, c->norm_eps);
            project(&l->q, N, Q, nt, h, h, 0);
            project(&l->k, N, K, nt, h, kv, 0);
            project(&l->v, N, Vv, nt, h, kv, 0);
            for (size_t t = 0; t < nt && !bad; ++t)
                bad = attend_core(s, li, pos0 + t, Q + t * h, K + t * kv, Vv + t * kv, s->qr, s->kr, X + t * h) != OR_OK;
            if (bad) break;
            project(&l->o, X, O, nt, h, h, 0);
            if (!finite_all(O, nt * h)) { bad = 1; break; }
            for (size_t i = 0; i < nt * h; ++i) R[i] = H[i] + O[i];
            if (!finite_all(R, nt * h)) { bad = 1; break; }
            for (size_t t = 0; t < nt; ++t) rms_row(R + t * h, l->ffn_norm, N + t * h, h, c->norm_eps);
            project(&l->gate, N, G, nt, h, ff, 0);
            project(&l->up, N, U, nt, h, ff, 0);
            if (!finite_all(G, nt * ff)) { bad = 1; break; }
            for (size_t i = 0; i < nt * ff; ++i) A[i] = silu1(G[i]);
            for (size_t i = 0; i < nt * ff; ++i) A[i] *= U[i];
            if (!finite_all(A, nt * ff)) { bad = 1; break; }
            project(&l->down, A, O, nt, ff, h, 0);
            for (size_t i = 0; i < nt * h; ++i) H[i] = R[i] + O[i];
            if (!finite_all(H, nt * h)) { bad = 1; break; }
        }
        if (!bad && c0 + nt == n) {
            rms_row(H + (nt - 1) * h, m->final_norm, N, h, c->norm_eps);
            project(head_matrix(m), N, logits, 1, h, c->vocab, 1);
            bad = !finite_all(logits, c->vocab);
        }
        if (bad) {
            /* the serial path, from the same state (processed is unchanged) */
            for (size_t t = 0; t < nt && !status; ++t)
                status = or_session_step(s, tokens[c0 + t], logits, logits_len);
        } else {
            s->processed += nt;
        }
    }
    free(H); free(N); free(R); free(Q); free(K); free(Vv); free(X); free(O); free(G); free(U); free(A);
    return status;
}

/* Greedy argmax with a strict `>`, so the lowest id wins ties
 * (src/sampling.rs:65-70, src/generation.rs:60-65). */
size_t or_argmax(const float *logits, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* Cached greedy token loop: serial prefill of the prompt, then `max_new`
 * emissions, each followed (except the last) by one cached step; stops on a
 * stop token.  Equivalent to GenerationSession::{start,next_token},
 * src/generation.rs:139-170,258-337, with greedy sampling.  Returns the
 * number of generated ids written to `out` (or a negative status). */
long or_greedy(or_session *s, const size_t *prompt, size_t n, const size_t *stops, size_t nstops,
               size_t max_new, size_t *out) {
    size_t V = s->m->c.vocab;
    float *logits = (float *)malloc(V * 4);
    int st = or_session_append(s, prompt, n, logits, V, 1);
    if (st) { free(logits); return -(long)st; }
    size_t g = 0;
    for (;;) {
        size_t next = or_argmax(logits, V);
        out[g++] = next;
        int stop = 0;
        for (size_t i = 0; i < nstops; ++i) if (stops[i] == next) stop = 1;
        if (stop || g == max_new) break;
        st = or_session_step(s, next, logits, V);
        if (st) { free(logits); return -(long)st; }
    }
    free(logits);
    return (long)g;
}

/* Last evaluated logits of a whole history via the uncached path:
 * uncached_greedy, src/generation.rs:27-81. */
long or_uncached_greedy(const or_model *m, const size_t *prompt, size_t n, const size_t *stops,
                        size_t nstops, size_t max_new, size_t *out) {
    const or_config *c = &m->c;
    if (n == 0) return -(long)OR_EMPTY_PROMPT;
    if (max_new == 0) return -(long)OR_OUTPUT_LIMIT;
    for (size_t i = 0; i < n; ++i) if (prompt[i] >= c->vocab) return -(long)OR_INVALID_TOKEN;
    for (size_t i = 0; i < nstops; ++i) if (stops[i] >= c->vocab) return -(long)OR_INVALID_TOKEN;
    if (max_new > SIZE_MAX - n || n + max_new > c->max_tokens) return -(long)OR_CONTEXT_LIMIT;
    size_t *hist = (size_t *)malloc((n + max_new) * sizeof(size_t));
    memcpy(hist, prompt, n * sizeof(size_t));
    float *logits = (float *)malloc(c->vocab * 4);
    size_t len = n, g = 0;
    for (size_t step = 0; step < max_new; ++step) {
        int st = or_forward(m, hist, len, logits, NULL);
        if (st) { free(hist); free(logits); return -(long)st; }
        size_t next = or_argmax(logits, c->vocab);
        hist[len++] = next;
        out[g++] = next;
        int stop = 0;
        for (size_t i = 0; i < nstops; ++i) if (stops[i] == next) stop = 1;
        if (stop) break;
    }
    free(hist);
    free(logits);
    return (long)g;
}

/* ------------------------------------------------------------------ */
/* Synthetic inputs (not a reference function).  Every value is a pure  */
/* function of (seed, stream, index):                                   */
/*   mix(z)   = splitmix64 finalizer of z + 0x9E3779B97F4A7C15          */
/*   base     = mix(seed * 0x100000001B3 ^ mix(stream))                  */
/*   pair k   : a = mix(base + 2k), b = mix(base + 2k + 1),              */
/*              u1 = ((a >> 11) + 1) 2^-53, u2 = (b >> 11) 2^-53,        */
/*              r = sqrt(-2 ln u1), z0 = r cos(2 pi u2), z1 = r sin(..)  */
/*   element 2k + e = (float)(z_e * stddev) (then BF16 nearest-even)     */
/*   token i  : mix(base + i) mod vocab                                  */
/* ------------------------------------------------------------------ */

static uint64_t syn_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t syn_base(uint64_t seed, uint64_t stream) {
    return syn_mix(seed * 0x100000001B3ull ^ syn_mix(stream));
}

int or_synthetic_normal(uint64_t seed, uint64_t stream, size_t n, double stddev, int out_dtype,
                        void *out) {
    if ((!out && n) || (out_dtype != 0 && out_dtype != 1)) return OR_INVALID_LENGTH;
    const uint64_t base = syn_base(seed, stream);
    const long long pairs = (long long)((n + 1) / 2);
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long long k = 0; k < pairs; ++k) {
        uint64_t a = syn_mix(base + 2 * (uint64_t)k), b = syn_mix(base + 2 * (uint64_t)k + 1);
        double u1 = (double)((a >> 11) + 1) * (1.0 / 9007199254740992.0);
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        double z[2] = {r * cos(two_pi * u2), r * sin(two_pi * u2)};
        for (int e = 0; e < 2; ++e) {
            size_t i = 2 * (size_t)k + e;
            if (i >= n) break;
            float v = (float)(z[e] * stddev);
            if (out_dtype == 0) {
                ((float *)out)[i] = v;
            } else {
                float r16 = or_round_bf16(v);
                uint32_t u;
                memcpy(&u, &r16, 4);
                ((uint16_t *)out)[i] = (uint16_t)(u >> 16);
            }
        }
    }
    return OR_OK;
}

int or_synthetic_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab, uint32_t *out) {
    if (vocab == 0 || (!out && n)) return OR_INVALID_LENGTH;
    const uint64_t base = syn_base(seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)(syn_mix(base + i) % vocab);
    return OR_OK;
}

/* ------------------------------------------------------------------ */
/* seeded temperature / top-k sampling (src/sampling.rs:71-110)        */
/* ------------------------------------------------------------------ */
/* The reference draws from rand_chacha 0.9.0's ChaCha8Rng seeded by
 * rand_core 0.9.5's SeedableRng::seed_from_u64 (neither is vendored in the
 * reference tree).  Restated from their published algorithms: the ChaCha
 * block function (RFC 7539 quarter rounds, 8 rounds = 4 double rounds,
 * 64-bit block counter in words 12-13, stream 0 in words 14-15, key words
 * little-endian from the 32-byte seed, output = keystream words in block
 * order); seed_from_u64 fills the seed 4 bytes at a time with a PCG32 step
 * (state = state * 6364136223846793005 + 11634580027462260723, output
 * rotr(((state >> 18) ^ state) >> 27, state >> 59), little-endian);
 * next_u64 = word[i] | word[i + 1] << 32; random::<f64>() =
 * (next_u64 >> 11) * 2^-53. */

static uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

/* The ChaCha block function: `rounds` rounds over `in`, plus the input. */
void or_chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]) {
    uint32_t x[16];
    memcpy(x, in, sizeof(x));
#define QR(a, b, c, d)                                              \
    x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl32(x[d], 16);            \
    x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl32(x[b], 12);            \
    x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl32(x[d], 8);             \
    x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl32(x[b], 7);
    for (int r = 0; r < rounds; r += 2) {
        QR(0, 4, 8, 12) QR(1, 5, 9, 13) QR(2, 6, 10, 14) QR(3, 7, 11, 15)
        QR(0, 5, 10, 15) QR(1, 6, 11, 12) QR(2, 7, 8, 13) QR(3, 4, 9, 14)
    }
#undef QR
    for (int i = 0; i < 16; ++i) out[i] = x[i] + in[i];
}

/* ChaCha8Rng::from_seed: the key words are the seed's little-endian words;
 * block counter and stream start at 0. */
void or_rng_from_seed(or_rng *g, const uint8_t seed[32]) {
    for (int i = 0; i < 8; ++i)
        g->key[i] = (uint32_t)seed[4 * i] | (uint32_t)seed[4 * i + 1] << 8 | (uint32_t)seed[4 * i + 2] << 16 |
                    (uint32_t)seed[4 * i + 3] << 24;
    g->counter = 0;
    g->index = 64;  /* empty buffer */
}

void or_rng_seed(or_rng *g, uint64_t seed) {
    uint8_t bytes[32];
    uint64_t state = seed;
    for (int i = 0; i < 8; ++i) {
        state = state * 6364136223846793005ull + 11634580027462260723ull;
        uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27);
        uint32_t rot = (uint32_t)(state >> 59);
        uint32_t x = (xs >> rot) | (xs << ((32 - rot) & 31));
        for (int b = 0; b < 4; ++b) bytes[4 * i + b] = (uint8_t)(x >> (8 * b));
    }
    or_rng_from_seed(g, bytes);
}

static void rng_refill(or_rng *g) {
    for (int b = 0; b < 4; ++b) {
        uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
        for (int i = 0; i < 8; ++i) in[4 + i] = g->key[i];
        uint64_t c = g->counter + (uint64_t)b;
        in[12] = (uint32_t)c;
        in[13] = (uint32_t)(c >> 32);
        in[14] = 0;
        in[15] = 0;
        or_chacha_block(in, 8, g->buf + 16 * b);
    }
    g->counter += 4;
    g->index = 0;
}

uint64_t or_rng_next_u64(or_rng *g) {
    if (g->index >= 64) rng_refill(g);
    /* the index is always even here: only whole u64 draws are made */
    uint64_t v = (uint64_t)g->buf[g->index] | ((uint64_t)g->buf[g->index + 1] << 32);
    g->index += 2;
    return v;
}

double or_rng_next_f64(or_rng *g) { return (double)(or_rng_next_u64(g) >> 11) * (1.0 / 9007199254740992.0); }

/* Sampler::new, src/sampling.rs:23-41 (greedy: temperature ignored). */
int or_sampler_init(or_sampler *s, int greedy, float temperature, size_t top_k, uint64_t seed) {
    if (!greedy && (!isfinite(temperature) || temperature <= 0.0f || top_k == 0)) return OR_INVALID_PARAMETERS;
    s->greedy = greedy;
    s->temperature = temperature;
    s->top_k = top_k;
    s->seed = greedy ? 0 : seed;
    or_rng_seed(&s->rng, s->seed);
    return OR_OK;
}

void or_sampler_reset(or_sampler *s) { or_rng_seed(&s->rng, s->seed); }

/* Sampler::validate_vocab, src/sampling.rs:43-49. */
int or_sampler_validate_vocab(const or_sampler *s, size_t vocab) {
    return (vocab == 0 || (!s->greedy && s->top_k > vocab)) ? OR_INVALID_PARAMETERS : OR_OK;
}

static const float *g_cmp_logits;
static int cmp_desc_id(const void *pa, const void *pb) {
    size_t a = *(const size_t *)pa, b = *(const size_t *)pb;
    float la = g_cmp_logits[a], lb = g_cmp_logits[b];
    if (lb > la) return 1;  /* logits[b].partial_cmp(&logits[a]) then id order */
    if (lb < la) return -1;
    return a < b ? -1 : (a > b ? 1 : 0);
}

/* Sampler::sample, src/sampling.rs:48-110. */
int or_sampler_sample(or_sampler *s, const float *logits, size_t n, size_t *out) {
    if (n == 0) return OR_EMPTY_LOGITS;
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(logits[i])) return OR_NONFINITE;
    if (or_sampler_validate_vocab(s, n)) return OR_INVALID_PARAMETERS;
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (logits[i] > logits[best]) best = i;
    if (s->greedy) { *out = best; return OR_OK; }
    /* The top-k in (logit desc, id asc) order: a full sort's first k equals
     * select_nth + truncate + sort under the same total order. */
    size_t *cand = (size_t *)malloc(n * sizeof(size_t));
    for (size_t i = 0; i < n; ++i) cand[i] = i;
    g_cmp_logits = logits;
    qsort(cand, n, sizeof(size_t), cmp_desc_id);
    size_t k = s->top_k < n ? s->top_k : n;
    double maximum = (double)logits[best], temp = (double)s->temperature;
    double total = 0.0;
    for (size_t i = 0; i < k; ++i) total += exp(((double)logits[cand[i]] - maximum) / temp);
    double target = or_rng_next_f64(&s->rng) * total;
    double cumulative = 0.0;
    size_t last_positive = best;
    for (size_t i = 0; i < k; ++i) {
        double w = exp(((double)logits[cand[i]] - maximum) / temp);
        if (w > 0.0) last_positive = cand[i];
        cumulative += w;
        if (target < cumulative) { *out = cand[i]; free(cand); return OR_OK; }
    }
    free(cand);
    *out = last_positive;
    return OR_OK;
}
