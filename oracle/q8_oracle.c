/*
 * q8_oracle.c -- TEST INFRASTRUCTURE ONLY (see q8_oracle.h).
 *
 * CPU restatement of ggml's Q8_0 arithmetic as synthesize.cpp reaches it:
 *   - packing:            tools/synthesize-quantize/quantize.cpp:300-301
 *                         -> ggml_quantize_chunk -> quantize_row_q8_0_ref
 *                         (restated in gguf-py quants.py:378-394, rounding :43-47)
 *   - MUL_MAT(Q8_0, F32): src/arch/qwen3-tts/operations.cpp:39-41,90-92,142,
 *                         talker.cpp:45,48,184, code-predictor.cpp:79
 *                         -> ggml-cpu: from_float(quantize_row_q8_0) then
 *                            vec_dot_q8_0_q8_0 per output element
 *   - GET_ROWS(Q8_0):     talker.cpp:44,86, code-predictor.cpp:31, model.cpp:1347
 *                         -> dequantize_row_q8_0 (gguf-py quants.py:396-401)
 *   - seeded inputs:      src/random-stream.cpp:10-48 (NormalRandomStream)
 *   - thread policy:      src/cpu-parallelism.cpp:93-99
 *
 * Build with -ffp-contract=off so every fp32 operation rounds where the C
 * source says it does.
 */
#include "q8_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 ---- */

/* IEEE binary32 -> binary16, round to nearest even (what GGML_FP32_TO_FP16
 * does through F16C or its portable fallback).  NaN maps to the canonical
 * quiet NaN 0x7e00 with the sign kept. */
uint16_t oracle_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp  = (x >> 23) & 0xffu;
    uint32_t       mant = x & 0x7fffffu;
    if (exp == 0xffu) {
        return (uint16_t) (sign | (mant ? 0x7e00u : 0x7c00u));
    }
    const int32_t e = (int32_t) exp - 127 + 15;
    if (e >= 31) {
        return (uint16_t) (sign | 0x7c00u);
    }
    if (e <= 0) {
        if (e < -10) {
            return (uint16_t) sign;
        }
        mant |= 0x800000u;
        const uint32_t shift = (uint32_t) (14 - e);
        uint32_t       m     = mant >> shift;
        const uint32_t rem   = mant & ((1u << shift) - 1u);
        const uint32_t half  = 1u << (shift - 1u);
        if (rem > half || (rem == half && (m & 1u))) {
            m++;
        }
        return (uint16_t) (sign | m);
    }
    uint32_t       h   = sign | ((uint32_t) e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
        h++; /* may carry into the exponent, up to infinity: that is correct */
    }
    return (uint16_t) h;
}

float oracle_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = ((uint32_t) h & 0x8000u) << 16;
    uint32_t       exp  = ((uint32_t) h >> 10) & 0x1fu;
    uint32_t       mant = (uint32_t) h & 0x3ffu;
    uint32_t       bits;
    if (exp == 0x1fu) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* subnormal: normalise */
            int e = -1;
            do {
                e++;
                mant <<= 1;
            } while ((mant & 0x400u) == 0);
            bits = sign | ((uint32_t) (127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
        }
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ------------------------------------------------------------ quantize ---- */

/* Converts a rounded code to int8.  Codes normally lie in [-127, 127], but
 * ggml's amax fold skips every value before the block's last NaN, so x*id can
 * be any float.  The reference stores roundf(x*id) straight into an int8_t,
 * undefined in C outside int32 and for non-finite values; gcc on x86 emits
 * cvttss2si, which gives 0x80000000 for NaN, infinities and anything outside
 * [-2^31, 2^31), and keeps the low byte: 0.  Inside int32 the low byte of the
 * integer is kept.  This restatement fixes those outcomes explicitly. */
static int8_t code_from_float(float r) {
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) {
        return 0;
    }
    return (int8_t) (uint8_t) ((uint32_t) (int32_t) r & 0xffu);
}

void oracle_quantize_row_q8_0(const float * x, void * vy, int64_t k, int mode) {
    uint8_t *     y  = (uint8_t *) vy;
    const int64_t nb = k / ORACLE_QK8_0;
    for (int64_t b = 0; b < nb; ++b) {
        const float * xb   = x + b * ORACLE_QK8_0;
        uint8_t *     yb   = y + b * ORACLE_BLOCK_BYTES;
        float         amax = 0.0f;
        for (int j = 0; j < ORACLE_QK8_0; ++j) {
            const float v = fabsf(xb[j]);
            amax          = (amax > v) ? amax : v; /* ggml's MAX(a, b) macro, argument order kept */
        }
        const float d = amax / 127.0f;
        float       id;
        if (mode == ORACLE_QUANT_CPU_X86) {
            id = (amax != 0.0f) ? 127.0f / amax : 0.0f;
        } else {
            id = (d != 0.0f) ? 1.0f / d : 0.0f;
        }
        const uint16_t dh = oracle_fp32_to_fp16(d);
        yb[0]             = (uint8_t) (dh & 0xffu);
        yb[1]             = (uint8_t) (dh >> 8);
        for (int j = 0; j < ORACLE_QK8_0; ++j) {
            const float x0 = xb[j] * id;
            const float r  = (mode == ORACLE_QUANT_REF) ? roundf(x0) : nearbyintf(x0);
            yb[2 + j]      = (uint8_t) code_from_float(r);
        }
    }
}

size_t oracle_quantize_chunk_q8_0(const float * src, void * dst, int64_t start, int64_t nrows, int64_t n_per_row) {
    const size_t  row_size  = (size_t) (n_per_row / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    const int64_t start_row = start / n_per_row;
    uint8_t *     out       = (uint8_t *) dst + (size_t) start_row * row_size;
    for (int64_t r = 0; r < nrows; ++r) {
        oracle_quantize_row_q8_0(src + start + r * n_per_row, out + (size_t) r * row_size, n_per_row,
                                 ORACLE_QUANT_REF);
    }
    return (size_t) nrows * row_size;
}

void oracle_dequantize_row_q8_0(const void * vx, float * y, int64_t k) {
    const uint8_t * x  = (const uint8_t *) vx;
    const int64_t   nb = k / ORACLE_QK8_0;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t * xb = x + b * ORACLE_BLOCK_BYTES;
        const float     d  = oracle_fp16_to_fp32((uint16_t) (xb[0] | (xb[1] << 8)));
        for (int j = 0; j < ORACLE_QK8_0; ++j) {
            y[b * ORACLE_QK8_0 + j] = (float) (int8_t) xb[2 + j] * d;
        }
    }
}

/* ----------------------------------------------------------------- dot ---- */

static inline float block_scale(const uint8_t * b) {
    return oracle_fp16_to_fp32((uint16_t) (b[0] | (b[1] << 8)));
}

float oracle_vec_dot_q8_0_q8_0(int64_t n, const void * vx, const void * vy, double * abs_bound) {
    const uint8_t * x    = (const uint8_t *) vx;
    const uint8_t * y    = (const uint8_t *) vy;
    const int64_t   nb   = n / ORACLE_QK8_0;
    float           sumf = 0.0f;
    double          bnd  = 0.0;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t * xb   = x + b * ORACLE_BLOCK_BYTES;
        const uint8_t * yb   = y + b * ORACLE_BLOCK_BYTES;
        const int8_t *  qx   = (const int8_t *) (xb + 2);
        const int8_t *  qy   = (const int8_t *) (yb + 2);
        int32_t         sumi = 0;
        for (int j = 0; j < ORACLE_QK8_0; ++j) {
            sumi += (int32_t) qx[j] * (int32_t) qy[j];
        }
        const float dd = block_scale(xb) * block_scale(yb);
        sumf += (float) sumi * dd;
        bnd += fabs((double) sumi * (double) dd);
    }
    if (abs_bound) {
        *abs_bound = bnd;
    }
    return sumf;
}

void oracle_mul_mat_q8_0_q8_0(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const void * xq, int64_t M,
                              float * y, size_t y_col_stride, double * bound, int threads) {
    const size_t xq_row = (size_t) (K / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(static)
#endif
    for (int64_t n = 0; n < N; ++n) {
        const uint8_t * wr = (const uint8_t *) w + (size_t) n * w_row_bytes;
        for (int64_t m = 0; m < M; ++m) {
            double b                                                   = 0.0;
            const float v = oracle_vec_dot_q8_0_q8_0(K, wr, (const uint8_t *) xq + (size_t) m * xq_row, &b);
            *(float *) ((uint8_t *) y + (size_t) m * y_col_stride + (size_t) n * sizeof(float)) = v;
            if (bound) {
                bound[m * N + n] = b;
            }
        }
    }
    (void) threads;
}

void oracle_mul_mat_q8_0_f32(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const float * x, int64_t M,
                             size_t x_col_stride, float * y, size_t y_col_stride, int mode, double * bound,
                             int threads) {
    const size_t xq_row = (size_t) (K / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    uint8_t *    xq     = (uint8_t *) malloc(xq_row * (size_t) (M > 0 ? M : 1));
    for (int64_t m = 0; m < M; ++m) {
        oracle_quantize_row_q8_0((const float *) ((const uint8_t *) x + (size_t) m * x_col_stride), xq + m * xq_row,
                                 K, mode);
    }
    oracle_mul_mat_q8_0_q8_0(w, K, N, w_row_bytes, xq, M, y, y_col_stride, bound, threads);
    free(xq);
}

/* ------------------------------------------------------------- get_rows ---- */

int oracle_get_rows_q8_0(const void * table, int64_t K, int64_t rows, const int32_t * ids, int64_t n_ids,
                         float * out) {
    const size_t row_bytes = (size_t) (K / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    int          status    = 0;
    for (int64_t i = 0; i < n_ids; ++i) {
        const int32_t r = ids[i];
        if (r < 0 || r >= rows) {
            memset(out + i * K, 0, (size_t) K * sizeof(float));
            status = -1;
            continue;
        }
        oracle_dequantize_row_q8_0((const uint8_t *) table + (size_t) r * row_bytes, out + i * K, K);
    }
    return status;
}

/* ---------------------------------------------------------------- rng ---- */

typedef struct {
    uint64_t state;
    float    spare;
    int      has_spare;
} oracle_rng;

static uint64_t rng_next_u64(oracle_rng * r) {
    r->state += UINT64_C(0x9e3779b97f4a7c15);
    uint64_t v = r->state;
    v          = (v ^ (v >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    v          = (v ^ (v >> 27)) * UINT64_C(0x94d049bb133111eb);
    return v ^ (v >> 31);
}

static double rng_uniform_open(oracle_rng * r) {
    return ((double) (rng_next_u64(r) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

static float rng_normal(oracle_rng * r) {
    if (r->has_spare) {
        r->has_spare = 0;
        return r->spare;
    }
    double first, second, radius;
    do {
        first  = 2.0 * rng_uniform_open(r) - 1.0;
        second = 2.0 * rng_uniform_open(r) - 1.0;
        radius = first * first + second * second;
    } while (radius >= 1.0 || radius == 0.0);
    const double scale = sqrt(-2.0 * log(radius) / radius);
    r->spare           = (float) (second * scale);
    r->has_spare       = 1;
    return (float) (first * scale);
}

void oracle_normal_fill(uint64_t seed, float * out, size_t count) {
    oracle_rng r = { seed, 0.0f, 0 };
    for (size_t i = 0; i < count; ++i) {
        out[i] = rng_normal(&r);
    }
}

void oracle_uniform_fill(uint64_t seed, float * out, size_t count) {
    oracle_rng r = { seed, 0.0f, 0 };
    for (size_t i = 0; i < count; ++i) {
        out[i] = (float) rng_uniform_open(&r);
    }
}

void oracle_normal_fill_scaled(uint64_t seed, float scale, float * out, size_t count) {
    oracle_rng r = { seed, 0.0f, 0 };
    for (size_t i = 0; i < count; ++i) {
        out[i] = scale * rng_normal(&r);
    }
}

/* Fills n independent tensors, tensor j from its own stream seeds[j] times
 * scales[j]; tensors are spread over OpenMP threads (each stream is still
 * drawn in order, so the values equal oracle_normal_fill_scaled's). */
void oracle_normal_fill_scaled_many(int n, const uint64_t * seeds, const float * scales, float * const * outs,
                                    const size_t * counts, int threads) {
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int j = 0; j < n; ++j) {
        oracle_normal_fill_scaled(seeds[j], scales[j], outs[j], counts[j]);
    }
}

/* oracle_quantize_row_q8_0 over rows rows of k values (dense), rows spread
 * over OpenMP threads; each row's bytes are independent of the split. */
void oracle_quantize_rows_mt(const float * x, void * dst, int64_t rows, int64_t k, int mode, int threads) {
    const size_t row_size = (size_t) (k / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    const int    nt       = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        oracle_quantize_row_q8_0(x + r * k, (uint8_t *) dst + (size_t) r * row_size, k, mode);
    }
}

/* ------------------------------------------------------------ threads ---- */

int oracle_default_synthesis_threads(int available) {
    if (available <= 2) {
        return 1;
    }
    return (available / 2 < available - 1) ? available / 2 : available - 1;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* --------------------------------------------------------- decode chain ---- */

/* rms_norm followed by the elementwise weight: src/arch/qwen3-tts/operations.cpp:31
 * (ggml_rms_norm sums x*x in double, then scale = 1/sqrtf(mean + eps)). */
static void rms_norm_mul(const float * x, const float * w, float * y, int64_t n, float eps) {
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        sum += (double) (x[i] * x[i]);
    }
    const float mean  = (float) (sum / (double) n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; ++i) {
        y[i] = (x[i] * scale) * w[i];
    }
}

static float silu_f32(float x) {
    return x / (1.0f + expf(-x));
}

/* x[r][i] = silu(x[r][i] + b[i]) in fp32: ggml_silu(ggml_add(mul_mat(W1, t), b1))
 * of the talker's text projection (src/arch/qwen3-tts/talker.cpp:45-47). */
void oracle_bias_silu_rows(float * x, const float * b, int64_t rows, int64_t n) {
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t i = 0; i < n; ++i) {
            x[r * n + i] = silu_f32(x[r * n + i] + b[i]);
        }
    }
}

/* Qwen3's per-head RMS norm followed by NEOX RoPE, in place, for one token:
 * x holds n_heads heads of head_dim values (src/arch/qwen3-tts/operations.cpp:
 * 95-101: rms_norm(q, q_norm) then ggml_rope_ext(..., GGML_ROPE_TYPE_NEOX,
 * freq_base = rope_theta, freq_scale 1, ext_factor 0, attn_factor 1)).  The
 * rotation angle follows ggml's published RoPE recurrence: theta_0 = pos,
 * theta_{i+1} = theta_i * base^(-2/head_dim) in fp32; NEOX pairs element i with
 * element i + head_dim/2.  w == NULL skips the norm (v is not normed). */
void oracle_head_norm_rope(float * x, int64_t n_heads, int64_t head_dim, const float * w, float eps, int32_t pos,
                           float theta_base, int rope) {
    float * t = (float *) malloc(sizeof(float) * (size_t) head_dim);
    for (int64_t h = 0; h < n_heads; ++h) {
        float * xh = x + h * head_dim;
        if (w != NULL) {
            rms_norm_mul(xh, w, t, head_dim, eps);
            memcpy(xh, t, sizeof(float) * (size_t) head_dim);
        }
        if (!rope) {
            continue;
        }
        const float   theta_scale = powf(theta_base, -2.0f / (float) head_dim);
        float         theta       = (float) pos;
        const int64_t half        = head_dim / 2;
        for (int64_t i = 0; i < half; ++i) {
            const float c  = cosf(theta);
            const float sn = sinf(theta);
            const float x0 = xh[i];
            const float x1 = xh[i + half];
            t[i]           = x0 * c - x1 * sn;
            t[i + half]    = x0 * sn + x1 * c;
            theta          = theta * theta_scale;
        }
        memcpy(xh, t, sizeof(float) * (size_t) head_dim);
    }
    free(t);
}

/* Single-token attention over npos cached positions (operations.cpp:120-131:
 * scores = K q / sqrt(head_dim), softmax, then the softmax-weighted sum of V),
 * query head h reading kv head h / (n_head / n_kv).  kc / vc hold npos rows of
 * n_kv * head_dim floats.  Sums in double, one rounding to fp32 at the end:
 * the reference's summation order is ggml-cpu's SIMD order, which the GPU
 * does not follow either, so this is the tolerance anchor. */
void oracle_attend(const float * q, const float * kc, const float * vc, int64_t npos, int64_t n_head, int64_t n_kv,
                   int64_t head_dim, float * out) {
    const int64_t group  = n_head / n_kv;
    const int64_t kv_dim = n_kv * head_dim;
    const double  scale  = 1.0 / sqrt((double) head_dim);
    double *      p      = (double *) malloc(sizeof(double) * (size_t) npos);
    for (int64_t h = 0; h < n_head; ++h) {
        const float * qh = q + h * head_dim;
        const int64_t kh = h / group;
        double        mx = -INFINITY;
        for (int64_t j = 0; j < npos; ++j) {
            const float * kj  = kc + j * kv_dim + kh * head_dim;
            double        dot = 0.0;
            for (int64_t d = 0; d < head_dim; ++d) {
                dot += (double) qh[d] * (double) kj[d];
            }
            p[j] = dot * scale;
            mx   = p[j] > mx ? p[j] : mx;
        }
        double sum = 0.0;
        for (int64_t j = 0; j < npos; ++j) {
            p[j] = exp(p[j] - mx);
            sum += p[j];
        }
        for (int64_t d = 0; d < head_dim; ++d) {
            double acc = 0.0;
            for (int64_t j = 0; j < npos; ++j) {
                acc += p[j] * (double) vc[j * kv_dim + kh * head_dim + d];
            }
            out[h * head_dim + d] = (float) (acc / sum);
        }
    }
    free(p);
}

void oracle_decoder_chain(int n_layers, const void * const * weights, const float * norms, int64_t hidden,
                          int64_t n_head, int64_t n_kv, int64_t head_dim, int64_t inter, float eps,
                          const void * table, int64_t table_rows, const int32_t * ids, const float * x_in, int64_t M,
                          float * h_out, int mode, int threads) {
    const int64_t q_dim  = n_head * head_dim;
    const int64_t kv_dim = n_kv * head_dim;
    const int64_t group  = n_head / n_kv;
    const size_t  rb_h   = (size_t) (hidden / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    const size_t  rb_q   = (size_t) (q_dim / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    const size_t  rb_i   = (size_t) (inter / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    float *       h      = h_out;
    float *       tmp    = (float *) malloc(sizeof(float) * (size_t) (M * (hidden > q_dim ? hidden : q_dim)));
    float *       q      = (float *) malloc(sizeof(float) * (size_t) (M * q_dim));
    float *       k      = (float *) malloc(sizeof(float) * (size_t) (M * kv_dim));
    float *       v      = (float *) malloc(sizeof(float) * (size_t) (M * kv_dim));
    float *       a      = (float *) malloc(sizeof(float) * (size_t) (M * q_dim));
    float *       o      = (float *) malloc(sizeof(float) * (size_t) (M * hidden));
    float *       g      = (float *) malloc(sizeof(float) * (size_t) (M * inter));
    float *       u      = (float *) malloc(sizeof(float) * (size_t) (M * inter));
    float *       s      = (float *) malloc(sizeof(float) * (size_t) (M * inter));

    /* h = x_in + get_rows(table, ids) */
    oracle_get_rows_q8_0(table, hidden, table_rows, ids, M, h);
    for (int64_t i = 0; i < M * hidden; ++i) {
        h[i] = x_in[i] + h[i];
    }
    for (int l = 0; l < n_layers; ++l) {
        const void * const * W      = weights + 7 * l;
        const float *        n_in   = norms + (size_t) (2 * l) * hidden;
        const float *        n_post = norms + (size_t) (2 * l + 1) * hidden;
        for (int64_t m = 0; m < M; ++m) {
            rms_norm_mul(h + m * hidden, n_in, tmp + m * hidden, hidden, eps);
        }
        oracle_mul_mat_q8_0_f32(W[0], hidden, q_dim, rb_h, tmp, M, hidden * 4, q, q_dim * 4, mode, NULL, threads);
        oracle_mul_mat_q8_0_f32(W[1], hidden, kv_dim, rb_h, tmp, M, hidden * 4, k, kv_dim * 4, mode, NULL, threads);
        oracle_mul_mat_q8_0_f32(W[2], hidden, kv_dim, rb_h, tmp, M, hidden * 4, v, kv_dim * 4, mode, NULL, threads);
        /* single cached position: softmax over one score is 1, so query head
         * j attends to exactly kv head j / group */
        for (int64_t m = 0; m < M; ++m) {
            for (int64_t j = 0; j < q_dim; ++j) {
                const int64_t head = j / head_dim;
                a[m * q_dim + j]   = v[m * kv_dim + (head / group) * head_dim + j % head_dim];
            }
        }
        oracle_mul_mat_q8_0_f32(W[3], q_dim, hidden, rb_q, a, M, q_dim * 4, o, hidden * 4, mode, NULL, threads);
        for (int64_t i = 0; i < M * hidden; ++i) {
            h[i] = h[i] + o[i];
        }
        for (int64_t m = 0; m < M; ++m) {
            rms_norm_mul(h + m * hidden, n_post, tmp + m * hidden, hidden, eps);
        }
        oracle_mul_mat_q8_0_f32(W[4], hidden, inter, rb_h, tmp, M, hidden * 4, g, inter * 4, mode, NULL, threads);
        oracle_mul_mat_q8_0_f32(W[5], hidden, inter, rb_h, tmp, M, hidden * 4, u, inter * 4, mode, NULL, threads);
        for (int64_t i = 0; i < M * inter; ++i) {
            s[i] = silu_f32(g[i]) * u[i];
        }
        oracle_mul_mat_q8_0_f32(W[6], inter, hidden, rb_i, s, M, inter * 4, o, hidden * 4, mode, NULL, threads);
        for (int64_t i = 0; i < M * hidden; ++i) {
            h[i] = h[i] + o[i];
        }
    }
    free(tmp);
    free(q);
    free(k);
    free(v);
    free(a);
    free(o);
    free(g);
    free(u);
    free(s);
}

/* Final RMS norm of each of `rows` rows (talker.cpp:169, code-predictor.cpp:66:
 * rms_norm(hidden, model.norm.weight)). */
void oracle_rms_norm_rows(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        rms_norm_mul(x + r * n, w, y + r * n, n, eps);
    }
}

/* oracle_decoder_chain with the reference's attention: per layer the q and k
 * heads are RMS-normed (qk_norms: per layer q_norm then k_norm, head_dim
 * floats each) and rotated at pos[m]; k and v go into the caches at pos[m] of
 * slot slots[m] (slots == NULL: slot m; kcache / vcache:
 * [n_layers][n_slots][n_ctx][n_kv * head_dim], updated in place); token m
 * attends over cached positions 0..pos[m] of its slot.  Tokens are processed
 * in order, so tokens of one slot at increasing positions see each other
 * causally, as ggml's masked block does.  table == NULL: h = x_in. */
void oracle_decoder_chain_attn(int n_layers, const void * const * weights, const float * norms,
                               const float * qk_norms, int64_t hidden, int64_t n_head, int64_t n_kv, int64_t head_dim,
                               int64_t inter, float eps, float rope_theta, const void * table, int64_t table_rows,
                               const int32_t * ids, const float * x_in, const int32_t * pos, const int32_t * slots,
                               int64_t M, int64_t n_slots, int64_t n_ctx, float * kcache, float * vcache, float * h_out,
                               int mode, int threads) {
    const int64_t q_dim  = n_head * head_dim;
    const int64_t kv_dim = n_kv * head_dim;
    const size_t  rb_h   = (size_t) (hidden / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    const size_t  rb_q   = (size_t) (q_dim / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    const size_t  rb_i   = (size_t) (inter / ORACLE_QK8_0) * ORACLE_BLOCK_BYTES;
    float *       h      = h_out;
    float *       tmp    = (float *) malloc(sizeof(float) * (size_t) (M * (hidden > q_dim ? hidden : q_dim)));
    float *       q      = (float *) malloc(sizeof(float) * (size_t) (M * q_dim));
    float *       k      = (float *) malloc(sizeof(float) * (size_t) (M * kv_dim));
    float *       v      = (float *) malloc(sizeof(float) * (size_t) (M * kv_dim));
    float *       a      = (float *) malloc(sizeof(float) * (size_t) (M * q_dim));
    float *       o      = (float *) malloc(sizeof(float) * (size_t) (M * hidden));
    float *       g      = (float *) malloc(sizeof(float) * (size_t) (M * inter));
    float *       u      = (float *) malloc(sizeof(float) * (size_t) (M * inter));
    float *       s      = (float *) malloc(sizeof(float) * (size_t) (M * inter));
    if (table != NULL) {
        oracle_get_rows_q8_0(table, hidden, table_rows, ids, M, h);
        for (int64_t i = 0; i < M * hidden; ++i) {
            h[i] = x_in[i] + h[i];
        }
    } else {
        memcpy(h, x_in, sizeof(float) * (size_t) (M * hidden));
    }
    for (int l = 0; l < n_layers; ++l) {
        const void * const * W      = weights + 7 * l;
        const float *        n_in   = norms + (size_t) (2 * l) * hidden;
        const float *        n_post = norms + (size_t) (2 * l + 1) * hidden;
        const float *        qn     = qk_norms + (size_t) (2 * l) * head_dim;
        const float *        kn     = qk_norms + (size_t) (2 * l + 1) * head_dim;
        for (int64_t m = 0; m < M; ++m) {
            rms_norm_mul(h + m * hidden, n_in, tmp + m * hidden, hidden, eps);
        }
        oracle_mul_mat_q8_0_f32(W[0], hidden, q_dim, rb_h, tmp, M, hidden * 4, q, q_dim * 4, mode, NULL, threads);
        oracle_mul_mat_q8_0_f32(W[1], hidden, kv_dim, rb_h, tmp, M, hidden * 4, k, kv_dim * 4, mode, NULL, threads);
        oracle_mul_mat_q8_0_f32(W[2], hidden, kv_dim, rb_h, tmp, M, hidden * 4, v, kv_dim * 4, mode, NULL, threads);
        for (int64_t m = 0; m < M; ++m) {
            oracle_head_norm_rope(q + m * q_dim, n_head, head_dim, qn, eps, pos[m], rope_theta, 1);
            oracle_head_norm_rope(k + m * kv_dim, n_kv, head_dim, kn, eps, pos[m], rope_theta, 1);
            const int64_t slot = slots != NULL ? slots[m] : m;
            float * kc = kcache + (((size_t) l * n_slots + slot) * n_ctx) * kv_dim;
            float * vc = vcache + (((size_t) l * n_slots + slot) * n_ctx) * kv_dim;
            memcpy(kc + (size_t) pos[m] * kv_dim, k + m * kv_dim, sizeof(float) * (size_t) kv_dim);
            memcpy(vc + (size_t) pos[m] * kv_dim, v + m * kv_dim, sizeof(float) * (size_t) kv_dim);
            oracle_attend(q + m * q_dim, kc, vc, (int64_t) pos[m] + 1, n_head, n_kv, head_dim, a + m * q_dim);
        }
        oracle_mul_mat_q8_0_f32(W[3], q_dim, hidden, rb_q, a, M, q_dim * 4, o, hidden * 4, mode, NULL, threads);
        for (int64_t i = 0; i < M * hidden; ++i) {
            h[i] = h[i] + o[i];
        }
        for (int64_t m = 0; m < M; ++m) {
            rms_norm_mul(h + m * hidden, n_post, tmp + m * hidden, hidden, eps);
        }
        oracle_mul_mat_q8_0_f32(W[4], hidden, inter, rb_h, tmp, M, hidden * 4, g, inter * 4, mode, NULL, threads);
        oracle_mul_mat_q8_0_f32(W[5], hidden, inter, rb_h, tmp, M, hidden * 4, u, inter * 4, mode, NULL, threads);
        for (int64_t i = 0; i < M * inter; ++i) {
            s[i] = silu_f32(g[i]) * u[i];
        }
        oracle_mul_mat_q8_0_f32(W[6], inter, hidden, rb_i, s, M, inter * 4, o, hidden * 4, mode, NULL, threads);
        for (int64_t i = 0; i < M * hidden; ++i) {
            h[i] = h[i] + o[i];
        }
    }
    free(tmp);
    free(q);
    free(k);
    free(v);
    free(a);
    free(o);
    free(g);
    free(u);
    free(s);
}
