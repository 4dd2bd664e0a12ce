/*
 * q8_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the CPU arithmetic that synthesize.cpp runs on its
 * Q8_0 hot path.  The arithmetic itself lives in ggml (an un-vendored git
 * submodule of the reference, pinned at ggml 707321c4cf6d21cb4bc831aa8b687dbf01a521ce
 * per docs/porting/families/vits.md:244), so every function below restates the
 * published algorithm and cites the reference call site that reaches it.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * call into this library.  The product path (libb200q8.so) never links it.
 *
 * Pinning: the packing routine is checked byte-for-byte against gguf-py 0.19.0
 * (gguf/quants.py:378-394, the version the reference pins in
 * scripts/envs/qwen3-tts/uv.lock:291-293), whose Q8_0 quantizer states that it
 * is bit-exact with ggml-quants.c.  The fixtures generated from it live in
 * tests/golden/ together with the script that made them.
 */
#ifndef Q8_ORACLE_H
#define Q8_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_QK8_0 32
#define ORACLE_BLOCK_BYTES 34

/* Activation-quantizer variants (see oracle_quantize_row_q8_0). */
#define ORACLE_QUANT_REF 0     /* quantize_row_q8_0_ref: id = 1/d, round half away from zero */
#define ORACLE_QUANT_CPU_X86 1 /* ggml-cpu AVX path: id = 127/amax, round half to even       */
#define ORACLE_QUANT_CPU_ARM 2 /* ggml-cpu NEON path: id = 1/d, round half to even           */

uint16_t oracle_fp32_to_fp16(float f);
float    oracle_fp16_to_fp32(uint16_t h);

/* One row of k floats (k % 32 == 0) -> k/32 blocks of 34 bytes. */
void oracle_quantize_row_q8_0(const float * x, void * y, int64_t k, int mode);

/* ggml_quantize_chunk(GGML_TYPE_Q8_0, src, dst, start, nrows, n_per_row, NULL):
 * start is an element offset that must be a multiple of n_per_row.  Returns
 * the bytes written (nrows * n_per_row/32 * 34). */
size_t oracle_quantize_chunk_q8_0(const float * src, void * dst, int64_t start, int64_t nrows, int64_t n_per_row);

void oracle_dequantize_row_q8_0(const void * x, float * y, int64_t k);

/* vec_dot_q8_0_q8_0 over n elements: per block an exact int32 sum of code
 * products, scaled by fp32(dx)*fp32(dy), accumulated in fp32 in block order.
 * If abs_bound is non-NULL it receives sum_b |fp32(dx)*fp32(dy)*isum_b| in
 * double, the quantity the parity tolerance is relative to. */
float oracle_vec_dot_q8_0_q8_0(int64_t n, const void * vx, const void * vy, double * abs_bound);

/* ggml_mul_mat(W[K,N] Q8_0, x[K,M] F32) -> y[N,M] F32 in ggml layout:
 * W row n starts at w + n*w_row_bytes, token m of x at x + m*x_col_stride
 * bytes, output token m at y + m*y_col_stride bytes.  x is first quantized
 * with the given activation mode (the from_float step ggml-cpu performs).
 * bound (nullable) receives N*M abs bounds laid out like y with a dense
 * stride of N.  threads <= 0 uses every OpenMP thread. */
void oracle_mul_mat_q8_0_f32(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const float * x, int64_t M,
                             size_t x_col_stride, float * y, size_t y_col_stride, int mode, double * bound,
                             int threads);

/* Same, with x already quantized: xq holds M rows of K/32 blocks. */
void oracle_mul_mat_q8_0_q8_0(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const void * xq, int64_t M,
                              float * y, size_t y_col_stride, double * bound, int threads);

/* ggml_get_rows(table[K,rows] Q8_0, ids[n_ids] I32) -> out[K,n_ids] F32.
 * Returns 0, or -1 (with the offending row zero-filled) for an id outside
 * [0, rows). */
int oracle_get_rows_q8_0(const void * table, int64_t K, int64_t rows, const int32_t * ids, int64_t n_ids, float * out);

/* synth::NormalRandomStream(seed).fill(out, count): splitmix64 + Marsaglia
 * polar method in double, spare value reused. */
void oracle_normal_fill(uint64_t seed, float * out, size_t count);
/* The same stream drawn as uniforms on [0,1) (next_uniform). */
void oracle_uniform_fill(uint64_t seed, float * out, size_t count);
/* out[i] = scale * normal_i: the synthetic weight generator. */
void oracle_normal_fill_scaled(uint64_t seed, float scale, float * out, size_t count);

/* Test-fixture helpers: many seeded tensors, and many packed rows, on OpenMP
 * threads; the values are those of the single-threaded routines above. */
void oracle_normal_fill_scaled_many(int n, const uint64_t * seeds, const float * scales, float * const * outs,
                                    const size_t * counts, int threads);
void oracle_quantize_rows_mt(const float * x, void * dst, int64_t rows, int64_t k, int mode, int threads);

/* min(n/2, n-1) threads for n available (1 when n <= 2):
 * src/cpu-parallelism.cpp:93-99. */
int oracle_default_synthesis_threads(int available);

/* The talker-shaped decode step: the dataflow of decoder_layer
 * (src/arch/qwen3-tts/operations.cpp:44-148) over n_layers layers with the
 * attention reduced to a single cached position (softmax of one score is 1,
 * so query head j reads kv head j/(n_head/n_kv)), and the step input
 * h = x_in + get_rows(table, ids) (talker.cpp:86, model.cpp:1347).
 * weights: n_layers*7 pointers in the order q,k,v,o,gate,up,down (ggml
 * layout ne=[in,out]); norms: n_layers*2*hidden floats (input_layernorm,
 * post_attention_layernorm per layer).  h_out: [M][hidden]. */
void oracle_decoder_chain(int n_layers, const void * const * weights, const float * norms, int64_t hidden,
                          int64_t n_head, int64_t n_kv, int64_t head_dim, int64_t inter, float eps,
                          const void * table, int64_t table_rows, const int32_t * ids, const float * x_in, int64_t M,
                          float * h_out, int mode, int threads);

void oracle_head_norm_rope(float * x, int64_t n_heads, int64_t head_dim, const float * w, float eps, int32_t pos,
                           float theta_base, int rope);
void oracle_attend(const float * q, const float * kc, const float * vc, int64_t npos, int64_t n_head, int64_t n_kv,
                   int64_t head_dim, float * out);
void oracle_decoder_chain_attn(int n_layers, const void * const * weights, const float * norms,
                               const float * qk_norms, int64_t hidden, int64_t n_head, int64_t n_kv, int64_t head_dim,
                               int64_t inter, float eps, float rope_theta, const void * table, int64_t table_rows,
                               const int32_t * ids, const float * x_in, const int32_t * pos, const int32_t * slots,
                               int64_t M, int64_t n_slots, int64_t n_ctx, float * kcache, float * vcache, float * h_out,
                               int mode, int threads);
void oracle_bias_silu_rows(float * x, const float * b, int64_t rows, int64_t n);
void oracle_rms_norm_rows(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps);
int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif

#endif
