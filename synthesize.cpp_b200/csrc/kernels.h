// kernels.h -- host-side launchers of the sm_100a kernels (internal).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200q8 {

cudaError_t launch_quantize(const float * x, int64_t rows, int64_t K, size_t x_stride, void * dst, size_t dst_stride,
                            int mode, cudaStream_t stream, int sm_count);

// Source element types of the packing kernels (ggml type ids).
enum SrcType : int { kSrcF32 = 0, kSrcF16 = 1, kSrcBF16 = 30 };

// F32 / F16 / BF16 rows -> Q8_0 rows (16-bit sources widened exactly first).
cudaError_t launch_quantize_typed(const void * x, int src_type, int64_t rows, int64_t K, size_t x_stride, void * dst,
                                  size_t dst_stride, int mode, cudaStream_t stream, int sm_count);

cudaError_t launch_dequant_rows(const void * src, size_t src_stride, int64_t src_rows, const int32_t * ids,
                                int64_t n_out, int64_t K, float * out, size_t out_stride, cudaStream_t stream,
                                int sm_count);

// How the GEMV derives its fp32 input from the buffers it is given.
enum Prologue : int {
    kProPlain   = 0,  // x_eff = x
    kProRmsNorm = 1,  // x_eff = (x * 1/sqrtf(mean(x^2)+eps)) * norm_w
    kProGqa     = 2,  // x_eff[j] = x[(j/head_dim/group)*head_dim + j%head_dim]
    kProSwiGlu  = 3,  // x_eff[i] = silu(x[i]) * x2[i]
};

struct GemvParams {
    // weights: N rows of K/32 Q8_0 blocks, row n at w + n*row_bytes
    const uint8_t * w;
    size_t          row_bytes;
    int             K;
    int             N;
    int             M;  // tokens
    // input
    int             pro;
    const float *   x;
    const float *   x2;
    size_t          x_stride;  // floats between tokens
    const float *   norm_w;
    float           eps;
    int             head_dim;
    int             group;
    float *         pro_out;  // optional: x_eff written by CTA 0
    size_t          pro_out_stride;
    // output
    float *         y;
    size_t          y_stride;  // floats between tokens
    const float *   res;       // optional residual: y_res = res + y
    float *         y_res;
    size_t          res_stride;
    int             mode;
};

// True when the streaming GEMV supports this shape (K % 256 == 0, 16-byte
// aligned weight rows, M <= 8, activation tile fits in shared memory).
bool gemv_supported(const GemvParams & p);

// pdl: launch with programmatic stream serialization (weights are prefetched
// before the wait on the previous kernel; only for chains whose weights no
// kernel in the stream writes).
cudaError_t launch_gemv(const GemvParams & p, cudaStream_t stream, int sm_count, bool pdl);

// Fallback for any K % 32 == 0 / alignment: x already quantized into xq
// (M rows of K/32 standard blocks).
cudaError_t launch_gemv_generic(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const uint8_t * xq,
                                int64_t M, float * y, size_t y_stride_bytes, cudaStream_t stream);

// ---- int8 tensor-core GEMM for M > 8 (gemm.cu)

// Token chunking shared by the stage kernels and the GEMM: n_tc chunks of tm
// tokens (tm a multiple of 8, at most 64; the last chunk may be partial).
struct GemmChunking {
    int tm;
    int n_tc;
};
GemmChunking gemm_chunking(int64_t M);
// Bytes of the staged activations of M tokens of K values (K % 256 == 0).
size_t       gemm_workspace_bytes(int64_t K, int64_t M);
bool         gemm_supported(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, int64_t M);
// Stage (quantize) x into the workspace, then the GEMM.
cudaError_t  launch_gemm(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const float * x, size_t x_stride,
                         int64_t M, float * y, size_t y_stride, int mode, void * workspace, cudaStream_t stream,
                         int sm_count);
// The GEMM on activations already staged by launch_stage_rows.
// Room for split-K partial sums (part, part_floats floats) and per-block
// arrival counters (cnt, n_cnt words, zero when no launch is running; each
// launch leaves them zero).  Launches on one split area must be ordered.
struct GemmSplit {
    float *    part;
    size_t     part_floats;
    unsigned * cnt;
    size_t     n_cnt;
};
cudaError_t  launch_gemm_staged(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const uint8_t * xrec,
                                int64_t M, float * y, size_t y_stride, cudaStream_t stream, int sm_count, bool pdl,
                                const GemmSplit * split = nullptr);
// Large-M MUL_MAT on the tcgen05 tensor cores (gemm_tc.cu): the weights and
// the quantized activations as code / scale planes in the workspace, then one
// persistent kernel over 128-row x 128-token tiles.  gemm_tc_min_m() is 0
// (off) unless B200Q8_TC_MIN_M sets it.
int64_t      gemm_tc_min_m();
bool         gemm_tc_supported(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, int64_t M, const float * x,
                               size_t x_stride);
size_t       gemm_tc_workspace_bytes(int64_t K, int64_t N, int64_t M);
cudaError_t  launch_gemm_tc(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const float * x,
                            size_t x_stride, int64_t M, float * y, size_t y_stride, int mode, void * workspace,
                            cudaStream_t stream, int sm_count);
// Per-token prologue (one CTA per token): kind 0 = rms_norm(a [+ b]) * norm
// (a + b also written to sum_out), 1 = GQA expansion of a, 2 = silu(a) * b,
// 3 = a; the result is quantized into the staged records xrec.
cudaError_t  launch_stage_rows(int kind, const float * a, const float * b, size_t ab_stride, float * sum_out,
                               size_t sum_stride, const float * norm, float eps, int K, int head_dim, int group,
                               float * trace, size_t trace_stride, int64_t M, int mode, uint8_t * xrec,
                               cudaStream_t stream, bool pdl);
cudaError_t launch_residual_rows(const float * a, const float * b, size_t ab_stride, float * out, size_t out_stride,
                                 int K, int64_t M, cudaStream_t stream, bool pdl);

// ---- attention with a KV cache (attention.cu)

constexpr int kAttnMaxSplits = 32;

struct AttnArgs {
    const float *   qkv;         // [M][qkv_stride]: q heads, then k heads, then v heads
    size_t          qkv_stride;  // floats
    int             n_head, n_kv, head_dim;
    float           eps, rope_theta;
    const float *   q_norm;      // [head_dim] of this layer
    const float *   k_norm;
    const int32_t * pos;         // [M] positions
    const int32_t * slots;       // [M] cache slots, or null: slot = slot_base + token index
    int             slot_base;
    int             n_ctx, n_slots;
    float *         q_rot;       // [M][n_head*head_dim] normed, rotated q
    float *         k_cache;     // this layer: [n_slots][n_ctx][n_kv][head_dim]
    float *         v_cache;
    float *         partial;     // [M][n_head][splits][head_dim + 2]
    unsigned *      counters;    // [M][n_head], zero between launches
    float *         out;         // [M][out_stride]: attention output, head-major
    size_t          out_stride;
};

bool        attention_supported(int head_dim, int n_head, int n_kv);
int         attention_splits(int64_t M, int n_head, int sm_count);
cudaError_t launch_attention(const AttnArgs & a, int64_t M, int splits, cudaStream_t stream, bool pdl);

// ---- the persistent decode step (decode_step.cu)

struct StepLayerDev {
    const uint8_t * w_qkv;   // [Q + 2*KV rows] of K = H
    const uint8_t * w_o;     // [H rows] of K = Q
    const uint8_t * w_gate;  // [I rows] of K = H
    const uint8_t * w_up;    // [I rows] of K = H
    const uint8_t * w_down;  // [H rows] of K = I
    const float *   norm_in;
    const float *   norm_post;
    const float *   q_norm;  // [head_dim] (attention steps only)
    const float *   k_norm;
};

struct StepArgs {
    const StepLayerDev * layers;  // device array [n_layers]
    int                  n_layers;
    int                  H, Q, KV, I, head_dim, group;
    int                  lg_head_dim, lg_group;  // log2 of head_dim and group (both powers of two)
    float                eps;
    size_t               rb_h, rb_q, rb_i;
    const uint8_t *      table;
    int64_t              table_rows;
    const int32_t *      ids;
    const float *        x_in;
    float *              h_out;
    int                  M;
    int                  mode;
    // LL words, per layer [qkv | att | o | s | d], each [ll_m][width]
    // (width Q + 2 KV, Q, H, I, H)
    unsigned long long * ll;
    size_t               ll_layer;  // words per layer
    int                  ll_m;      // token stride of the LL buffers
    // attention over the KV cache (attn != 0; else the single cached position)
    int                  attn;
    float                rope_theta;
    const int32_t *      pos;       // [M]
    const int32_t *      slots;     // [M] or nullptr: slot m
    int                  n_ctx, n_cache_slots;
    float *              k_cache;   // [n_layers][n_cache_slots][n_ctx][KV]
    float *              v_cache;
    // output stage (head != nullptr): hidden_out = rms_norm(h) * out_norm,
    // logits = head * Q(hidden_out); h_out is written in full either way
    const float *        out_norm;
    const uint8_t *      head;      // [vocab rows] of K = H
    int                  vocab;
    float *              hidden_out;
    float *              logits;
    float *              trace;     // optional per-layer activation copies (chain buffer layout)
    size_t               trace_layer;
    size_t               trace_off[10];
    unsigned *           sync;      // [0] launch counter, [1] abort word
    int                  n_slots;   // set by the launcher
    unsigned long long * timeline;  // analysis builds (B200Q8_TIMELINE) only: stamps, else unused
};

bool        decode_step_supported(const StepArgs & a, int grid);
int         decode_step_max_m(const StepArgs & a);
size_t      decode_step_smem_bytes(const StepArgs & a, int mt, int & n_slots);
cudaError_t launch_decode_step(StepArgs a, int grid, cudaStream_t stream);

}  // namespace b200q8
