/*
 * b200q8.h -- C ABI of the B200 (sm_100a) Q8_0 hot path of synthesize.cpp.
 *
 * The reference reaches this arithmetic only through ggml's op set; each entry
 * point below replaces one call that synthesize.cpp makes into ggml (the ggml
 * submodule itself, pinned at 707321c4cf6d21cb4bc831aa8b687dbf01a521ce, is not
 * vendored in the reference tree):
 *
 *   b200q8_mul_mat        ggml_mul_mat(Q8_0 W, F32 x) as executed by a backend:
 *                         src/arch/qwen3-tts/operations.cpp:39-41,90-92,142,
 *                         talker.cpp:45,48,184, code-predictor.cpp:56,79
 *   b200q8_get_rows       ggml_get_rows(Q8_0 table, I32 ids): talker.cpp:44,86,
 *                         code-predictor.cpp:31, model.cpp:1347,1449
 *   b200q8_quantize_rows  quantize_row_q8_0_ref / ggml-cpu from_float for Q8_0
 *   b200q8_quantize_chunk ggml_quantize_chunk(GGML_TYPE_Q8_0, ...):
 *                         tools/synthesize-quantize/quantize.cpp:300-301
 *   b200q8_dequantize_rows  type_traits(Q8_0)->to_float: quantize.cpp:67-83,
 *                         tests/synthesize_quantize_test.cpp:273-276
 *   b200q8_chain_*        the per-frame talker step that builds and computes
 *                         those ops: talker.cpp:135-185 via model.cpp:101-126
 *                         (GraphRun::run), operations.cpp:44-148
 *
 * Conventions (the same as ggml's for these ops):
 *   - Q8_0 data are rows of K/32 blocks, each block an fp16 scale d followed by
 *     32 int8 codes (34 bytes); K % 32 == 0 (quantize.cpp:239-242).
 *   - A MUL_MAT weight W has ne = [K, N]: N rows of K/32 blocks, row n at
 *     w + n*w_row_bytes.  Activations x have ne = [K, M]: token m at
 *     x + m*x_col_stride bytes.  The result y has ne = [N, M].
 *   - Every pointer passed to a compute entry point is a device pointer; work
 *     is enqueued on the caller's CUDA stream and is asynchronous.  No compute
 *     entry point allocates memory; the caller owns every buffer.
 *   - Return values are synth_status_t codes (include/synthesize.h:34-55 in the
 *     reference): B200Q8_OK on success, never an exception or abort across the
 *     ABI.  b200q8_last_error() gives the message of the calling thread's last
 *     failure.  Errors that only a kernel can see (an out-of-range row id, a
 *     wait that ran out) are recorded in a per-device status word that
 *     b200q8_device_status() reads.
 */
#ifndef B200Q8_H
#define B200Q8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t b200q8_status_t;
#define B200Q8_OK                ((b200q8_status_t) 0)  /* SYNTH_OK                    */
#define B200Q8_ERR_INVALID_ARG   ((b200q8_status_t) 1)  /* SYNTH_ERR_INVALID_ARG       */
#define B200Q8_ERR_UNSUPPORTED   ((b200q8_status_t) 8)  /* SYNTH_ERR_UNSUPPORTED_INPUT */
#define B200Q8_ERR_OOM           ((b200q8_status_t) 16) /* SYNTH_ERR_OOM               */
#define B200Q8_ERR_BACKEND       ((b200q8_status_t) 17) /* SYNTH_ERR_BACKEND           */
#define B200Q8_ERR_INTERNAL      ((b200q8_status_t) 20) /* SYNTH_ERR_INTERNAL          */
/* Recorded in the device status word by a kernel whose bounded wait ran out. */
#define B200Q8_ERR_DEVICE_TIMEOUT ((b200q8_status_t) 21)

/* Activation quantizer variants.  REF is quantize_row_q8_0_ref (what the
 * packing tool uses, and ggml-cpu's portable path); CPU_X86 and CPU_ARM are
 * the two SIMD forms of ggml-cpu's quantize_row_q8_0 (id = 127/amax with
 * round-half-even, and id = 1/d with round-half-even). */
#define B200Q8_QUANT_REF     0
#define B200Q8_QUANT_CPU_X86 1
#define B200Q8_QUANT_CPU_ARM 2

#define B200Q8_QK8_0       32
#define B200Q8_BLOCK_BYTES 34

/* cudaStream_t without requiring the CUDA headers. NULL = legacy stream. */
typedef struct CUstream_st * b200q8_stream_t;

/* Library version, major*10000 + minor*100 + patch. */
int32_t b200q8_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to len) and returns its status code. */
b200q8_status_t b200q8_last_error(char * buf, size_t len);

/* Synchronises `device` and returns the status word its kernels recorded
 * (B200Q8_OK if none); clear != 0 resets it.  Replaces ggml's GGML_ASSERT
 * aborts for conditions only the device can check. */
b200q8_status_t b200q8_device_status(int32_t device, int32_t clear);

/* ---- packing and activation quantization (ggml_quantize_chunk,
 *      quantize_row_q8_0_ref, ggml-cpu from_float) ------------------------- */

/* rows x K floats (row r at x + r*x_row_stride bytes) -> rows of K/32 Q8_0
 * blocks (row r at dst + r*dst_row_stride bytes).  mode: B200Q8_QUANT_*.
 * Bit-exact with the reference for every input; for non-finite inputs the
 * codes follow the reference on x86 (a non-finite x*id stores 0) and a NaN
 * scale is stored as 0x7e00. */
b200q8_status_t b200q8_quantize_rows(const float * x, int64_t rows, int64_t K, size_t x_row_stride, void * dst,
                                     size_t dst_row_stride, int32_t mode, b200q8_stream_t stream);

/* ggml_quantize_chunk(GGML_TYPE_Q8_0, src, dst, start, nrows, n_per_row, NULL)
 * on device memory: quantizes nrows rows starting at element `start` (a
 * multiple of n_per_row) of a dense src into the matching rows of a dense
 * dst.  *written receives nrows * n_per_row/32 * 34, the value ggml returns. */
b200q8_status_t b200q8_quantize_chunk(const float * src, void * dst, int64_t start, int64_t nrows,
                                      int64_t n_per_row, size_t * written, b200q8_stream_t stream);

/* ggml_quantize_chunk(GGML_TYPE_Q8_0, src, dst, start, nrows, n_per_row, NULL)
 * on HOST buffers -- the call tools/synthesize-quantize/quantize.cpp:300-301
 * makes, with its arguments' meaning.  Rows stream through `device` in
 * chunks (pinned host staging -> device -> pinned staging, two chunks in
 * flight); bytes identical to quantize_row_q8_0_ref.  Blocking; calls on one
 * device are serialised.  Unlike the compute entry points it allocates: the
 * first call on a device creates about 170 MB of pinned and device staging
 * that later calls reuse, until b200q8_quantize_chunk_host_release().  A tool
 * call, not a hot-path one. */
b200q8_status_t b200q8_quantize_chunk_host(const float * src, void * dst, int64_t start, int64_t nrows,
                                           int64_t n_per_row, size_t * written, int32_t device);

/* Frees the staging b200q8_quantize_chunk_host keeps (every device).  No
 * reference counterpart: ggml_quantize_chunk has no state to release. */
void b200q8_quantize_chunk_host_release(void);

/* Source element types for the typed packing calls (ggml type ids). */
#define B200Q8_SRC_F32  0
#define B200Q8_SRC_F16  1
#define B200Q8_SRC_BF16 30

/* b200q8_quantize_rows for F32, F16 or BF16 source rows.  A 16-bit value is
 * widened to fp32 exactly, as the quantize tool's dequantize_to_f32
 * (tools/synthesize-quantize/quantize.cpp:67-83) does before
 * ggml_quantize_chunk, so the Q8_0 bytes equal those of the F32 path on the
 * widened values.  x_row_stride in bytes (a multiple of the element size). */
b200q8_status_t b200q8_quantize_rows_typed(const void * x, int32_t src_type, int64_t rows, int64_t K,
                                           size_t x_row_stride, void * dst, size_t dst_row_stride, int32_t mode,
                                           b200q8_stream_t stream);

/* b200q8_quantize_chunk_host for an F32, F16 or BF16 host source: replaces
 * the tool's dequantize_to_f32 + ggml_quantize_chunk pair
 * (quantize.cpp:297-301) for Q8_0 targets; start counts elements. */
b200q8_status_t b200q8_quantize_chunk_host_typed(const void * src, int32_t src_type, void * dst, int64_t start,
                                                 int64_t nrows, int64_t n_per_row, size_t * written, int32_t device);

/* Q8_0 rows -> F32 rows: out = q * fp32(d) (exact). */
b200q8_status_t b200q8_dequantize_rows(const void * src, int64_t rows, int64_t K, size_t src_row_stride, float * dst,
                                       size_t dst_row_stride, b200q8_stream_t stream);

/* ---- GET_ROWS ----------------------------------------------------------- */

/* out[i] = dequantize(table row ids[i]) for i < n_ids; K floats per output
 * row at out + i*out_row_stride bytes.  An id outside [0, rows) zero-fills
 * its output row and records B200Q8_ERR_INVALID_ARG in the device status
 * word (ggml-cpu asserts instead). */
b200q8_status_t b200q8_get_rows(const void * table, int64_t K, int64_t rows, size_t table_row_stride,
                                const int32_t * ids, int64_t n_ids, float * out, size_t out_row_stride,
                                b200q8_stream_t stream);

/* ---- MUL_MAT ------------------------------------------------------------ */

/* Bytes of caller-provided scratch b200q8_mul_mat needs for these sizes
 * (0 when the fused decode path needs none).  With B200Q8_TC_MIN_M=<M> set in
 * the environment (read once), M >= that many tokens also count the tcgen05
 * GEMM's planes; b200q8_mul_mat uses that GEMM only when the workspace holds
 * them, and otherwise needs only the smaller size. */
size_t b200q8_mul_mat_workspace_size(int64_t K, int64_t N, int64_t M);

/* y = W * quantize(x): y[m][n] = sum_b fp32(dw[n,b]) * fp32(dx[m,b]) * sum_i qw*qx,
 * the arithmetic of ggml-cpu's vec_dot_q8_0_q8_0 after from_float.  Codes and
 * scales of x are bit-exact with the reference quantizer `mode`; y agrees
 * with the reference within 1e-5 * sum_b |dw*dx*isum_b| per element (only
 * the fp32 summation order differs).  workspace may be NULL when
 * b200q8_mul_mat_workspace_size() returns 0. */
b200q8_status_t b200q8_mul_mat(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const float * x, int64_t M,
                               size_t x_col_stride, float * y, size_t y_col_stride, int32_t mode, void * workspace,
                               size_t workspace_bytes, b200q8_stream_t stream);

/* The same MUL_MAT for callers that cannot allocate device memory at the
 * point of the call -- a ggml backend computing a graph whose buffers were all
 * placed before the graph ran, a real-time streaming callback that must not
 * block on cudaMalloc's device-wide synchronisation.  No counterpart in the reference (its CPU path allocates nothing
 * on the device).  It allocates nothing: its scratch (quantized or staged
 * activations) is a fixed 1 MiB array in the library's own device memory,
 * held by every GPU that loads the library until the process exits.  Requires
 * M * (K/32) * 34 <= 1048576 bytes (else B200Q8_ERR_INVALID_ARG).  It runs the
 * path b200q8_mul_mat runs with a workspace of the array's size (the
 * tensor-core GEMM when its records fit, else the streaming GEMV, which needs
 * no scratch, else the general kernel).  Every call on a device shares that
 * array, so calls whose kernels overlap on the GPU race; order them on one
 * stream.  The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  Calls on a stream that is not capturing look it
 * up again, so a device reset is picked up by the next such call.  Results as
 * b200q8_mul_mat. */
b200q8_status_t b200q8_mul_mat_noalloc(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const float * x,
                                       int64_t M, size_t x_col_stride, float * y, size_t y_col_stride, int32_t mode,
                                       b200q8_stream_t stream);

/* ---- the talker-shaped decode step -------------------------------------- */

/* One decoder layer of the Qwen3 talker as the step chain sees it (ggml
 * layouts, device pointers).  wq..wd are Q8_0 matrices with ne = [in, out];
 * norm_in / norm_post are F32 [hidden] (input_layernorm, post_attn_norm). */
typedef struct b200q8_layer {
    const void *  wq;
    const void *  wk;
    const void *  wv;
    const void *  wo;
    const void *  wgate;
    const void *  wup;
    const void *  wdown;
    const float * norm_in;
    const float * norm_post;
} b200q8_layer;

/* The reference's attention in the step (src/arch/qwen3-tts/operations.cpp:
 * 86-135): per-head RMS norms of q and k (q_norm / k_norm weights), NEOX RoPE
 * at each token's position (ggml_rope_ext, freq_base = rope_theta), an F32
 * KV cache per stream slot, softmax(q K^T / sqrt(head_dim)) V over the
 * cached prefix.  Chains built with it run through b200q8_chain_run_at. */
typedef struct b200q8_attention_desc {
    float                 rope_theta; /* synthesize.qwen3-tts.talker.rope_theta           */
    int64_t               n_ctx;      /* cache capacity in positions, per slot            */
    int64_t               n_slots;    /* independent streams with a cache                 */
    const float * const * q_norm;     /* n_layers device pointers, F32 [head_dim]         */
    const float * const * k_norm;     /* n_layers device pointers, F32 [head_dim]         */
} b200q8_attention_desc;

/* The output side of a step (src/arch/qwen3-tts/talker.cpp:169-185,
 * code-predictor.cpp:66-80): the final RMS norm of the residual stream and
 * one or more Q8_0 heads applied to it.  The talker has one head
 * (codec_head), the code predictor one per acoustic group (lm_head.{g}). */
typedef struct b200q8_output_desc {
    const float *        norm;    /* F32 [hidden] (model.norm.weight)                      */
    const void * const * heads;   /* n_heads device pointers, Q8_0 with ne = [hidden, vocab] */
    int32_t              n_heads;
    int64_t              vocab;
} b200q8_output_desc;

typedef struct b200q8_chain_desc {
    int32_t              n_layers;
    int64_t              hidden;   /* 1024 for the 0.6B talker          */
    int64_t              n_head;   /* 16                                */
    int64_t              n_kv;     /* 8                                 */
    int64_t              head_dim; /* 128                               */
    int64_t              inter;    /* 3072                              */
    float                eps;      /* rms_norm_eps                      */
    int64_t              max_m;    /* largest token batch run() accepts */
    int32_t              mode;     /* B200Q8_QUANT_*                    */
    const b200q8_layer * layers;   /* n_layers entries, copied          */
    const void *         table;    /* Q8_0 embedding [hidden, table_rows] */
    int64_t              table_rows;
    /* NULL: attention over a single cached position (query head h returns v
     * of kv head h / (n_head / n_kv)), the talker-shaped benchmark step. */
    const b200q8_attention_desc * attention;
    /* NULL: the step ends at the residual stream (h_out). */
    const b200q8_output_desc *    output;
} b200q8_chain_desc;

typedef struct b200q8_chain b200q8_chain;

/* Builds a step plan: packs each layer's q|k|v and gate|up weights into
 * contiguous device copies (one allocation, at plan time), allocates the
 * per-layer activation buffers, and prepares the launch sequence.  The only
 * entry points that allocate are b200q8_chain_create and nothing else. */
b200q8_status_t b200q8_chain_create(const b200q8_chain_desc * desc, int32_t device, b200q8_chain ** out);

/* One decode step for M tokens (M <= max_m):
 *   h = x_in + get_rows(table, ids); then per layer
 *   h1 = h + Wo*Q(attend(Wq,Wk,Wv * Q(rms_norm(h)*norm_in)))
 *   h  = h1 + Wd*Q(silu(Wg*Q(n)) * (Wu*Q(n))),  n = rms_norm(h1)*norm_post
 * where attend is attention over a single cached position (query head j
 * reads kv head j/(n_head/n_kv)).  ids [M] I32, x_in and h_out [M][hidden]
 * F32, all device pointers. */
b200q8_status_t b200q8_chain_run(b200q8_chain * chain, const int32_t * ids, const float * x_in, float * h_out,
                                 int64_t M, b200q8_stream_t stream);

/* Device pointer to one of layer l's activation buffers of the last run
 * (which: 0 = normalised input, 1 = q|k|v, 2 = attention output, 3 = o,
 * 4 = h1, 5 = normalised h1, 6 = gate|up, 7 = silu(gate)*up, 8 = down,
 * 9 = h after the layer); row stride in floats via *stride. */
b200q8_status_t b200q8_chain_buffer(b200q8_chain * chain, int32_t layer, int32_t which, float ** ptr,
                                    int64_t * stride);

void b200q8_chain_destroy(b200q8_chain * chain);

/* One step of a chain built with an attention desc: token m belongs to
 * stream slot slots[m] (slots == NULL: slot m) and sits at position pos[m]
 * (device int32 arrays of M entries).  Its k and v are written to that
 * slot's cache at pos[m] and it attends over positions 0..pos[m], so a stream
 * decodes with pos = 0, 1, 2, ...  A position outside [0, n_ctx) or a slot
 * outside [0, n_slots) records B200Q8_ERR_INVALID_ARG in the device status
 * and zeroes that token's attention. */
b200q8_status_t b200q8_chain_run_at(b200q8_chain * chain, const int32_t * ids, const float * x_in,
                                    const int32_t * pos, const int32_t * slots, float * h_out, int64_t M,
                                    b200q8_stream_t stream);

/* One step with every input and output the reference's graphs vary
 * (talker.cpp:135-185 for the talker, code-predictor.cpp:34-80 for the code
 * predictor, whose calls differ in input table, head and input rows):
 *   h0     = x_in + get_rows(table, ids)    (either term may be absent)
 *   h      = the layers of b200q8_chain_run / _run_at applied to h0
 *   hidden = rms_norm(h) * output.norm
 *   logits = heads[head] * Q(hidden)
 * All pointers are device pointers; the buffers must not overlap. */
typedef struct b200q8_step_args {
    int64_t         M;          /* tokens, 1..max_m                                         */
    const int32_t * ids;        /* [M] rows of `table`, or NULL: no lookup                  */
    const void *    table;      /* Q8_0 [hidden, table_rows]; NULL: the desc's table        */
    int64_t         table_rows;
    const float *   x_in;       /* [M][hidden], or NULL: zeros (ids then required)          */
    const int32_t * pos;        /* [M] positions (attention chains only, else NULL)         */
    const int32_t * slots;      /* [M] stream slots, or NULL: slot m                        */
    float *         h_out;      /* [M][hidden] residual stream after the last layer, or NULL */
    float *         hidden_out; /* [M][hidden], or NULL (chains with an output desc)        */
    float *         logits;     /* [M][vocab], or NULL (chains with an output desc)         */
    int32_t         head;       /* which head computes logits                               */
} b200q8_step_args;

/* Runs one step as a CUDA graph captured once per distinct argument set
 * (pointers, M, head).  With hidden_out and logits both NULL the output stage
 * is skipped.  Errors: B200Q8_ERR_INVALID_ARG for a missing required pointer,
 * M outside [1, max_m], pos on a chain without attention (or none on one
 * with), an output on a chain without an output desc, head outside
 * [0, n_heads). */
b200q8_status_t b200q8_chain_step(b200q8_chain * chain, const b200q8_step_args * args, b200q8_stream_t stream);

/* ---- one frame of Qwen3-TTS decoding: talker + code predictor ----------- */

/* A frame as src/arch/qwen3-tts/model.cpp:1310-1489 computes it, for M
 * independent streams in one CUDA graph, with G = groups codes per frame:
 *
 *   x      = sum_{g=1..G-1} ptable[g-1][prev[g]]  + ttable[prev[0]] + text
 *            (sum_code_embeddings, code-predictor.cpp:84-109, in group order;
 *            then build_talker_step_input, talker.cpp:120-133)
 *   talker step at pos -> hidden, logits        -> codes[0]
 *   predictor at positions 0, 1 over [hidden, ttable[codes[0]]], head 0
 *                                               -> codes[1]
 *   for g = 1..G-2: predictor at position g+1 over ptable[g-1][codes[g]],
 *                   head g                      -> codes[g+1]
 *
 * (the schedule of code-predictor-host.cpp:15-41).  A code is either the
 * replayed one (request.replay_codes) or the reference's greedy choice
 * (request.sample == false): the first index of the largest logit
 * (std::max_element, code-predictor-host.cpp:45-49,71-80), after the
 * talker's repetition penalty over the stream's previously chosen semantic
 * codes (apply_repetition_penalty, code-predictor-host.cpp:51-69).  Sampling
 * with a temperature is not done on the device. */
typedef struct b200q8_frame_desc {
    b200q8_chain *       talker;     /* attention + output desc with >= 1 head; its table = ttable  */
    b200q8_chain *       predictor;  /* attention + output desc with >= G-1 heads, n_ctx >= G,
                                        max_m >= 2 * the frame's M, same device; same hidden width
                                        unless an input projection is given                        */
    int32_t              groups;     /* code_group_count (16)                                       */
    const void * const * tables;     /* G-1 device pointers: predictor codec_embedding.{g}, Q8_0
                                        [talker hidden, table_rows]                                 */
    int64_t              table_rows;
    float                repetition_penalty;  /* the talker's; values <= 1 apply none             */
    /* A predictor narrower than the talker (the 1.7B packages): every
     * predictor input row (talker width) is first projected,
     * x = W * Q(x) + b (small_to_mtp_projection, code-predictor.cpp:49-58).
     * NULL / NULL when the widths agree. */
    const void *         input_projection;       /* Q8_0 with ne = [talker hidden, predictor hidden] */
    const float *        input_projection_bias;  /* F32 [predictor hidden]                          */
    /* The talker's text side, for frames run from text token ids
     * (build_text_projection, src/arch/qwen3-tts/talker.cpp:37-50):
     *   text = W2 * Q(silu(W1 * Q(text_embedding[id]) + b1)) + b2
     * (a Q8_0 GET_ROWS, then two Q8_0 MUL_MATs with F32 biases).  All NULL:
     * frames take precomputed text rows only. */
    const void *         text_embedding;         /* Q8_0 with ne = [text hidden, text_rows]             */
    int64_t              text_rows;              /* the text vocabulary                                 */
    int64_t              text_hidden;
    const void *         text_fc1;               /* Q8_0 ne = [text hidden, text hidden] (linear_fc1)   */
    const float *        text_fc1_bias;          /* F32 [text hidden]                                   */
    const void *         text_fc2;               /* Q8_0 ne = [text hidden, talker hidden] (linear_fc2) */
    const float *        text_fc2_bias;          /* F32 [talker hidden]                                 */
} b200q8_frame_desc;

typedef struct b200q8_frame b200q8_frame;

/* Builds the frame plan: device copies of the table list, the predictor's
 * position arrays and a per-slot history of chosen semantic codes (cleared;
 * one per talker slot).  The chains stay owned by the caller and must
 * outlive the frame. */
b200q8_status_t b200q8_frame_create(const b200q8_frame_desc * desc, b200q8_frame ** out);

typedef struct b200q8_frame_args {
    int64_t         M;
    /* 1: the talker already ran (the prompt pass, through b200q8_chain_step);
     * hidden and talker_logits then hold its outputs and are read, text /
     * prev / pos are ignored, and the frame starts at selecting codes[0]. */
    int32_t         skip_talker;
    const float *   text;           /* [M][hidden] the frame's text-side input row             */
    const int32_t * prev;           /* [M][G] the previous frame's codes                        */
    const int32_t * pos;            /* [M] the talker position of this frame's token            */
    const int32_t * slots;          /* [M] stream slots (both caches and the history); NULL: m  */
    const int32_t * replay;         /* [M][G] codes to take instead of choosing; NULL: greedy   */
    int32_t *       codes;          /* [M][G] out                                               */
    float *         hidden;         /* [M][hidden] talker hidden: out (in when skip_talker); may be NULL unless skip_talker */
    float *         talker_logits;  /* [M][talker vocab]: same                                  */
    /* [M] text token ids (device): the frame computes its text rows through
     * the desc's text projection, and `text` is ignored.  NULL: `text`
     * holds the rows.  An id outside [0, text_rows) gives a zero embedding
     * row and records B200Q8_ERR_INVALID_ARG in b200q8_device_status. */
    const int32_t * text_ids;
} b200q8_frame_args;

b200q8_status_t b200q8_frame_run(b200q8_frame * frame, const b200q8_frame_args * args, b200q8_stream_t stream);

/* The talker's text rows for M text token ids through the frame's text
 * projection (build_text_projection, src/arch/qwen3-tts/talker.cpp:37-50):
 * out [M][talker hidden] = W2 * Q(silu(W1 * Q(text_embedding[id]) + b1)) + b2,
 * the rows a frame run with text_ids adds to its input.  h1 (may be NULL)
 * receives silu(W1 * Q(text_embedding[id]) + b1), [M][text hidden].  Device
 * pointers, enqueued on `stream`; M <= the frame's max M.  The frame must have
 * been built with a text projection. */
b200q8_status_t b200q8_frame_text_rows(b200q8_frame * frame, const int32_t * text_ids, int64_t M, float * h1,
                                       float * out, b200q8_stream_t stream);

/* Forgets the chosen-code history of one slot (slot < 0: every slot), as a
 * new utterance starts with an empty history.  Enqueued on `stream`. */
b200q8_status_t b200q8_frame_reset_history(b200q8_frame * frame, int32_t slot, b200q8_stream_t stream);

void b200q8_frame_destroy(b200q8_frame * frame);

/* Fault injection for tests (host side; no GPU fault): skew != 0 shifts the
 * persistent step's launch counter by `skew`, so that (unless skew is a
 * multiple of the step's CTA count) the CTAs of the next persistent runs
 * disagree on the step's epoch and the hand-off waits run out (about a
 * second); such a run must end with B200Q8_ERR_DEVICE_TIMEOUT in
 * b200q8_device_status and leave the context usable.  skew == 0 restores the
 * chain: the counter is realigned and one epoch skipped, so no hand-off word
 * written by a skewed run is taken as current later.  Synchronizes the device.
 * No reference counterpart. */
b200q8_status_t b200q8_chain_inject_epoch_skew(b200q8_chain * chain, int32_t skew);

#ifdef __cplusplus
}
#endif

#endif /* B200Q8_H */
