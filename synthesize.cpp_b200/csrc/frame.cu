// frame.cu -- one frame of Qwen3-TTS decoding (talker + code predictor) as one
// CUDA graph.
//
// The reference's frame loop (src/arch/qwen3-tts/model.cpp:1310-1489) builds
// and computes one talker graph and then code_group_count - 1 predictor graphs
// per frame on the CPU, reading the logits back after each to choose the next
// code on the host.  Here every part of a frame stays on the device:
//
//   frame_embed_kernel    talker input = sum of the previous frame's code
//                         embeddings (predictor tables for groups 1..G-1 in
//                         group order, then the talker's table for group 0)
//                         + the text row
//   talker step           chain_enqueue (attention, final norm, codec_head)
//   frame_select_kernel   codes[0] (greedy after the repetition penalty, or
//                         replayed)
//   frame_prefill_kernel  the predictor's two-position input [hidden,
//                         ttable[codes[0]]]
//   predictor prefill     chain_enqueue (positions 0, 1; head 0) -> codes[1]
//   G - 2 predictor steps chain_enqueue (position g+1; table g-1; head g)
//                         -> codes[g+1]
//
// The whole sequence is captured once per argument set and replayed with one
// graph launch, so a frame costs no host round trip at all; the caller reads
// the codes back once per frame (or not at all).
#include "chain.h"
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <new>
#include <vector>

namespace b200q8 {
b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...);
b200q8_status_t cuda_error(cudaError_t e, const char * what);

namespace {

constexpr int kSelectThreads = 256;
constexpr int kMaxFrameGraphs = 16;

// The dequantized value of element k of row r of a Q8_0 table: q * fp32(d)
// (ggml_get_rows through Q8_0 to_float).  An out-of-range row records
// INVALID_ARG and reads as 0.
__device__ __forceinline__ float table_value(const uint8_t * table, size_t row_bytes, int64_t rows, int64_t r,
                                             int64_t k) {
    if (r < 0 || r >= rows) {
        record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
        return 0.0f;
    }
    const uint8_t * blk = table + r * row_bytes + (k / kQK) * kBlockBytes;
    const float     d   = __half2float(__ushort_as_half((unsigned short) (blk[0] | (blk[1] << 8))));
    return __fmul_rn((float) (int8_t) blk[2 + k % kQK], d);
}

// slots1[m] = slots ? slots[m] : m; pslots[2m] = pslots[2m+1] = slots1[m].
__global__ void frame_setup_kernel(const int32_t * __restrict__ slots, int32_t * __restrict__ slots1,
                                   int32_t * __restrict__ pslots, int64_t M) {
    for (int64_t m = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; m < M; m += (int64_t) gridDim.x * blockDim.x) {
        const int32_t s = slots != nullptr ? slots[m] : (int32_t) m;
        slots1[m]       = s;
        pslots[2 * m]   = s;
        pslots[2 * m + 1] = s;
    }
}

// x[m] = ((ptab[0][prev[m][1]] + ptab[1][prev[m][2]] + ... + ptab[G-2][prev[m][G-1]])
//         + ttab[prev[m][0]]) + text[m], in fp32 in that order
// (sum_code_embeddings, code-predictor.cpp:84-109, then ggml_add(acoustic,
// semantic) at model.cpp:1344-1350 and build_talker_step_input's
// ggml_add(summed, text), talker.cpp:120-133).
__global__ void frame_embed_kernel(const uint8_t * const * __restrict__ ptabs, int64_t prows,
                                   const uint8_t * __restrict__ ttab, int64_t trows, size_t row_bytes,
                                   const int32_t * __restrict__ prev, int G, const float * __restrict__ text,
                                   float * __restrict__ x, int64_t M, int64_t H) {
    const int64_t total = M * H;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t   m  = i / H;
        const int64_t   k  = i % H;
        const int32_t * pc = prev + m * G;
        float           acc = table_value(ptabs[0], row_bytes, prows, pc[1], k);
        for (int g = 2; g < G; ++g) {
            acc = __fadd_rn(acc, table_value(ptabs[g - 1], row_bytes, prows, pc[g], k));
        }
        acc  = __fadd_rn(acc, table_value(ttab, row_bytes, trows, pc[0], k));
        x[i] = __fadd_rn(acc, text[i]);
    }
}

// The predictor prefill's input, ggml_concat(t_hidden, get_rows(ttab, code0), 1)
// (model.cpp:1444-1451) per stream: xp[2m] = hidden[m], xp[2m+1] = ttab[code0[m]].
__global__ void frame_prefill_kernel(const float * __restrict__ hidden, const uint8_t * __restrict__ ttab,
                                     int64_t trows, size_t row_bytes, const int32_t * __restrict__ code0,
                                     float * __restrict__ xp, int64_t M, int64_t H) {
    const int64_t total = M * H;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t m = i / H;
        const int64_t k = i % H;
        xp[(2 * m) * H + k]     = hidden[i];
        xp[(2 * m + 1) * H + k] = table_value(ttab, row_bytes, trows, code0[m], k);
    }
}

// (value, index) ordering of std::max_element over the row: a larger value
// wins, equal values keep the lower index, NaN never wins.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// One CTA per stream: code = replay[m][g], or the first index of the largest
// logit of row (m * row_mul + row_add), after the repetition penalty when
// `history` is given: a logit whose code is in the stream's history becomes
// v / penalty if v > 0, else v * penalty (apply_repetition_penalty,
// code-predictor-host.cpp:51-69).  std::max_element's sequential rule with
// NaN: a NaN at index 0 is never replaced (result 0); a NaN elsewhere never
// wins.  Writes codes[m][g] and cur[m]; marks the code in the history.
__global__ void __launch_bounds__(kSelectThreads)
frame_select_kernel(const float * __restrict__ logits, int64_t vocab, int row_mul, int row_add,
                    const int32_t * __restrict__ replay, int G, int g, float penalty, uint8_t * __restrict__ history,
                    const int32_t * __restrict__ slots1, int64_t n_slots, int32_t * __restrict__ codes,
                    int32_t * __restrict__ cur) {
    const int64_t m = blockIdx.x;
    __shared__ float sv[kSelectThreads / 32];
    __shared__ int   si[kSelectThreads / 32];
    int code = 0;
    if (replay != nullptr) {
        code = replay[m * G + g];
    } else {
        const float *   row  = logits + ((int64_t) m * row_mul + row_add) * vocab;
        const int32_t   slot = slots1 != nullptr ? slots1[m] : (int32_t) m;
        const uint8_t * hist = (history != nullptr && slot >= 0 && slot < n_slots) ? history + slot * vocab : nullptr;
        const bool      pen  = hist != nullptr && penalty > 1.0f;
        float           bv   = -INFINITY;
        int             bi   = INT_MAX;
        for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
            float v = row[i];
            if (pen && hist[i]) {
                v = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
            }
            if (!(v != v) && (bi == INT_MAX || better(v, (int) i, bv, bi))) {
                bv = v;
                bi = (int) i;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int   oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != INT_MAX && (bi == INT_MAX || better(ov, oi, bv, bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if ((threadIdx.x & 31) == 0) {
            sv[threadIdx.x >> 5] = bv;
            si[threadIdx.x >> 5] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            bv = sv[0];
            bi = si[0];
            for (int w = 1; w < (int) (blockDim.x >> 5); ++w) {
                if (si[w] != INT_MAX && (bi == INT_MAX || better(sv[w], si[w], bv, bi))) {
                    bv = sv[w];
                    bi = si[w];
                }
            }
            float v0 = row[0];
            if (pen && hist[0]) {
                v0 = v0 > 0.0f ? __fdiv_rn(v0, penalty) : __fmul_rn(v0, penalty);
            }
            code = (bi == INT_MAX || v0 != v0) ? 0 : bi;
            if (hist != nullptr) {
                history[slot * vocab + code] = 1;
            }
        }
    }
    if (threadIdx.x == 0) {
        codes[m * G + g] = code;
        cur[m]           = code;
    }
}

__global__ void fill_positions_kernel(int32_t * __restrict__ ppos, int32_t * __restrict__ spos, int64_t max_m,
                                      int G) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < 2 * max_m; i += (int64_t) gridDim.x * blockDim.x) {
        ppos[i] = (int32_t) (i & 1);
    }
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t) (G - 2) * max_m;
         i += (int64_t) gridDim.x * blockDim.x) {
        spos[i] = (int32_t) (i / max_m) + 2;  // group g = i / max_m + 1 sits at position g + 1
    }
}

// y[m][n] += b[n] (the projection's bias: ggml_add(mul_mat(W, x), b)).
__global__ void add_bias_kernel(float * __restrict__ y, const float * __restrict__ b, int64_t M, int64_t N) {
    const int64_t total = M * N;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        y[i] = __fadd_rn(y[i], b[i % N]);
    }
}

// y[m][n] = silu(y[m][n] + b[n]): the text projection's first Linear and its
// activation (ggml_silu(ggml_add(mul_mat(W1, x), b1)), talker.cpp:45-47).
__global__ void add_bias_silu_kernel(float * __restrict__ y, const float * __restrict__ b, int64_t M, int64_t N) {
    const int64_t total = M * N;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        y[i] = silu_f32(__fadd_rn(y[i], b[i % N]));
    }
}

int frame_grid(int64_t total, int sms) {
    return (int) std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t) sms * 4));
}

}  // namespace
}  // namespace b200q8

using namespace b200q8;

struct b200q8_frame {
    b200q8_chain *       talker    = nullptr;
    b200q8_chain *       predictor = nullptr;
    ChainInfo            ti = {}, pi = {};
    int                  G         = 0;
    float                penalty   = 1.0f;
    int                  mode      = 0;  // the predictor chain's quantizer
    int                  tmode     = 0;  // the talker chain's quantizer
    int64_t              prows     = 0;
    int64_t              max_m     = 0;
    size_t               rb        = 0;  // Q8_0 row bytes at the hidden width
    std::vector<void *>  owned;
    const uint8_t **     ptabs     = nullptr;  // device [G-1]
    std::vector<const uint8_t *> ptabs_host;
    float *              xt        = nullptr;  // [max_m][H]
    float *              thid      = nullptr;  // [max_m][H]
    float *              tlog      = nullptr;  // [max_m][talker vocab]
    float *              th        = nullptr;  // [max_m][H] talker residual stream
    float *              xp        = nullptr;  // [2 max_m][H] predictor input
    float *              ph        = nullptr;  // [2 max_m][H] predictor residual stream
    float *              phid      = nullptr;  // [2 max_m][H] predictor hidden
    float *              plog      = nullptr;  // [2 max_m][predictor vocab]
    int32_t *            cur       = nullptr;  // [max_m]
    int32_t *            slots1    = nullptr;  // [max_m]
    int32_t *            pslots    = nullptr;  // [2 max_m]
    int32_t *            ppos      = nullptr;  // [2 max_m]: 0, 1, 0, 1, ...
    int32_t *            spos      = nullptr;  // [G-2][max_m]: g + 1 for group g
    uint8_t *            history   = nullptr;  // [talker n_slots][talker vocab]
    // input projection (predictor narrower than the talker)
    const uint8_t *      proj_w    = nullptr;  // Q8_0 [predictor hidden rows] of K = talker hidden
    const float *        proj_b    = nullptr;
    float *              xe        = nullptr;  // [max_m][talker hidden] embedded codes
    float *              xq        = nullptr;  // [2 max_m][predictor hidden] projected input rows
    void *               proj_ws   = nullptr;  // MUL_MAT workspace
    // text projection (frames run from text token ids)
    const uint8_t *      txt_emb   = nullptr;  // Q8_0 [txt_rows][txt_hidden]
    int64_t              txt_rows  = 0;
    int64_t              txt_hidden = 0;
    const uint8_t *      txt_w1    = nullptr;  // Q8_0 [txt_hidden rows] of K = txt_hidden
    const float *        txt_b1    = nullptr;
    const uint8_t *      txt_w2    = nullptr;  // Q8_0 [talker hidden rows] of K = txt_hidden
    const float *        txt_b2    = nullptr;
    float *              tx0       = nullptr;  // [max_m][txt_hidden] embedded text tokens
    float *              tx1       = nullptr;  // [max_m][txt_hidden] after fc1 + silu
    float *              tx2       = nullptr;  // [max_m][talker hidden] text rows
    void *               txt_ws    = nullptr;  // MUL_MAT workspace
    cudaStream_t         cap       = nullptr;

    struct Graph {
        b200q8_frame_args a;
        cudaGraphExec_t   exec;
    };
    std::vector<Graph> graphs;
};

namespace {

bool same_args(const b200q8_frame_args & x, const b200q8_frame_args & y) {
    return x.M == y.M && x.skip_talker == y.skip_talker && x.text == y.text && x.prev == y.prev && x.pos == y.pos &&
           x.slots == y.slots && x.replay == y.replay && x.codes == y.codes && x.hidden == y.hidden &&
           x.talker_logits == y.talker_logits && x.text_ids == y.text_ids;
}

void frame_free(b200q8_frame * f) {
    if (f == nullptr) {
        return;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(f->ti.device);
    for (auto & g : f->graphs) {
        cudaGraphExecDestroy(g.exec);
    }
    for (void * p : f->owned) {
        cudaFree(p);
    }
    if (f->cap) {
        cudaStreamDestroy(f->cap);
    }
    cudaSetDevice(prev);
    delete f;
}

// The talker's text rows for M token ids (build_text_projection,
// talker.cpp:37-50): out = W2 * Q(silu(W1 * Q(text_embedding[id]) + b1)) + b2.
// h1 (nullable) receives silu(W1 * Q(.) + b1), [M][text hidden].
cudaError_t enqueue_text(b200q8_frame * f, cudaStream_t st, const int32_t * ids, int64_t M, float * h1, float * out) {
    const int64_t Th  = f->txt_hidden, H = f->ti.hidden;
    const int     sms = f->ti.sms;
    const size_t  rt  = (size_t) (Th / kQK) * kBlockBytes;
    float *       y1  = h1 != nullptr ? h1 : f->tx1;
    cudaError_t   e   = launch_dequant_rows(f->txt_emb, rt, f->txt_rows, ids, M, Th, f->tx0,
                                            (size_t) Th * sizeof(float), st, sms);
    if (e == cudaSuccess) {
        e = launch_gemm(f->txt_w1, rt, Th, Th, f->tx0, (size_t) Th, M, y1, (size_t) Th, f->tmode, f->txt_ws, st, sms);
    }
    if (e == cudaSuccess) {
        add_bias_silu_kernel<<<frame_grid(M * Th, sms), 256, 0, st>>>(y1, f->txt_b1, M, Th);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        e = launch_gemm(f->txt_w2, rt, Th, H, y1, (size_t) Th, M, out, (size_t) H, f->tmode, f->txt_ws, st, sms);
    }
    if (e == cudaSuccess) {
        add_bias_kernel<<<frame_grid(M * H, sms), 256, 0, st>>>(out, f->txt_b2, M, H);
        e = cudaGetLastError();
    }
    return e;
}

cudaError_t enqueue_frame(b200q8_frame * f, cudaStream_t st, const b200q8_frame_args & a) {
    const int64_t M = a.M, H = f->ti.hidden;
    const int     sms = f->ti.sms;
    float *       hid = a.hidden != nullptr ? a.hidden : f->thid;
    float *       tlg = a.talker_logits != nullptr ? a.talker_logits : f->tlog;
    frame_setup_kernel<<<1, 256, 0, st>>>(a.slots, f->slots1, f->pslots, M);
    cudaError_t e = cudaGetLastError();
    const float * text = a.text;
    if (e == cudaSuccess && !a.skip_talker && a.text_ids != nullptr) {
        e    = enqueue_text(f, st, a.text_ids, M, nullptr, f->tx2);
        text = f->tx2;
    }
    if (e == cudaSuccess && !a.skip_talker) {
        frame_embed_kernel<<<frame_grid(M * H, sms), 256, 0, st>>>(f->ptabs, f->prows, f->ti.table, f->ti.table_rows,
                                                                 f->rb, a.prev, f->G, text, f->xt, M, H);
        e = cudaGetLastError();
        if (e == cudaSuccess) {
            StepIO io;
            io.M = M; io.x_in = f->xt; io.pos = a.pos; io.slots = f->slots1;
            io.h_out = f->th; io.hidden_out = hid; io.logits = tlg; io.head = 0;
            e = chain_enqueue(f->talker, st, io);
        }
    }
    // codes[0] from the talker's logits
    if (e == cudaSuccess) {
        frame_select_kernel<<<(unsigned) M, kSelectThreads, 0, st>>>(
            tlg, f->ti.vocab, 1, 0, a.replay, f->G, 0, f->penalty, a.replay ? nullptr : f->history, f->slots1,
            f->ti.n_slots, a.codes, f->cur);
        e = cudaGetLastError();
    }
    // predictor prefill: [hidden, ttable[codes[0]]] at positions 0, 1; head 0 on the second
    if (e == cudaSuccess) {
        frame_prefill_kernel<<<frame_grid(M * H, sms), 256, 0, st>>>(hid, f->ti.table, f->ti.table_rows, f->rb, f->cur,
                                                                   f->xp, M, H);
        e = cudaGetLastError();
    }
    // x = W * Q(x) + b for n rows of talker width (the predictor's input projection)
    auto project = [&](const float * x, int64_t n) -> cudaError_t {
        const int64_t Ht = f->ti.hidden, Hp = f->pi.hidden;
        cudaError_t   e2 = launch_gemm(f->proj_w, (size_t) (Ht / kQK) * kBlockBytes, Ht, Hp, x, (size_t) Ht, n, f->xq,
                                       (size_t) Hp, f->mode, f->proj_ws, st, sms);
        if (e2 == cudaSuccess) {
            add_bias_kernel<<<frame_grid(n * Hp, sms), 256, 0, st>>>(f->xq, f->proj_b, n, Hp);
            e2 = cudaGetLastError();
        }
        return e2;
    };
    if (e == cudaSuccess && f->proj_w != nullptr) {
        e = project(f->xp, 2 * M);
    }
    if (e == cudaSuccess) {
        StepIO io;
        io.M = 2 * M; io.x_in = f->proj_w ? f->xq : f->xp; io.pos = f->ppos; io.slots = f->pslots;
        io.h_out = f->ph; io.hidden_out = f->phid; io.logits = f->plog; io.head = 0;
        e = chain_enqueue(f->predictor, st, io);
    }
    if (e == cudaSuccess) {
        frame_select_kernel<<<(unsigned) M, kSelectThreads, 0, st>>>(f->plog, f->pi.vocab, 2, 1, a.replay, f->G, 1,
                                                                      1.0f, nullptr, nullptr, 0, a.codes, f->cur);
        e = cudaGetLastError();
    }
    // groups 1..G-2: embed the last code through its group's table, predict the next
    for (int g = 1; g + 1 < f->G && e == cudaSuccess; ++g) {
        StepIO io;
        io.M = M;
        if (f->proj_w != nullptr) {  // embed at talker width, then project
            e = launch_dequant_rows(f->ptabs_host[g - 1], f->rb, f->prows, f->cur, M, H, f->xe,
                                    (size_t) H * sizeof(float), st, sms);  // row strides in bytes
            if (e == cudaSuccess) e = project(f->xe, M);
            if (e != cudaSuccess) break;
            io.x_in = f->xq;
        } else {
            io.ids = f->cur; io.table = f->ptabs_host[g - 1]; io.table_rows = f->prows;
        }
        io.pos = f->spos + (int64_t) (g - 1) * f->max_m; io.slots = f->slots1;
        io.h_out = f->ph; io.hidden_out = f->phid; io.logits = f->plog; io.head = g;
        e = chain_enqueue(f->predictor, st, io);
        if (e == cudaSuccess) {
            frame_select_kernel<<<(unsigned) M, kSelectThreads, 0, st>>>(f->plog, f->pi.vocab, 1, 0, a.replay, f->G,
                                                                          g + 1, 1.0f, nullptr, nullptr, 0, a.codes,
                                                                          f->cur);
            e = cudaGetLastError();
        }
    }
    return e;
}

}  // namespace

extern "C" {

b200q8_status_t b200q8_frame_create(const b200q8_frame_desc * desc, b200q8_frame ** out) {
    if (desc == nullptr || out == nullptr || desc->talker == nullptr || desc->predictor == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: null argument");
    }
    *out               = nullptr;
    const ChainInfo ti = chain_info(desc->talker), pi = chain_info(desc->predictor);
    const int       G  = desc->groups;
    if (G < 2 || G > 4096 || desc->tables == nullptr || desc->table_rows < 1) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: groups must be >= 2 with G-1 tables of >= 1 row");
    }
    for (int g = 0; g + 1 < G; ++g) {
        if (desc->tables[g] == nullptr || reinterpret_cast<uintptr_t>(desc->tables[g]) % 2 != 0) {
            return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: table %d is null or misaligned", g);
        }
    }
    if (!ti.attn || !pi.attn || ti.n_heads < 1 || pi.n_heads < G - 1) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: both chains need attention and an output desc "
                                                 "(talker >= 1 head, predictor >= groups - 1 heads)");
    }
    if (ti.device != pi.device) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: the chains must share a device");
    }
    const bool proj = desc->input_projection != nullptr || desc->input_projection_bias != nullptr;
    if (proj ? (desc->input_projection == nullptr || desc->input_projection_bias == nullptr ||
                reinterpret_cast<uintptr_t>(desc->input_projection) % 16 != 0 || ti.hidden % 256 != 0 ||
                !gemm_supported(static_cast<const uint8_t *>(desc->input_projection),
                                (size_t) (ti.hidden / kQK) * kBlockBytes, ti.hidden, pi.hidden, 2 * pi.max_m))
             : ti.hidden != pi.hidden) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: a predictor of another width than the talker needs "
                                                 "both the input projection (16-byte aligned Q8_0) and its bias");
    }
    const bool txt = desc->text_embedding != nullptr || desc->text_fc1 != nullptr || desc->text_fc2 != nullptr ||
                     desc->text_fc1_bias != nullptr || desc->text_fc2_bias != nullptr;
    if (txt) {
        const int64_t Th = desc->text_hidden;
        const size_t  rt = Th > 0 ? (size_t) (Th / kQK) * kBlockBytes : 0;
        const int64_t mm = std::min<int64_t>(ti.max_m, pi.max_m / 2);
        if (desc->text_embedding == nullptr || desc->text_fc1 == nullptr || desc->text_fc2 == nullptr ||
            desc->text_fc1_bias == nullptr || desc->text_fc2_bias == nullptr || desc->text_rows < 1 || Th < 256 ||
            Th % 256 != 0 || reinterpret_cast<uintptr_t>(desc->text_embedding) % 2 != 0 || mm < 1 ||
            !gemm_supported(static_cast<const uint8_t *>(desc->text_fc1), rt, Th, Th, mm) ||
            !gemm_supported(static_cast<const uint8_t *>(desc->text_fc2), rt, Th, ti.hidden, mm)) {
            return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: a text projection needs the embedding, both "
                                                     "Linears (16-byte aligned Q8_0) and both biases, with a text "
                                                     "width that is a multiple of 256");
        }
    }
    if (pi.n_ctx < G || pi.n_slots < ti.n_slots) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: the predictor needs n_ctx >= groups and n_slots >= "
                                                 "the talker's");
    }
    const int64_t max_m = std::min<int64_t>(ti.max_m, pi.max_m / 2);
    if (max_m < 1) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_create: the predictor's max_m must be >= 2");
    }
    b200q8_frame * f = new (std::nothrow) b200q8_frame();
    if (f == nullptr) {
        return set_error(B200Q8_ERR_OOM, "frame_create: out of host memory");
    }
    f->talker    = desc->talker;
    f->predictor = desc->predictor;
    f->ti        = ti;
    f->pi        = pi;
    f->G         = G;
    f->penalty   = desc->repetition_penalty;
    f->prows     = desc->table_rows;
    f->max_m     = max_m;
    f->rb        = (size_t) (ti.hidden / kQK) * kBlockBytes;
    f->mode      = chain_mode(desc->predictor);
    f->tmode     = chain_mode(desc->talker);
    if (txt) {
        f->txt_emb    = static_cast<const uint8_t *>(desc->text_embedding);
        f->txt_rows   = desc->text_rows;
        f->txt_hidden = desc->text_hidden;
        f->txt_w1     = static_cast<const uint8_t *>(desc->text_fc1);
        f->txt_b1     = desc->text_fc1_bias;
        f->txt_w2     = static_cast<const uint8_t *>(desc->text_fc2);
        f->txt_b2     = desc->text_fc2_bias;
    }
    f->proj_w    = static_cast<const uint8_t *>(desc->input_projection);
    f->proj_b    = desc->input_projection_bias;
    for (int g = 0; g + 1 < G; ++g) {
        f->ptabs_host.push_back(static_cast<const uint8_t *>(desc->tables[g]));
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(ti.device);
    const int64_t H = ti.hidden;
    auto alloc = [&](size_t bytes) -> void * {
        void * p = nullptr;
        if (e == cudaSuccess) e = cudaMalloc(&p, std::max<size_t>(bytes, 256));
        if (e == cudaSuccess) { f->owned.push_back(p); e = cudaMemset(p, 0, std::max<size_t>(bytes, 256)); }
        return e == cudaSuccess ? p : nullptr;
    };
    f->ptabs   = static_cast<const uint8_t **>(alloc(sizeof(void *) * (size_t) (G - 1)));
    f->xt      = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * H)));
    f->th      = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * H)));
    f->thid    = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * H)));
    f->tlog    = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * ti.vocab)));
    f->xp      = static_cast<float *>(alloc(sizeof(float) * (size_t) (2 * max_m * H)));
    const int64_t Hp = pi.hidden;
    f->ph      = static_cast<float *>(alloc(sizeof(float) * (size_t) (2 * max_m * Hp)));
    f->phid    = static_cast<float *>(alloc(sizeof(float) * (size_t) (2 * max_m * Hp)));
    if (f->proj_w != nullptr) {
        f->xe      = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * H)));
        f->xq      = static_cast<float *>(alloc(sizeof(float) * (size_t) (2 * max_m * Hp)));
        f->proj_ws = alloc(gemm_workspace_bytes(H, 2 * max_m));
    }
    if (f->txt_emb != nullptr) {
        const int64_t Th = f->txt_hidden;
        f->tx0    = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * Th)));
        f->tx1    = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * Th)));
        f->tx2    = static_cast<float *>(alloc(sizeof(float) * (size_t) (max_m * H)));
        f->txt_ws = alloc(gemm_workspace_bytes(Th, max_m));
    }
    f->plog    = static_cast<float *>(alloc(sizeof(float) * (size_t) (2 * max_m * pi.vocab)));
    f->cur     = static_cast<int32_t *>(alloc(sizeof(int32_t) * (size_t) max_m));
    f->slots1  = static_cast<int32_t *>(alloc(sizeof(int32_t) * (size_t) max_m));
    f->pslots  = static_cast<int32_t *>(alloc(sizeof(int32_t) * (size_t) (2 * max_m)));
    f->ppos    = static_cast<int32_t *>(alloc(sizeof(int32_t) * (size_t) (2 * max_m)));
    f->spos    = static_cast<int32_t *>(alloc(sizeof(int32_t) * (size_t) (std::max(G - 2, 1) * max_m)));
    f->history = static_cast<uint8_t *>(alloc((size_t) ti.n_slots * (size_t) ti.vocab));
    if (e == cudaSuccess) {
        e = cudaMemcpy(f->ptabs, f->ptabs_host.data(), sizeof(void *) * (size_t) (G - 1), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) {
        fill_positions_kernel<<<frame_grid(std::max<int64_t>(2, G - 2) * max_m, ti.sms), 256>>>(f->ppos, f->spos, max_m, G);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&f->cap, cudaStreamNonBlocking);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        frame_free(f);
        return cuda_error(e, "frame_create");
    }
    *out = f;
    return B200Q8_OK;
}

b200q8_status_t b200q8_frame_run(b200q8_frame * f, const b200q8_frame_args * a, b200q8_stream_t stream) {
    if (f == nullptr || a == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_run: null argument");
    }
    if (a->M < 1 || a->M > f->max_m || a->codes == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_run: M (%lld) must be in [1, %lld] and codes given",
                         (long long) a->M, (long long) f->max_m);
    }
    if (a->skip_talker ? (a->hidden == nullptr || a->talker_logits == nullptr)
                       : ((a->text == nullptr && a->text_ids == nullptr) || a->prev == nullptr || a->pos == nullptr)) {
        return set_error(B200Q8_ERR_INVALID_ARG, a->skip_talker ? "frame_run: skip_talker needs hidden and talker_logits"
                                                                : "frame_run: needs text (or text_ids), prev and pos");
    }
    if (a->text_ids != nullptr && !a->skip_talker && f->txt_emb == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_run: text_ids given to a frame built without a text projection");
    }
    if (a->slots == nullptr && a->M > f->ti.n_slots) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_run: M (%lld) streams need explicit slots beyond n_slots",
                         (long long) a->M);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(f->ti.device);
    if (e != cudaSuccess) {
        return cuda_error(e, "frame_run: cudaSetDevice");
    }
    b200q8_frame_args key = *a;
    key.skip_talker       = a->skip_talker ? 1 : 0;
    cudaGraphExec_t exec  = nullptr;
    for (size_t i = 0; i < f->graphs.size(); ++i) {
        if (same_args(f->graphs[i].a, key)) {
            exec = f->graphs[i].exec;
            std::rotate(f->graphs.begin() + i, f->graphs.begin() + i + 1, f->graphs.end());
            break;
        }
    }
    if (exec == nullptr) {
        for (int attempt = 0; attempt < 2; ++attempt) {
            cudaGraph_t graph = nullptr;
            exec              = nullptr;
            e                 = cudaStreamBeginCapture(f->cap, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                const cudaError_t e2 = enqueue_frame(f, f->cap, key);
                e                    = cudaStreamEndCapture(f->cap, &graph);
                if (e2 != cudaSuccess) {
                    e = e2;
                }
            }
            if (e == cudaSuccess) {
                e = cudaGraphInstantiate(&exec, graph, 0);
            }
            if (graph) {
                cudaGraphDestroy(graph);
            }
            const bool persistent = chain_persistent_in_graph(f->talker, false) ||
                                    chain_persistent_in_graph(f->predictor, false);
            if (e == cudaSuccess || attempt > 0 || !persistent) {
                break;
            }
            // a graph that cannot hold the persistent steps' cooperative launches: per-op steps instead
            cudaGetLastError();
            chain_persistent_in_graph(f->talker, true);
            chain_persistent_in_graph(f->predictor, true);
        }
        if (e != cudaSuccess) {
            cudaSetDevice(prev);
            return cuda_error(e, "frame_run: graph capture");
        }
        if (f->graphs.size() >= (size_t) kMaxFrameGraphs) {
            cudaGraphExecDestroy(f->graphs.front().exec);
            f->graphs.erase(f->graphs.begin());
        }
        f->graphs.push_back({ key, exec });
    }
    e = cudaGraphLaunch(exec, reinterpret_cast<cudaStream_t>(stream));
    cudaSetDevice(prev);
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "frame_run: graph launch");
}

b200q8_status_t b200q8_frame_text_rows(b200q8_frame * f, const int32_t * text_ids, int64_t M, float * h1,
                                       float * out, b200q8_stream_t stream) {
    if (f == nullptr || text_ids == nullptr || out == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_text_rows: null argument");
    }
    if (f->txt_emb == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_text_rows: the frame was built without a text projection");
    }
    if (M < 1 || M > f->max_m) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_text_rows: M (%lld) must be in [1, %lld]", (long long) M,
                         (long long) f->max_m);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(f->ti.device);
    if (e == cudaSuccess) {
        e = enqueue_text(f, reinterpret_cast<cudaStream_t>(stream), text_ids, M, h1, out);
    }
    cudaSetDevice(prev);
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "frame_text_rows");
}

b200q8_status_t b200q8_frame_reset_history(b200q8_frame * f, int32_t slot, b200q8_stream_t stream) {
    if (f == nullptr || slot >= f->ti.n_slots) {
        return set_error(B200Q8_ERR_INVALID_ARG, "frame_reset_history: bad frame or slot");
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(f->ti.device);
    if (e == cudaSuccess) {
        const size_t v = (size_t) f->ti.vocab;
        e = slot < 0 ? cudaMemsetAsync(f->history, 0, (size_t) f->ti.n_slots * v, reinterpret_cast<cudaStream_t>(stream))
                     : cudaMemsetAsync(f->history + (size_t) slot * v, 0, v, reinterpret_cast<cudaStream_t>(stream));
    }
    cudaSetDevice(prev);
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "frame_reset_history");
}

void b200q8_frame_destroy(b200q8_frame * f) {
    frame_free(f);
}

}  // extern "C"
