// chain.cu -- the talker-shaped decode step as one replayable launch sequence.
//
// The reference rebuilds and computes a ggml graph per frame on the CPU
// (src/arch/qwen3-tts/model.cpp:101-126 GraphRun::run, talker.cpp:135-185,
// operations.cpp:44-148).  Here the step is a fixed sequence of kernels:
//
//   embed: h = x_in + get_rows(table, ids)
//   per layer:  qkv  = W_qkv * Q(rms_norm(h) * norm_in)      (one GEMV, 4096 rows)
//               h1   = h + W_o * Q(attend(v))                (GEMV + residual)
//               gu   = W_gu * Q(rms_norm(h1) * norm_post)    (one GEMV, 6144 rows)
//               h    = h1 + W_d * Q(silu(g) * u)             (GEMV + residual)
//
// where attend is either attention over a single cached position (the
// softmax of one score is 1, so query head j reads kv head j / (n_head /
// n_kv)) or, for chains built with an attention desc, the reference's
// attention over a per-slot KV cache (attention.cu).  The norms, the GQA
// expansion and SwiGLU are folded into the prologue of the GEMV that consumes
// them, the residual adds into its epilogue, so the step is 1 + 4 * n_layers
// kernels (+ 2 per layer with attention, + 1 with an output head).  They are
// launched with programmatic dependent launch (each GEMV streams its weights
// into shared memory before waiting on its predecessor) and captured once per
// argument set into a CUDA graph that run() replays.
#include "chain.h"
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

namespace b200q8 {
b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...);
b200q8_status_t cuda_error(cudaError_t e, const char * what);
int             current_sm_count();

namespace {

// From this many tokens on a step runs as the per-op int8 tensor-core GEMM
// chain: its MMAs take 8 tokens at once, so 3 to 8 tokens cost about what 8
// do (0.755 ms per 28-layer step at M = 4 and at M = 8 on B200, against
// 0.566 ms for the persistent step at M = 2 and 0.97 / 1.88 ms for a
// persistent step of 4 / 8 tokens).
constexpr int64_t kBatchedMinM = 3;

// h = x_in + get_rows(table, ids); a NULL ids or x_in drops that term (the
// other is copied exactly).
__global__ void embed_add_kernel(const uint8_t * __restrict__ table, size_t table_stride, int64_t table_rows,
                                 const int32_t * __restrict__ ids, const float * __restrict__ x_in,
                                 float * __restrict__ h, int64_t M, int64_t H) {
    const int64_t total = M * H;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t m = i / H;
        const int64_t k = i % H;
        if (ids == nullptr) {
            h[i] = x_in[i];
            continue;
        }
        const int64_t r = ids[m];
        float         e = 0.0f;
        if (r < 0 || r >= table_rows) {
            if (k == 0) {
                record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
            }
        } else {
            const uint8_t * blk = table + r * table_stride + (k / kQK) * kBlockBytes;
            const float     d   = __half2float(__ushort_as_half((unsigned short) (blk[0] | (blk[1] << 8))));
            e                   = __fmul_rn((float) (int8_t) blk[2 + k % kQK], d);
        }
        h[i] = x_in != nullptr ? __fadd_rn(x_in[i], e) : e;
    }
}

enum Buf : int {
    kN1 = 0, kQkv, kAttn, kO, kH1, kN2, kGu, kS, kDown, kHout, kNumBufs
};

}  // namespace
}  // namespace b200q8

using namespace b200q8;

struct b200q8_chain {
    int                          device = 0;
    b200q8_chain_desc            d      = {};
    std::vector<b200q8_layer>    layers;
    std::vector<void *>          owned;  // device allocations to free
    std::vector<const uint8_t *> w_qkv, w_o, w_gu, w_d;
    size_t                       rb_h = 0, rb_q = 0, rb_i = 0;
    int64_t                      qkv_dim = 0;
    float *                      act     = nullptr;  // per-layer activation buffers
    size_t                       buf_off[kNumBufs] = {};
    size_t                       buf_stride[kNumBufs] = {};
    size_t                       layer_floats = 0;
    float *                      h0           = nullptr;
    cudaStream_t                 cap_stream   = nullptr;
    int                          sms          = 148;
    // persistent single-launch step (M <= 2)
    StepLayerDev *               step_layers  = nullptr;  // device array
    unsigned long long *         ll           = nullptr;
    size_t                       ll_layer     = 0;
    unsigned *                   sync         = nullptr;
    bool                         persistent   = false;
    int                          persistent_max_m = 0;  // largest M the persistent step takes
    int                          ll_m         = 2;      // token stride of the hand-off words
    bool                         persistent_in_graph = true;  // cleared if a graph cannot hold its launch
    void *                       timeline     = nullptr;  // B200Q8_TIMELINE analysis builds only
    void *                       planes       = nullptr;  // batched path (M >= kBatchedMinM): GEMM code/scale planes
    GemmSplit                    split        = {};       // batched path: split-K partials and counters
    // attention with a KV cache (desc.attention != nullptr)
    bool                         attn         = false;
    b200q8_attention_desc        ad           = {};
    std::vector<const float *>   q_norm, k_norm;
    float *                      kv_cache     = nullptr;  // K then V: [n_layers][n_slots][n_ctx][KV] each
    float *                      q_rot        = nullptr;  // [max_m][Q]
    float *                      attn_partial = nullptr;  // [max_m][n_head][kAttnMaxSplits][head_dim + 2]
    unsigned *                   attn_count   = nullptr;  // [max_m][n_head]
    // output stage (desc.output != nullptr)
    int                          n_heads      = 0;
    const float *                out_norm     = nullptr;
    std::vector<const uint8_t *> heads;
    int64_t                      vocab        = 0;
    float *                      h_last       = nullptr;  // [max_m][hidden] when the caller passes no h_out
    float *                      hid          = nullptr;  // [max_m][hidden] when the caller passes no hidden_out
    float *                      lg           = nullptr;  // [max_m][vocab] when the caller passes no logits

    struct Graph {
        StepIO          io;
        cudaGraphExec_t exec;
    };

    // attention arguments of layer l for tokens [m0, m0 + M)
    AttnArgs attn_args(int l, float * qkv, size_t qkv_stride, float * out, size_t out_stride, const int32_t * pos,
                       const int32_t * slots, int64_t m0) const {
        AttnArgs a   = {};
        const int64_t KV = d.n_kv * d.head_dim;
        a.qkv        = qkv;
        a.qkv_stride = qkv_stride;
        a.n_head     = (int) d.n_head;
        a.n_kv       = (int) d.n_kv;
        a.head_dim   = (int) d.head_dim;
        a.eps        = d.eps;
        a.rope_theta = ad.rope_theta;
        a.q_norm     = q_norm[l];
        a.k_norm     = k_norm[l];
        a.pos        = pos + m0;
        a.slots      = slots ? slots + m0 : nullptr;
        a.slot_base  = (int) m0;
        a.n_ctx      = (int) ad.n_ctx;
        a.n_slots    = (int) ad.n_slots;
        a.q_rot      = q_rot + m0 * d.n_head * d.head_dim;
        const size_t layer = (size_t) ad.n_slots * ad.n_ctx * KV;
        a.k_cache    = kv_cache + (size_t) l * layer;
        a.v_cache    = kv_cache + (size_t) d.n_layers * layer + (size_t) l * layer;
        a.partial    = attn_partial + m0 * d.n_head * kAttnMaxSplits * (d.head_dim + 2);
        a.counters   = attn_count + m0 * d.n_head;
        a.out        = out;
        a.out_stride = out_stride;
        return a;
    }
    std::vector<Graph> graphs;

    float * buf(int layer, int which) { return act + (size_t) layer * layer_floats + buf_off[which]; }
};

namespace {

void chain_free(b200q8_chain * c) {
    if (c == nullptr) {
        return;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    for (auto & g : c->graphs) {
        cudaGraphExecDestroy(g.exec);
    }
    for (void * p : c->owned) {
        cudaFree(p);
    }
    if (c->cap_stream) {
        cudaStreamDestroy(c->cap_stream);
    }
    cudaSetDevice(prev);
    delete c;
}

// Returns a contiguous copy base for [a | b | c] row blocks, or a if they are
// already contiguous (no copy).
const uint8_t * contiguous(b200q8_chain * c, const void * a, size_t a_bytes, const void * b, size_t b_bytes,
                           const void * e, size_t e_bytes, cudaError_t & err) {
    const uint8_t * pa = static_cast<const uint8_t *>(a);
    if (pa + a_bytes == b && (e == nullptr || static_cast<const uint8_t *>(b) + b_bytes == e)) {
        return pa;
    }
    void * dst = nullptr;
    err        = cudaMalloc(&dst, a_bytes + b_bytes + e_bytes);
    if (err != cudaSuccess) {
        return nullptr;
    }
    c->owned.push_back(dst);
    uint8_t * o = static_cast<uint8_t *>(dst);
    err         = cudaMemcpy(o, a, a_bytes, cudaMemcpyDeviceToDevice);
    if (err == cudaSuccess) {
        err = cudaMemcpy(o + a_bytes, b, b_bytes, cudaMemcpyDeviceToDevice);
    }
    if (err == cudaSuccess && e != nullptr) {
        err = cudaMemcpy(o + a_bytes + b_bytes, e, e_bytes, cudaMemcpyDeviceToDevice);
    }
    return o;
}

// The persistent single-launch step's arguments for io; false when the step
// cannot run it (M > 2, a shape or head it does not support, or disabled).
bool persistent_args(b200q8_chain * c, const StepIO & io, StepArgs & a) {
    if (!c->persistent || io.M > c->persistent_max_m || (io.M >= kBatchedMinM && c->planes != nullptr)) {
        return false;
    }
    const b200q8_chain_desc & d = c->d;
    a = StepArgs();
    a.layers = c->step_layers; a.n_layers = d.n_layers;
    a.H = (int) d.hidden; a.Q = (int) (d.n_head * d.head_dim); a.KV = (int) (d.n_kv * d.head_dim);
    a.I = (int) d.inter; a.head_dim = (int) d.head_dim; a.group = (int) (d.n_head / d.n_kv); a.eps = d.eps;
    while ((1 << a.lg_head_dim) < a.head_dim) ++a.lg_head_dim;
    while ((1 << a.lg_group) < a.group) ++a.lg_group;
    a.rb_h = c->rb_h; a.rb_q = c->rb_q; a.rb_i = c->rb_i;
    a.table = io.table; a.table_rows = io.table_rows;
    a.ids = io.ids; a.x_in = io.x_in; a.h_out = io.h_out; a.M = (int) io.M; a.mode = d.mode;
    a.ll = c->ll; a.ll_layer = c->ll_layer; a.ll_m = c->ll_m;
    a.trace = c->act; a.trace_layer = c->layer_floats;
    for (int i = 0; i < kNumBufs; ++i) a.trace_off[i] = c->buf_off[i];
    a.sync = c->sync;
    if (c->attn) {
        a.attn = 1; a.rope_theta = c->ad.rope_theta; a.pos = io.pos; a.slots = io.slots;
        a.n_ctx = (int) c->ad.n_ctx; a.n_cache_slots = (int) c->ad.n_slots;
        const size_t layer = (size_t) c->ad.n_slots * c->ad.n_ctx * (d.n_kv * d.head_dim);
        a.k_cache = c->kv_cache;
        a.v_cache = c->kv_cache + (size_t) d.n_layers * layer;
    }
    if (io.hidden_out != nullptr) {
        a.out_norm = c->out_norm; a.head = c->heads[io.head]; a.vocab = (int) c->vocab;
        a.hidden_out = io.hidden_out; a.logits = io.logits;
    }
#ifdef B200Q8_TIMELINE
    a.timeline = static_cast<unsigned long long *>(c->timeline);  // allocated by chain_create
#endif
    return decode_step_supported(a, c->sms);
}

// M >= kBatchedMinM: per op, a per-token prologue kernel (norm / GQA / SwiGLU + residual,
// quantized into code and scale planes) then the int8 tensor-core GEMM;
// 2 launches per op with programmatic dependent launch between them.
cudaError_t enqueue_step_batched(b200q8_chain * c, cudaStream_t st, const StepIO & io) {
    const b200q8_chain_desc & d = c->d;
    const int64_t   M = io.M;
    const int32_t * pos = io.pos, * slots = io.slots;
    float *         h_out = io.h_out;
    const int64_t H = d.hidden, Q = d.n_head * d.head_dim, KV = d.n_kv * d.head_dim, I = d.inter;
    const int     hd = (int) d.head_dim, grp = (int) (d.n_head / d.n_kv);
    uint8_t *     xrec = static_cast<uint8_t *>(c->planes);
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < d.n_layers && e == cudaSuccess; ++l) {
        auto B = [&](int layer, int which) { return c->buf(layer, which); };
        const float * h_in   = l == 0 ? c->h0 : B(l - 1, kHout);
        // qkv: n1 = rms_norm(h) * norm_in with h = h1(l-1) + d(l-1)
        if (l == 0) {
            e = launch_stage_rows(0, c->h0, nullptr, (size_t) H, nullptr, 0, c->layers[l].norm_in, d.eps, (int) H, hd,
                                  grp, B(l, kN1), (size_t) H, M, d.mode, xrec, st, true);
        } else {
            e = launch_stage_rows(0, B(l - 1, kH1), B(l - 1, kDown), (size_t) H, B(l - 1, kHout), (size_t) H,
                                  c->layers[l].norm_in, d.eps, (int) H, hd, grp, B(l, kN1), (size_t) H, M, d.mode, xrec,
                                  st, true);
        }
        if (e == cudaSuccess)
            e = launch_gemm_staged(c->w_qkv[l], c->rb_h, H, c->qkv_dim, xrec, M, B(l, kQkv),
                                   (size_t) c->qkv_dim, st, c->sms, true);
        // o: attend(v) -- over the cache when the chain has attention, else the single cached position
        if (e == cudaSuccess && c->attn) {
            const AttnArgs aa = c->attn_args(l, B(l, kQkv), (size_t) c->qkv_dim, B(l, kAttn), (size_t) Q, pos, slots, 0);
            e = launch_attention(aa, M, attention_splits(M, (int) d.n_head, c->sms), st, true);
            if (e == cudaSuccess)
                e = launch_stage_rows(3, B(l, kAttn), nullptr, (size_t) Q, nullptr, 0, nullptr, d.eps, (int) Q, hd,
                                      grp, nullptr, 0, M, d.mode, xrec, st, true);
        } else if (e == cudaSuccess) {
            e = launch_stage_rows(1, B(l, kQkv) + Q + KV, nullptr, (size_t) c->qkv_dim, nullptr, 0, nullptr, d.eps,
                                  (int) Q, hd, grp, B(l, kAttn), (size_t) Q, M, d.mode, xrec, st, true);
        }
        if (e == cudaSuccess)
            e = launch_gemm_staged(c->w_o[l], c->rb_q, Q, H, xrec, M, B(l, kO), (size_t) H, st, c->sms, true,
                                   &c->split);
        // gate|up: n2 = rms_norm(h1) * norm_post with h1 = h + o
        if (e == cudaSuccess)
            e = launch_stage_rows(0, h_in, B(l, kO), (size_t) H, B(l, kH1), (size_t) H, c->layers[l].norm_post, d.eps,
                                  (int) H, hd, grp, B(l, kN2), (size_t) H, M, d.mode, xrec, st, true);
        if (e == cudaSuccess)
            e = launch_gemm_staged(c->w_gu[l], c->rb_h, H, 2 * I, xrec, M, B(l, kGu), (size_t) (2 * I), st,
                                   c->sms, true);
        // down: silu(g) * u
        if (e == cudaSuccess)
            e = launch_stage_rows(2, B(l, kGu), B(l, kGu) + I, (size_t) (2 * I), nullptr, 0, nullptr, d.eps, (int) I, hd,
                                  grp, B(l, kS), (size_t) I, M, d.mode, xrec, st, true);
        if (e == cudaSuccess)
            e = launch_gemm_staged(c->w_d[l], c->rb_i, I, H, xrec, M, B(l, kDown), (size_t) H, st, c->sms,
                                   true, &c->split);
    }
    if (e == cudaSuccess) {
        const int L = d.n_layers - 1;
        e           = launch_residual_rows(c->buf(L, kH1), c->buf(L, kDown), (size_t) H, h_out, (size_t) H, (int) H, M,
                                           st, true);
    }
    // output: hidden = rms_norm(h) * norm, logits = head * Q(hidden)
    if (e == cudaSuccess && io.hidden_out != nullptr) {
        e = launch_stage_rows(0, h_out, nullptr, (size_t) H, nullptr, 0, c->out_norm, d.eps, (int) H, hd, grp,
                              io.hidden_out, (size_t) H, M, d.mode, xrec, st, true);
        if (e == cudaSuccess)
            e = launch_gemm_staged(c->heads[io.head], c->rb_h, H, c->vocab, xrec, M, io.logits, (size_t) c->vocab, st,
                                   c->sms, true);
    }
    return e;
}

cudaError_t enqueue_step(b200q8_chain * c, cudaStream_t st, const StepIO & io) {
    const b200q8_chain_desc & d = c->d;
    const int64_t H = d.hidden, Q = d.n_head * d.head_dim, KV = d.n_kv * d.head_dim, I = d.inter;
    const int64_t   M = io.M;
    const int32_t * pos = io.pos, * slots = io.slots;
    float *         h_out = io.h_out;
    StepArgs        sa;
    if (c->persistent_in_graph && persistent_args(c, io, sa)) {
        return launch_decode_step(sa, c->sms, st);
    }
    {
        const int64_t total = M * H;
        const int     grid  = (int) std::min<int64_t>((total + 255) / 256, (int64_t) c->sms * 4);
        embed_add_kernel<<<grid, 256, 0, st>>>(io.table, (size_t) c->rb_h, io.table_rows, io.ids, io.x_in, c->h0, M,
                                                H);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            return e;
        }
    }
    if (M >= kBatchedMinM && c->planes != nullptr) {
        return enqueue_step_batched(c, st, io);
    }
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        const int   mc = (int) std::min<int64_t>(M - m0, 8);
        const float * h = c->h0 + m0 * H;
        for (int l = 0; l < d.n_layers; ++l) {
            const bool last = l == d.n_layers - 1;
            auto       B    = [&](int which) { return c->buf(l, which) + m0 * c->buf_stride[which]; };
            GemvParams p    = {};
            p.M             = mc;
            p.mode          = d.mode;
            p.eps           = d.eps;
            // qkv = W_qkv * Q(rms_norm(h) * norm_in)
            p.w = c->w_qkv[l]; p.row_bytes = c->rb_h; p.K = (int) H; p.N = (int) c->qkv_dim;
            p.pro = kProRmsNorm; p.x = h; p.x_stride = (size_t) H; p.norm_w = c->layers[l].norm_in;
            p.pro_out = B(kN1); p.pro_out_stride = (size_t) H;
            p.y = B(kQkv); p.y_stride = (size_t) c->qkv_dim; p.res = nullptr; p.y_res = nullptr;
            cudaError_t e = launch_gemv(p, st, c->sms, true);
            if (e != cudaSuccess) return e;
            // h1 = h + W_o * Q(attend(v))
            p.w = c->w_o[l]; p.row_bytes = c->rb_q; p.K = (int) Q; p.N = (int) H;
            if (c->attn) {
                const AttnArgs aa = c->attn_args(l, B(kQkv), (size_t) c->qkv_dim, B(kAttn), (size_t) Q, pos, slots, m0);
                e = launch_attention(aa, mc, attention_splits(mc, (int) d.n_head, c->sms), st, true);
                if (e != cudaSuccess) return e;
                p.pro = kProPlain; p.x = B(kAttn); p.x_stride = (size_t) Q; p.pro_out = nullptr;
            } else {
                p.pro = kProGqa; p.x = B(kQkv) + Q + KV; p.x_stride = (size_t) c->qkv_dim;
                p.head_dim = (int) d.head_dim; p.group = (int) (d.n_head / d.n_kv);
                p.pro_out = B(kAttn); p.pro_out_stride = (size_t) Q;
            }
            p.y = B(kO); p.y_stride = (size_t) H; p.res = h; p.y_res = B(kH1); p.res_stride = (size_t) H;
            e = launch_gemv(p, st, c->sms, true);
            if (e != cudaSuccess) return e;
            // gu = W_gu * Q(rms_norm(h1) * norm_post)
            p.w = c->w_gu[l]; p.row_bytes = c->rb_h; p.K = (int) H; p.N = (int) (2 * I);
            p.pro = kProRmsNorm; p.x = B(kH1); p.x_stride = (size_t) H; p.norm_w = c->layers[l].norm_post;
            p.pro_out = B(kN2); p.pro_out_stride = (size_t) H;
            p.y = B(kGu); p.y_stride = (size_t) (2 * I); p.res = nullptr; p.y_res = nullptr;
            e = launch_gemv(p, st, c->sms, true);
            if (e != cudaSuccess) return e;
            // h = h1 + W_d * Q(silu(g) * u)
            p.w = c->w_d[l]; p.row_bytes = c->rb_i; p.K = (int) I; p.N = (int) H;
            p.pro = kProSwiGlu; p.x = B(kGu); p.x2 = B(kGu) + I; p.x_stride = (size_t) (2 * I);
            p.pro_out = B(kS); p.pro_out_stride = (size_t) I;
            p.y = B(kDown); p.y_stride = (size_t) H; p.res = B(kH1); p.res_stride = (size_t) H;
            p.y_res = last ? h_out + m0 * H : B(kHout);
            e = launch_gemv(p, st, c->sms, true);
            if (e != cudaSuccess) return e;
            h = p.y_res;
        }
        if (io.hidden_out != nullptr) {
            // hidden = rms_norm(h) * norm (written by the prologue), logits = head * Q(hidden)
            GemvParams p = {};
            p.M = mc; p.mode = d.mode; p.eps = d.eps;
            p.w = c->heads[io.head]; p.row_bytes = c->rb_h; p.K = (int) H; p.N = (int) c->vocab;
            p.pro = kProRmsNorm; p.x = h; p.x_stride = (size_t) H; p.norm_w = c->out_norm;
            p.pro_out = io.hidden_out + m0 * H; p.pro_out_stride = (size_t) H;
            p.y = io.logits + m0 * c->vocab; p.y_stride = (size_t) c->vocab;
            const cudaError_t e = launch_gemv(p, st, c->sms, true);
            if (e != cudaSuccess) return e;
        }
    }
    return cudaSuccess;
}

// The step as a CUDA graph, captured once per argument set and replayed
// (the most recently used kMaxGraphs are kept).
constexpr size_t kMaxGraphs = 64;

b200q8_status_t run_graph(b200q8_chain * c, const StepIO & io, b200q8_stream_t stream) {
    cudaError_t     e    = cudaSuccess;
    cudaGraphExec_t exec = nullptr;
    for (size_t i = 0; i < c->graphs.size(); ++i) {
        if (same_io(c->graphs[i].io, io)) {
            exec = c->graphs[i].exec;
            std::rotate(c->graphs.begin() + i, c->graphs.begin() + i + 1, c->graphs.end());  // most recent last
            break;
        }
    }
    if (exec == nullptr) {
        for (int attempt = 0; attempt < 2; ++attempt) {
            cudaGraph_t graph = nullptr;
            exec              = nullptr;
            e                 = cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                cudaError_t e2 = enqueue_step(c, c->cap_stream, io);
                e              = cudaStreamEndCapture(c->cap_stream, &graph);
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
            StepArgs probe;
            if (e == cudaSuccess || attempt > 0 || !c->persistent_in_graph || !persistent_args(c, io, probe)) {
                break;
            }
            // a graph that cannot hold the cooperative launch: capture the per-op form instead
            cudaGetLastError();
            c->persistent_in_graph = false;
        }
        if (e != cudaSuccess) {
            return cuda_error(e, "chain_run: graph capture");
        }
        if (c->graphs.size() >= kMaxGraphs) {
            cudaGraphExecDestroy(c->graphs.front().exec);
            c->graphs.erase(c->graphs.begin());
        }
        c->graphs.push_back({ io, exec });
    }
    e = cudaGraphLaunch(exec, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "chain_run: graph launch");
}

}  // namespace

extern "C" {

b200q8_status_t b200q8_chain_create(const b200q8_chain_desc * desc, int32_t device, b200q8_chain ** out) {
    if (out == nullptr || desc == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_create: null argument");
    }
    *out                = nullptr;
    const b200q8_chain_desc & d = *desc;
    if (d.n_layers < 1 || d.layers == nullptr || d.table == nullptr || d.hidden <= 0 || d.hidden % 256 != 0 ||
        d.inter % 256 != 0 || d.n_head <= 0 || d.n_kv <= 0 || d.n_head % d.n_kv != 0 || d.head_dim <= 0 ||
        (d.n_head * d.head_dim) % 256 != 0 || d.max_m < 1 || d.table_rows < 1 ||
        (d.mode != B200Q8_QUANT_REF && d.mode != B200Q8_QUANT_CPU_X86 && d.mode != B200Q8_QUANT_CPU_ARM)) {
        return set_error(B200Q8_ERR_INVALID_ARG,
                         "chain_create: bad shape (hidden, inter and n_head*head_dim must be multiples of 256)");
    }
    for (int l = 0; l < d.n_layers; ++l) {
        const b200q8_layer & L = d.layers[l];
        if (!L.wq || !L.wk || !L.wv || !L.wo || !L.wgate || !L.wup || !L.wdown || !L.norm_in || !L.norm_post) {
            return set_error(B200Q8_ERR_INVALID_ARG, "chain_create: layer %d has a null pointer", l);
        }
    }
    if (d.attention != nullptr) {
        const b200q8_attention_desc & ad = *d.attention;
        if (!attention_supported((int) d.head_dim, (int) d.n_head, (int) d.n_kv) || ad.n_ctx < 1 ||
            ad.n_ctx > (1 << 30) || ad.n_slots < 1 || ad.n_slots > (1 << 20) || !(ad.rope_theta > 0.0f) ||
            ad.q_norm == nullptr || ad.k_norm == nullptr) {
            return set_error(B200Q8_ERR_INVALID_ARG, "chain_create: bad attention desc (head_dim must be a multiple "
                                                     "of 32 up to 256; n_ctx, n_slots, rope_theta positive)");
        }
        for (int l = 0; l < d.n_layers; ++l) {
            if (ad.q_norm[l] == nullptr || ad.k_norm[l] == nullptr) {
                return set_error(B200Q8_ERR_INVALID_ARG, "chain_create: layer %d has a null q/k norm", l);
            }
        }
    }
    if (d.output != nullptr) {
        const b200q8_output_desc & od = *d.output;
        if (od.norm == nullptr || od.heads == nullptr || od.n_heads < 1 || od.vocab < 16 || od.vocab > (1 << 24)) {
            return set_error(B200Q8_ERR_INVALID_ARG, "chain_create: bad output desc (norm, heads, n_heads >= 1, "
                                                     "vocab in [16, 2^24])");
        }
        for (int i = 0; i < od.n_heads; ++i) {
            if (od.heads[i] == nullptr) {
                return set_error(B200Q8_ERR_INVALID_ARG, "chain_create: output head %d is null", i);
            }
        }
    }
    b200q8_chain * c = new (std::nothrow) b200q8_chain();
    if (c == nullptr) {
        return set_error(B200Q8_ERR_OOM, "chain_create: out of host memory");
    }
    if (d.output != nullptr) {
        c->n_heads  = d.output->n_heads;
        c->out_norm = d.output->norm;
        c->vocab    = d.output->vocab;
        for (int i = 0; i < c->n_heads; ++i) {
            c->heads.push_back(static_cast<const uint8_t *>(d.output->heads[i]));
        }
    }
    if (d.attention != nullptr) {
        c->attn = true;
        c->ad   = *d.attention;
        c->q_norm.assign(d.attention->q_norm, d.attention->q_norm + d.n_layers);
        c->k_norm.assign(d.attention->k_norm, d.attention->k_norm + d.n_layers);
        c->ad.q_norm = nullptr;
        c->ad.k_norm = nullptr;
    }
    c->device = device;
    c->d      = d;
    c->layers.assign(d.layers, d.layers + d.n_layers);
    c->d.layers    = nullptr;
    c->d.attention = nullptr;
    c->d.output    = nullptr;
    int prev    = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        delete c;
        return cuda_error(e, "chain_create: cudaSetDevice");
    }
    c->sms           = current_sm_count();
    const int64_t H  = d.hidden, Q = d.n_head * d.head_dim, KV = d.n_kv * d.head_dim, I = d.inter;
    c->rb_h          = (size_t) (H / kQK) * kBlockBytes;
    c->rb_q          = (size_t) (Q / kQK) * kBlockBytes;
    c->rb_i          = (size_t) (I / kQK) * kBlockBytes;
    c->qkv_dim       = Q + 2 * KV;
    for (int l = 0; l < d.n_layers && e == cudaSuccess; ++l) {
        const b200q8_layer & L = c->layers[l];
        const uint8_t * qkv = contiguous(c, L.wq, (size_t) Q * c->rb_h, L.wk, (size_t) KV * c->rb_h, L.wv,
                                         (size_t) KV * c->rb_h, e);
        const uint8_t * gu  = e == cudaSuccess ? contiguous(c, L.wgate, (size_t) I * c->rb_h, L.wup,
                                                            (size_t) I * c->rb_h, nullptr, 0, e)
                                               : nullptr;
        c->w_qkv.push_back(qkv);
        c->w_gu.push_back(gu);
        c->w_o.push_back(static_cast<const uint8_t *>(L.wo));
        c->w_d.push_back(static_cast<const uint8_t *>(L.wdown));
    }
    // per-layer activation buffers, each [max_m][width]
    const int64_t widths[kNumBufs] = { H, c->qkv_dim, Q, H, H, H, 2 * I, I, H, H };
    size_t        off              = 0;
    for (int i = 0; i < kNumBufs; ++i) {
        c->buf_off[i]    = off;
        c->buf_stride[i] = (size_t) widths[i];
        off += (size_t) (widths[i] * d.max_m + 63) / 64 * 64;
    }
    c->layer_floats = off;
    if (e == cudaSuccess) {
        void * p = nullptr;
        e        = cudaMalloc(&p, (off * d.n_layers + (size_t) (H * d.max_m + 63) / 64 * 64) * sizeof(float));
        if (e == cudaSuccess) {
            c->owned.push_back(p);
            c->act = static_cast<float *>(p);
            c->h0  = c->act + off * d.n_layers;
            e      = cudaMemset(p, 0, (off * d.n_layers + (size_t) H * d.max_m) * sizeof(float));
        }
    }
    if (e == cudaSuccess) {
        e = cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking);
    }
    // default output buffers: [max_m][hidden] twice, [max_m][vocab]
    if (e == cudaSuccess) {
        const size_t hm = (size_t) (H * d.max_m + 63) / 64 * 64;
        const size_t vm = c->n_heads > 0 ? (size_t) (c->vocab * d.max_m + 63) / 64 * 64 : 0;
        void *       p  = nullptr;
        e               = cudaMalloc(&p, (2 * hm + vm) * sizeof(float));
        if (e == cudaSuccess) {
            c->owned.push_back(p);
            c->h_last = static_cast<float *>(p);
            c->hid    = c->h_last + hm;
            c->lg     = vm ? c->hid + hm : nullptr;
            e         = cudaMemset(p, 0, (2 * hm + vm) * sizeof(float));
        }
    }
    bool batched_ok = d.max_m >= kBatchedMinM && d.head_dim % 4 == 0;
    for (int i = 0; i < c->n_heads && batched_ok; ++i) {
        batched_ok = gemm_supported(c->heads[i], c->rb_h, H, c->vocab, d.max_m);
    }
    for (int l = 0; l < d.n_layers && batched_ok; ++l) {
        batched_ok = gemm_supported(c->w_qkv[l], c->rb_h, H, c->qkv_dim, d.max_m) &&
                     gemm_supported(c->w_o[l], c->rb_q, Q, H, d.max_m) &&
                     gemm_supported(c->w_gu[l], c->rb_h, H, 2 * I, d.max_m) &&
                     gemm_supported(c->w_d[l], c->rb_i, I, H, d.max_m);
    }
    if (e == cudaSuccess && batched_ok && std::max(std::max(H, Q), I) <= 8192) {
        void * p = nullptr;
        e        = cudaMalloc(&p, gemm_workspace_bytes(std::max(std::max(H, Q), I), d.max_m));
        if (e == cudaSuccess) {
            c->owned.push_back(p);
            c->planes = p;
        }
        // split-K room for the ops whose row blocks leave SMs idle (o and
        // down: N = hidden); up to 4 splits of any op of this width, for the
        // token chunks of <= 16 that split (the launcher checks the room)
        const size_t part = 4 * (size_t) std::min<int64_t>(d.max_m, 16) * (size_t) std::max(H, Q);
        void *       q    = nullptr;
        if (e == cudaSuccess) e = cudaMalloc(&q, part * sizeof(float) + (size_t) c->sms * sizeof(unsigned));
        if (e == cudaSuccess) {
            c->owned.push_back(q);
            e = cudaMemset(q, 0, part * sizeof(float) + (size_t) c->sms * sizeof(unsigned));
            c->split = { static_cast<float *>(q), part, reinterpret_cast<unsigned *>(static_cast<float *>(q) + part),
                         (size_t) c->sms };
        }
    }
    if (e == cudaSuccess && c->attn) {
        const size_t kv_floats = 2 * (size_t) d.n_layers * c->ad.n_slots * c->ad.n_ctx * KV;
        void *       p1 = nullptr, *p2 = nullptr, *p3 = nullptr, *p4 = nullptr;
        e = cudaMalloc(&p1, kv_floats * sizeof(float));
        if (e == cudaSuccess) { c->owned.push_back(p1); e = cudaMemset(p1, 0, kv_floats * sizeof(float)); }
        if (e == cudaSuccess) e = cudaMalloc(&p2, sizeof(float) * (size_t) d.max_m * Q);
        if (e == cudaSuccess) {
            c->owned.push_back(p2);
            e = cudaMalloc(&p3, sizeof(float) * (size_t) d.max_m * d.n_head * kAttnMaxSplits * (d.head_dim + 2));
        }
        if (e == cudaSuccess) { c->owned.push_back(p3); e = cudaMalloc(&p4, sizeof(unsigned) * (size_t) d.max_m * d.n_head); }
        if (e == cudaSuccess) { c->owned.push_back(p4); e = cudaMemset(p4, 0, sizeof(unsigned) * (size_t) d.max_m * d.n_head); }
        if (e == cudaSuccess) {
            c->kv_cache     = static_cast<float *>(p1);
            c->q_rot        = static_cast<float *>(p2);
            c->attn_partial = static_cast<float *>(p3);
            c->attn_count   = static_cast<unsigned *>(p4);
        }
    }
    // persistent step (M <= 2): per-layer weight table, LL hand-off words,
    // sync words
    const char * per_op = getenv("B200Q8_CHAIN_PER_OP");
    if (e == cudaSuccess && !(per_op && per_op[0] == '1')) {
        std::vector<StepLayerDev> host_layers(d.n_layers);
        for (int l = 0; l < d.n_layers; ++l) {
            host_layers[l] = { c->w_qkv[l], c->w_o[l], c->w_gu[l], c->w_gu[l] + (size_t) I * c->rb_h, c->w_d[l],
                               c->layers[l].norm_in, c->layers[l].norm_post,
                               c->attn ? c->q_norm[l] : nullptr, c->attn ? c->k_norm[l] : nullptr };
        }
        // hand-off words for the persistent step's 2 tokens
        c->ll_m      = 2;
        c->ll_layer  = (size_t) c->ll_m * (c->qkv_dim + Q + H + I + H);
        void * p1 = nullptr, * p2 = nullptr, * p3 = nullptr;
        e = cudaMalloc(&p1, sizeof(StepLayerDev) * d.n_layers);
        if (e == cudaSuccess) { c->owned.push_back(p1); e = cudaMalloc(&p2, sizeof(unsigned long long) * c->ll_layer * d.n_layers); }
        if (e == cudaSuccess) { c->owned.push_back(p2); e = cudaMalloc(&p3, 64); }
        if (e == cudaSuccess) {
            c->owned.push_back(p3);
            c->step_layers = static_cast<StepLayerDev *>(p1);
            c->ll          = static_cast<unsigned long long *>(p2);
            c->sync        = static_cast<unsigned *>(p3);
            e = cudaMemcpy(p1, host_layers.data(), sizeof(StepLayerDev) * d.n_layers, cudaMemcpyHostToDevice);
        }
        if (e == cudaSuccess) e = cudaMemset(p2, 0, sizeof(unsigned long long) * c->ll_layer * d.n_layers);
        if (e == cudaSuccess) e = cudaMemset(p3, 0, 64);
        StepArgs probe = {};
        probe.H = (int) H; probe.Q = (int) (d.n_head * d.head_dim); probe.KV = (int) KV; probe.I = (int) I;
        probe.mode = d.mode; probe.attn = c->attn ? 1 : 0; probe.head_dim = (int) d.head_dim;
        probe.ll_m = c->ll_m;
        c->persistent_max_m = e == cudaSuccess ? std::min(decode_step_max_m(probe), c->ll_m) : 0;
        c->persistent       = c->persistent_max_m > 0;
#ifdef B200Q8_TIMELINE
        // analysis builds: the stamp buffer exists before any graph capture
        if (e == cudaSuccess && cudaMalloc(&c->timeline, sizeof(unsigned long long) * 8 * 4 * d.n_layers * c->sms) ==
                                    cudaSuccess) {
            c->owned.push_back(c->timeline);
            cudaMemset(c->timeline, 0, sizeof(unsigned long long) * 8 * 4 * d.n_layers * c->sms);
        }
#endif
    }
    for (int l = 0; l < d.n_layers && e == cudaSuccess; ++l) {
        GemvParams p = {};
        p.w = c->w_qkv[l]; p.row_bytes = c->rb_h; p.K = (int) H; p.N = (int) c->qkv_dim; p.M = 8;
        bool ok = gemv_supported(p);
        p.w = c->w_gu[l]; p.N = (int) (2 * I); ok = ok && gemv_supported(p);
        p.w = c->w_o[l]; p.row_bytes = c->rb_q; p.K = (int) Q; p.N = (int) H; ok = ok && gemv_supported(p);
        p.w = c->w_d[l]; p.row_bytes = c->rb_i; p.K = (int) I; ok = ok && gemv_supported(p);
        for (int i = 0; i < c->n_heads && l == 0; ++i) {
            p.w = c->heads[i]; p.row_bytes = c->rb_h; p.K = (int) H; p.N = (int) c->vocab;
            ok = ok && gemv_supported(p);
        }
        if (!ok) {
            cudaSetDevice(prev);
            chain_free(c);
            return set_error(B200Q8_ERR_UNSUPPORTED, "chain_create: layer %d weights are not 16-byte aligned "
                                                     "or too wide for the streaming GEMV", l);
        }
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        chain_free(c);
        return cuda_error(e, "chain_create");
    }
    *out = c;
    return B200Q8_OK;
}

b200q8_status_t b200q8_chain_run(b200q8_chain * c, const int32_t * ids, const float * x_in, float * h_out, int64_t M,
                                 b200q8_stream_t stream) {
    if (c == nullptr || ids == nullptr || x_in == nullptr || h_out == nullptr || M < 1 || M > c->d.max_m) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_run: bad argument (M must be in [1, max_m])");
    }
    if (c->attn) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_run: this chain has attention; use chain_run_at");
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) {
        return cuda_error(e, "chain_run: cudaSetDevice");
    }
    StepIO io;
    io.M = M; io.ids = ids; io.x_in = x_in; io.h_out = h_out;
    io.table = static_cast<const uint8_t *>(c->d.table); io.table_rows = c->d.table_rows;
    StepArgs a;
    if (persistent_args(c, io, a)) {
        e = launch_decode_step(a, c->sms, reinterpret_cast<cudaStream_t>(stream));
        cudaSetDevice(prev);
        return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "chain_run: persistent step launch");
    }
    const b200q8_status_t st = run_graph(c, io, stream);
    cudaSetDevice(prev);
    return st;
}

b200q8_status_t b200q8_chain_run_at(b200q8_chain * c, const int32_t * ids, const float * x_in, const int32_t * pos,
                                    const int32_t * slots, float * h_out, int64_t M, b200q8_stream_t stream) {
    if (c == nullptr || ids == nullptr || x_in == nullptr || pos == nullptr || h_out == nullptr || M < 1 ||
        M > c->d.max_m) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_run_at: bad argument (M must be in [1, max_m])");
    }
    if (!c->attn) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_run_at: the chain was built without an attention desc");
    }
    if (slots == nullptr && M > c->ad.n_slots) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_run_at: M (%lld) tokens need explicit slots beyond n_slots",
                         (long long) M);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) {
        return cuda_error(e, "chain_run_at: cudaSetDevice");
    }
    StepIO io;
    io.M = M; io.ids = ids; io.x_in = x_in; io.pos = pos; io.slots = slots; io.h_out = h_out;
    io.table = static_cast<const uint8_t *>(c->d.table); io.table_rows = c->d.table_rows;
    const b200q8_status_t st = run_graph(c, io, stream);
    cudaSetDevice(prev);
    return st;
}

b200q8_status_t b200q8_chain_step(b200q8_chain * c, const b200q8_step_args * a, b200q8_stream_t stream) {
    if (c == nullptr || a == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: null argument");
    }
    StepIO                io;
    const b200q8_status_t v = chain_resolve(c, *a, io);
    if (v != B200Q8_OK) {
        return v;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) {
        return cuda_error(e, "chain_step: cudaSetDevice");
    }
    const b200q8_status_t st = run_graph(c, io, stream);
    cudaSetDevice(prev);
    return st;
}

b200q8_status_t b200q8_chain_buffer(b200q8_chain * c, int32_t layer, int32_t which, float ** ptr, int64_t * stride) {
    if (c == nullptr || ptr == nullptr || layer < 0 || layer >= c->d.n_layers || which < 0 || which >= kNumBufs) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_buffer: bad layer or buffer index");
    }
    *ptr = c->buf(layer, which);
    if (stride) {
        *stride = (int64_t) c->buf_stride[which];
    }
    return B200Q8_OK;
}

#ifdef B200Q8_TIMELINE
// Analysis builds only: copies the last persistent step's stamps
// [cta][op][8] (events 0-4 consumer, 5 producer first issue) to the host.
b200q8_status_t b200q8_chain_timeline(b200q8_chain * c, unsigned long long * host, size_t n) {
    if (c == nullptr || c->timeline == nullptr) {
        return B200Q8_ERR_INVALID_ARG;
    }
    const size_t have = (size_t) 8 * 4 * c->d.n_layers * c->sms;
    cudaDeviceSynchronize();
    return cudaMemcpy(host, c->timeline, sizeof(unsigned long long) * std::min(n, have), cudaMemcpyDeviceToHost) ==
                   cudaSuccess
               ? B200Q8_OK
               : B200Q8_ERR_BACKEND;
}
#endif

b200q8_status_t b200q8_chain_inject_epoch_skew(b200q8_chain * c, int32_t skew) {
    if (c == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_inject_epoch_skew: null chain");
    }
    if (!c->persistent || c->sync == nullptr) {
        return set_error(B200Q8_ERR_UNSUPPORTED, "chain_inject_epoch_skew: the chain has no persistent step");
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(c->device);
    unsigned    counter = 0;
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&counter, c->sync, sizeof(unsigned), cudaMemcpyDeviceToHost);
    if (skew != 0) {
        counter += (unsigned) skew;
    } else {
        // realign to the CTA count and skip one epoch, so no LL word written
        // by a skewed run can be taken as current by the next one
        const unsigned g = (unsigned) c->sms;
        counter          = (counter + g - 1) / g * g + g;
    }
    if (e == cudaSuccess) e = cudaMemcpy(c->sync, &counter, sizeof(unsigned), cudaMemcpyHostToDevice);
    cudaSetDevice(prev);
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "chain_inject_epoch_skew");
}

void b200q8_chain_destroy(b200q8_chain * c) {
    chain_free(c);
}

}  // extern "C"

namespace b200q8 {

ChainInfo chain_info(const b200q8_chain * c) {
    ChainInfo i  = {};
    i.device     = c->device;
    i.sms        = c->sms;
    i.hidden     = c->d.hidden;
    i.max_m      = c->d.max_m;
    i.attn       = c->attn;
    i.n_ctx      = c->attn ? c->ad.n_ctx : 0;
    i.n_slots    = c->attn ? c->ad.n_slots : 0;
    i.n_heads    = c->n_heads;
    i.vocab      = c->vocab;
    i.table      = static_cast<const uint8_t *>(c->d.table);
    i.table_rows = c->d.table_rows;
    return i;
}

int chain_mode(const b200q8_chain * c) {
    return c->d.mode;
}

b200q8_status_t chain_resolve(b200q8_chain * c, const b200q8_step_args & a, StepIO & io) {
    if (a.M < 1 || a.M > c->d.max_m) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: M (%lld) must be in [1, max_m]", (long long) a.M);
    }
    if (a.ids == nullptr && a.x_in == nullptr) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: needs ids, x_in or both");
    }
    if (a.ids != nullptr && a.table != nullptr && a.table_rows < 1) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: a table needs table_rows >= 1");
    }
    if (a.table != nullptr && reinterpret_cast<uintptr_t>(a.table) % 2 != 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: table must be 2-byte aligned");
    }
    if (c->attn != (a.pos != nullptr)) {
        return set_error(B200Q8_ERR_INVALID_ARG, c->attn ? "chain_step: this chain has attention and needs pos"
                                                         : "chain_step: pos given to a chain without attention");
    }
    if (c->attn && a.slots == nullptr && a.M > c->ad.n_slots) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: M (%lld) tokens need explicit slots beyond n_slots",
                         (long long) a.M);
    }
    const bool out = a.hidden_out != nullptr || a.logits != nullptr;
    if (out && c->n_heads == 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: the chain was built without an output desc");
    }
    if (out && (a.head < 0 || a.head >= c->n_heads)) {
        return set_error(B200Q8_ERR_INVALID_ARG, "chain_step: head %d outside [0, %d)", a.head, c->n_heads);
    }
    io            = StepIO();
    io.M          = a.M;
    io.ids        = a.ids;
    io.table      = a.ids == nullptr ? nullptr
                    : a.table != nullptr ? static_cast<const uint8_t *>(a.table)
                                         : static_cast<const uint8_t *>(c->d.table);
    io.table_rows = a.ids == nullptr ? 0 : a.table != nullptr ? a.table_rows : c->d.table_rows;
    io.x_in       = a.x_in;
    io.pos        = a.pos;
    io.slots      = a.slots;
    io.h_out      = a.h_out != nullptr ? a.h_out : c->h_last;
    if (out) {
        io.hidden_out = a.hidden_out != nullptr ? a.hidden_out : c->hid;
        io.logits     = a.logits != nullptr ? a.logits : c->lg;
        io.head       = a.head;
    }
    return B200Q8_OK;
}

cudaError_t chain_enqueue(b200q8_chain * c, cudaStream_t st, const StepIO & io) {
    return enqueue_step(c, st, io);
}

bool chain_persistent_in_graph(b200q8_chain * c, bool disable) {
    const bool was = c->persistent && c->persistent_in_graph;
    if (disable) {
        c->persistent_in_graph = false;
    }
    return was;
}

}  // namespace b200q8
