// attention.cu -- the reference's attention in the talker step
// (src/arch/qwen3-tts/operations.cpp:86-135) for one new position per token:
//
//   q, k heads:  RMS norm over head_dim (q_norm / k_norm weights), then NEOX
//                RoPE at the token's position;
//   cache:       k and v written to the token's slot at that position (F32);
//   attention:   softmax(q . K / sqrt(head_dim)) over cached positions
//                0..pos, times V; query head h reads kv head h / (n_head / n_kv).
//
// The rotation angle follows ggml's RoPE recurrence: theta_0 = pos,
// theta_{i+1} = theta_i * base^(-2/head_dim) in fp32, cos/sin of each; NEOX
// pairs element i with i + head_dim/2.  Attention runs split over positions
// (online softmax per warp, fixed-order merge of the warps, then of the
// splits by the last CTA of each (token, head) to finish; the split count
// follows the token's position): deterministic.
// Scores, softmax and the V sum are fp32 -- ggml-cpu's are fp32 in its own
// SIMD order -- so parity with the oracle is to a tolerance.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace b200q8 {
namespace {

constexpr int kAttnThreads  = 256;  // 8 warps
constexpr int kPosPerSplit = 64;   // fewest cached positions a split CTA takes
constexpr int kAttnWarps   = kAttnThreads / 32;
constexpr int kMaxHeadDim  = 256;

// One block per (head, token); thread d holds element d of the head.
// blockIdx.x: [0, n_head) q heads, [n_head, n_head + n_kv) k heads,
// [n_head + n_kv, n_head + 2 n_kv) v heads.
__global__ void __launch_bounds__(kMaxHeadDim) qk_rope_cache_kernel(const AttnArgs a) {
    __shared__ float  y[kMaxHeadDim];
    __shared__ double part[kMaxHeadDim / 32];
    pdl_launch_dependents();
    pdl_wait_primary();
    const int m    = blockIdx.y;
    const int hb   = blockIdx.x;
    const int d    = threadIdx.x;
    const int hd   = a.head_dim;
    const int pos  = a.pos[m];
    const int slot = a.slots ? a.slots[m] : a.slot_base + m;
    if (pos < 0 || pos >= a.n_ctx || slot < 0 || slot >= a.n_slots) {
        if (d == 0 && hb == 0) {
            record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
        }
        return;
    }
    const int     kinds = hb < a.n_head ? 0 : (hb < a.n_head + a.n_kv ? 1 : 2);
    const int     h     = kinds == 0 ? hb : (kinds == 1 ? hb - a.n_head : hb - a.n_head - a.n_kv);
    const float * src   = a.qkv + (size_t) m * a.qkv_stride +
                        (kinds == 0 ? 0 : (kinds == 1 ? a.n_head * hd : (a.n_head + a.n_kv) * hd)) + h * hd;
    float x = src[d];
    if (kinds < 2) {
        // RMS norm over the head: fp64 sum of fp32 squares, as ggml's rms_norm
        double ss = (double) __fmul_rn(x, x);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, off);
        }
        if ((d & 31) == 0) {
            part[d >> 5] = ss;
        }
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < (hd >> 5); ++w) {
            tot += part[w];
        }
        const float mean  = (float) (tot / (double) hd);
        const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, a.eps)));
        const float w     = (kinds == 0 ? a.q_norm : a.k_norm)[d];
        y[d]              = __fmul_rn(__fmul_rn(x, scale), w);
        __syncthreads();
        // NEOX RoPE: thread i < hd/2 rotates the pair (i, i + hd/2)
        const int half = hd >> 1;
        if (d < half) {
            const float ts    = powf(a.rope_theta, __fdiv_rn(-2.0f, (float) hd));
            float       theta = (float) pos;
            for (int i = 0; i < d; ++i) {
                theta = __fmul_rn(theta, ts);
            }
            const float c  = cosf(theta);
            const float sn = sinf(theta);
            const float x0 = y[d];
            const float x1 = y[d + half];
            const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            const float r1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
            if (kinds == 0) {
                float * q = a.q_rot + (size_t) m * a.n_head * hd + h * hd;
                q[d]        = r0;
                q[d + half] = r1;
            } else {
                float * kc = a.k_cache + (((size_t) slot * a.n_ctx + pos) * a.n_kv + h) * hd;
                kc[d]        = r0;
                kc[d + half] = r1;
            }
        }
    } else {
        a.v_cache[(((size_t) slot * a.n_ctx + pos) * a.n_kv + h) * hd + d] = x;
    }
}

// One CTA per (head, token, split).  A token at position pos attends over
// npos = pos + 1 cached positions, split into ns_eff = ceil(npos /
// kPosPerSplit) parts (at most the launch's gridDim.z); CTAs beyond ns_eff
// leave at once, so short prefixes cost one CTA per head.  Each warp keeps an
// online softmax (running max, sum and weighted V) over its positions; lanes
// hold head_dim/32 elements.  The warps merge in a fixed order; with several
// splits, the last split CTA of a (token, head) to finish merges the splits'
// partials in split order.  ns_eff depends only on pos, so the result is
// deterministic.
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
    __shared__ float sq[kMaxHeadDim];
    __shared__ float wm[kAttnWarps], wl[kAttnWarps];
    __shared__ float wo[kAttnWarps][kMaxHeadDim];
    __shared__ float sw[kAttnMaxSplits];
    __shared__ float sL;
    __shared__ int   last;
    pdl_launch_dependents();
    pdl_wait_primary();
    const int h     = blockIdx.x;
    const int m     = blockIdx.y;
    const int split = blockIdx.z;
    const int hd    = a.head_dim;
    const int warp  = threadIdx.x >> 5;
    const int lane  = threadIdx.x & 31;
    const int pos   = a.pos[m];
    const int slot  = a.slots ? a.slots[m] : a.slot_base + m;
    const bool ok   = pos >= 0 && pos < a.n_ctx && slot >= 0 && slot < a.n_slots;
    const int npos  = ok ? pos + 1 : 0;
    const int ns    = max(1, min((int) gridDim.z, (npos + kPosPerSplit - 1) / kPosPerSplit));
    if (split >= ns) {
        return;
    }
    const int per = (npos + ns - 1) / ns;
    const int j0  = min(npos, split * per);
    const int j1  = min(npos, j0 + per);
    const int kvh = h / (a.n_head / a.n_kv);
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        sq[d] = ok ? a.q_rot[(size_t) m * a.n_head * hd + h * hd + d] : 0.0f;
    }
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, sqrtf((float) hd));
    const int   E     = hd >> 5;  // elements per lane (head_dim % 32 == 0)
    float       mx = -INFINITY, l = 0.0f;
    float       o[kMaxHeadDim / 32];
#pragma unroll
    for (int e = 0; e < kMaxHeadDim / 32; ++e) {
        o[e] = 0.0f;
    }
    const size_t  row = (size_t) a.n_kv * hd;
    const float * kb  = a.k_cache + ((size_t) slot * a.n_ctx) * row + (size_t) kvh * hd;
    const float * vb  = a.v_cache + ((size_t) slot * a.n_ctx) * row + (size_t) kvh * hd;
    for (int j = j0 + warp; j < j1; j += kAttnWarps) {
        const float * kj = kb + (size_t) j * row;
        const float * vj = vb + (size_t) j * row;
        float         kv[kMaxHeadDim / 32], vv[kMaxHeadDim / 32];
#pragma unroll
        for (int e = 0; e < kMaxHeadDim / 32; ++e) {
            if (e < E) {
                kv[e] = kj[lane + 32 * e];
                vv[e] = vj[lane + 32 * e];
            }
        }
        float dot = 0.0f;
#pragma unroll
        for (int e = 0; e < kMaxHeadDim / 32; ++e) {
            if (e < E) {
                dot = __fmaf_rn(sq[lane + 32 * e], kv[e], dot);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            dot += __shfl_xor_sync(0xffffffffu, dot, off);
        }
        const float s  = __fmul_rn(dot, scale);
        const float nm = fmaxf(mx, s);
        const float f  = expf(mx - nm);  // 0 on the first position (mx = -inf)
        const float p  = expf(s - nm);
        l              = __fmaf_rn(l, f, p);
#pragma unroll
        for (int e = 0; e < kMaxHeadDim / 32; ++e) {
            if (e < E) {
                o[e] = __fmaf_rn(o[e], f, __fmul_rn(p, vv[e]));
            }
        }
        mx = nm;
    }
    // merge the warps in a fixed order
    if (lane == 0) {
        wm[warp] = mx;
        wl[warp] = l;
    }
#pragma unroll
    for (int e = 0; e < kMaxHeadDim / 32; ++e) {
        if (e < E) {
            wo[warp][lane + 32 * e] = o[e];
        }
    }
    __syncthreads();
    float M_ = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) {
        M_ = fmaxf(M_, wm[w]);
    }
    if (threadIdx.x < kAttnWarps) {
        sw[threadIdx.x] = wm[threadIdx.x] != -INFINITY ? expf(wm[threadIdx.x] - M_) : 0.0f;
    }
    __syncthreads();
    float L = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w) {
        L = __fmaf_rn(wl[w], sw[w], L);
    }
    if (ns == 1) {
        for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
            float acc = 0.0f;
            for (int w = 0; w < kAttnWarps; ++w) {
                acc = __fmaf_rn(wo[w][d], sw[w], acc);
            }
            a.out[(size_t) m * a.out_stride + h * hd + d] = ok ? __fdiv_rn(acc, L) : 0.0f;
        }
        return;
    }
    float * part = a.partial + (((size_t) m * a.n_head + h) * kAttnMaxSplits + split) * (hd + 2);
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        float acc = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            acc = __fmaf_rn(wo[w][d], sw[w], acc);
        }
        part[d] = acc;
    }
    if (threadIdx.x == 0) {
        part[hd]     = M_;
        part[hd + 1] = L;
    }
    // the last split of this (token, head) to finish merges all splits in order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *     cnt  = a.counters + (size_t) m * a.n_head + h;
        const unsigned prev = atomicAdd(cnt, 1u);
        last                = prev == (unsigned) ns - 1;
        if (last) {
            *cnt = 0;  // ready for the next launch
        }
    }
    __syncthreads();
    if (!last) {
        return;
    }
    __threadfence();
    const float * base = a.partial + ((size_t) m * a.n_head + h) * kAttnMaxSplits * (hd + 2);
    if (threadIdx.x < ns) {
        sw[threadIdx.x] = __ldcg(base + threadIdx.x * (hd + 2) + hd);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float mx2 = -INFINITY;
        for (int s = 0; s < ns; ++s) {
            mx2 = fmaxf(mx2, sw[s]);
        }
        float L2 = 0.0f;
        for (int s = 0; s < ns; ++s) {
            const float ws = sw[s] != -INFINITY ? expf(sw[s] - mx2) : 0.0f;
            L2             = __fmaf_rn(__ldcg(base + s * (hd + 2) + hd + 1), ws, L2);
            sw[s]          = ws;
        }
        sL = L2;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        float acc = 0.0f;
        for (int s = 0; s < ns; ++s) {
            acc = __fmaf_rn(__ldcg(base + s * (hd + 2) + d), sw[s], acc);
        }
        a.out[(size_t) m * a.out_stride + h * hd + d] = ok ? __fdiv_rn(acc, sL) : 0.0f;
    }
}

template <typename F, typename... Args>
cudaError_t launch_attn(F fn, dim3 grid, dim3 block, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = grid;
    cfg.blockDim           = block;
    cfg.stream             = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs                                          = attr;
        cfg.numAttrs                                       = 1;
    }
    return cudaLaunchKernelEx(&cfg, fn, args...);
}

}  // namespace

bool attention_supported(int head_dim, int n_head, int n_kv) {
    return head_dim >= 32 && head_dim <= kMaxHeadDim && head_dim % 32 == 0 && n_kv > 0 && n_head % n_kv == 0;
}

int attention_splits(int64_t M, int n_head, int sm_count) {
    const int64_t heads = M * n_head;
    const int64_t want  = (4 * (int64_t) sm_count + heads - 1) / heads;
    return (int) std::max<int64_t>(1, std::min<int64_t>(kAttnMaxSplits, want));
}

cudaError_t launch_attention(const AttnArgs & a, int64_t M, int splits, cudaStream_t stream, bool pdl) {
    cudaError_t e = launch_attn(qk_rope_cache_kernel, dim3((unsigned) (a.n_head + 2 * a.n_kv), (unsigned) M),
                                dim3((unsigned) a.head_dim), stream, pdl, a);
    if (e != cudaSuccess) {
        return e;
    }
    return launch_attn(attn_decode_kernel, dim3((unsigned) a.n_head, (unsigned) M, (unsigned) splits),
                       dim3(kAttnThreads), stream, pdl, a);
}

}  // namespace b200q8
