// decode_step.cu -- the whole talker-shaped decode step as ONE persistent
// kernel launch (sm_100a), for M <= 2 tokens.
//
// Why: at M = 1 the step is 4 * n_layers dependent MUL_MATs of 1-7 MB each.
// Launched one by one (the reference's GraphRun per step, or a CUDA graph of
// per-op kernels) every op pays a launch, a DRAM round trip for its first
// weights and a grid-wide drain; the HBM pipe idles most of the step.  Here:
//
//  * one CTA per SM, co-resident (cooperative launch), each owning a fixed,
//    balanced slice of the rows of every op in the step;
//  * a producer warp streams the CTA's weight slices for the WHOLE step, op
//    after op, through a ring of shared-memory slots with 1-D bulk copies
//    (never multicast), so weights for later ops arrive while earlier ops
//    still wait on their inputs -- HBM stays busy across op boundaries;
//  * ops hand activations to each other through "LL" words in global memory:
//    each output value is stored as one 8-byte word {fp32 value, epoch}, a
//    single-copy-atomic store; consumers poll the words they need until the
//    epoch is the current launch's, so no grid barrier and no separate flag
//    round trip is needed (the epoch comes from a device-side launch counter,
//    so the kernel can be replayed without host bookkeeping);
//  * every CTA keeps the residual stream h in shared memory and applies the
//    residual adds, RMS norms, GQA expansion and SwiGLU to the full vectors
//    itself, then quantizes them bit-exactly (Q8_0, the reference quantizer)
//    into shared memory -- the same arithmetic as the per-op path;
//  * each wait is bounded (about a second); a timeout records
//    B200Q8_ERR_DEVICE_TIMEOUT, raises a global abort word the other CTAs
//    poll, and the producer drains its in-flight copies before exiting.
//
// Dataflow per layer (outputs published as LL words):
//   qkv  = W_qkv * Q(rms_norm(h) * norm_in)           -> v published
//   o    = W_o   * Q(attend(v))                        -> o published
//   h1   = h + o (every CTA, locally)
//   g|u  = W_gate|W_up * Q(rms_norm(h1) * norm_post)   -> s = silu(g)*u published
//   d    = W_down * Q(s)                               -> d published
//   h    = h1 + d (every CTA, locally, at the next layer's start)
#include "common.cuh"
#include "kernels.h"
#include "tile_dot.cuh"

#include <algorithm>

namespace b200q8 {

namespace {

constexpr int kStepConsumerWarps = 16;
constexpr int kStepConsumers     = kStepConsumerWarps * 32;
constexpr int kStepThreads       = kStepConsumers + 32;
constexpr int kStepSlotBytes     = 16384;
constexpr int kStepMaxSlots      = 16;
constexpr int kStepYMax          = 64;  // rows one CTA produces in one op (per token)
constexpr int kStepHeader        = 2048;

__device__ __forceinline__ unsigned long long ld_ll(const unsigned long long * p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_ll(unsigned long long * p, float v, unsigned epoch) {
    const unsigned long long w = ((unsigned long long) epoch << 32) | (unsigned long long) __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// Named barrier over the consumer threads that also ORs a predicate across
// them, so every consumer takes the same stop decision.
__device__ __forceinline__ bool consumers_any(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.cta.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t) pred), "r"(kStepConsumers)
        : "memory");
    return r != 0;
}

#ifdef B200Q8_TIMELINE
// Analysis builds only: per (CTA, op, event) globaltimer stamps.
__device__ __forceinline__ void tl_stamp(const StepArgs & a, int op, int ev) {
    if (threadIdx.x == 0 && a.timeline != nullptr) {
        unsigned long long g;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g));
        a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + op) * 8 + ev] = g;
    }
}
#define TL(op, ev) tl_stamp(a, (op), (ev))
#define TL_CYC(op)                                                                                      \
    do {                                                                                                \
        if (threadIdx.x == 0 && a.timeline != nullptr) {                                                \
            a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + (op)) * 8 + 6] = tl_wait_cycles;        \
            a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + (op)) * 8 + 7] = tl_dot_cycles;         \
        }                                                                                               \
    } while (0)
#else
#define TL(op, ev) ((void) 0)
#define TL_CYC(op) ((void) 0)
#endif

struct Part {
    int r0;
    int n;
};

__device__ __forceinline__ Part part(int N, int G, int c) {
    const int base = N / G;
    const int rem  = N % G;
    return { c * base + min(c, rem), base + (c < rem ? 1 : 0) };
}

struct Seg {
    const uint8_t * base;  // first row of this CTA's slice
    size_t          rb;    // bytes per row
    int             n;     // rows
    int             sr;    // rows per tile
};

__device__ __forceinline__ int seg_tiles(const Seg & s) {
    return s.n > 0 ? (s.n + s.sr - 1) / s.sr : 0;
}

struct Smem {
    uint64_t * full;
    uint64_t * empty;
    unsigned * epoch;
    int *      abort_local;
    double *   rms_part;   // [kStepConsumerWarps][2]
    float *    rms_scale;  // [2]
    float *    hbuf;       // [M_T][H]
    float *    h1buf;      // [M_T][H]
    float *    normbuf;    // [H] the RMS-norm weight of the current norm op
    float *    ybuf;       // [M_T][2*kStepYMax]
    uint8_t *  xc;         // codes [M_T][Kmax]
    float *    xd;         // scales [M_T][Kmax/32]
    uint8_t *  ring;
};

// The 5 weight segments of layer l for CTA c, in streaming order:
// qkv, o, gate, up, down.
__device__ __forceinline__ void layer_segs(const StepArgs & a, int l, int c, int G, Seg (&segs)[5]) {
    const StepLayerDev & L   = a.layers[l];
    const int            qkv = a.Q + 2 * a.KV;
    const Part           pq  = part(qkv, G, c);
    const Part           po  = part(a.H, G, c);
    const Part           pg  = part(a.I, G, c);
    const Part           pd  = part(a.H, G, c);
    const int            sr_h = max(1, (int) (kStepSlotBytes / a.rb_h));
    const int            sr_q = max(1, (int) (kStepSlotBytes / a.rb_q));
    const int            sr_i = max(1, (int) (kStepSlotBytes / a.rb_i));
    segs[0] = { L.w_qkv + (size_t) pq.r0 * a.rb_h, a.rb_h, pq.n, sr_h };
    segs[1] = { L.w_o + (size_t) po.r0 * a.rb_q, a.rb_q, po.n, sr_q };
    segs[2] = { L.w_gate + (size_t) pg.r0 * a.rb_h, a.rb_h, pg.n, sr_h };
    segs[3] = { L.w_up + (size_t) pg.r0 * a.rb_h, a.rb_h, pg.n, sr_h };
    segs[4] = { L.w_down + (size_t) pd.r0 * a.rb_i, a.rb_i, pd.n, sr_i };
}

__device__ __forceinline__ bool aborted(const StepArgs & a, const Smem & s) {
    return *(volatile int *) s.abort_local != 0 || *(volatile unsigned *) &a.sync[1] != 0;
}

__device__ void raise_abort(const StepArgs & a, const Smem & s) {
    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
    *(volatile int *) s.abort_local = 1;
    atomicExch(&a.sync[1], 1u);
}

// Reads n LL words (this thread's share, already loaded in w[]) until all
// carry `epoch`.  Returns false on timeout/abort.
template <int N>
__device__ __forceinline__ bool ll_settle(const StepArgs & a, const Smem & s, const unsigned long long * const (&src)[N],
                                          unsigned long long (&w)[N], int n, unsigned epoch) {
    long long start = -1;
    for (unsigned iter = 0;; ++iter) {
        bool done = true;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if (i < n && (unsigned) (w[i] >> 32) != epoch) {
                w[i] = ld_ll(src[i]);
                done = false;
            }
        }
        if (done) {
            return true;
        }
        if (start < 0) {
            start = clock64();
        } else if (clock64() - start > kWaitLimitCycles) {
            return false;
        } else if ((iter & 255u) == 255u && aborted(a, s)) {
            // the global abort word costs an L2 round trip: look rarely
            return false;
        }
    }
}

// Phase A of a norm stage: h_dst[m][i] = h_src[m][i] + published delta[m][i]
// for all i < H (delta read as LL words; delta == nullptr: h_dst already
// holds the values), accumulating sum of squares per token.  Then the
// per-token RMS scale.  Leaves the result in s.rms_scale.
template <int M_T>
__device__ void residual_and_rms(const StepArgs & a, const Smem & s, const unsigned long long * delta,
                                 const float * h_src, float * h_dst, int M, unsigned epoch, float * trace_h,
                                 const float * norm, bool & fail) {
    const int H = a.H;
    const int t = threadIdx.x;
    // The norm weight goes to shared memory now, its L2 latency hidden under
    // the wait for the previous op's outputs.
    for (int i = t; i < H; i += kStepConsumers) {
        s.normbuf[i] = norm[i];
    }
    double    ss[M_T];
#pragma unroll
    for (int m = 0; m < M_T; ++m) {
        ss[m] = 0.0;
    }
    constexpr int kPer = 4;  // elements per thread per pass (H <= 4 * 512 * passes)
    for (int base = 0; base < M * H; base += kStepConsumers * kPer) {
        const unsigned long long * src[kPer];
        unsigned long long         w[kPer];
        int                        n = 0;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = base + i * kStepConsumers + t;
            src[i]      = delta != nullptr ? delta + (e < M * H ? e : 0) : nullptr;
            w[i]        = 0;
            if (e < M * H) {
                n = i + 1;
            }
        }
        if (delta != nullptr) {
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                if (i < n) {
                    w[i] = ld_ll(src[i]);
                }
            }
            if (!fail && !ll_settle<kPer>(a, s, src, w, n, epoch)) {
                fail = true;
            }
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = base + i * kStepConsumers + t;
            if (e < M * H) {
                const int m = e / H;
                float     v;
                if (delta != nullptr) {
                    v = __fadd_rn(h_src[e], __uint_as_float((unsigned) (w[i] & 0xffffffffu)));
                    h_dst[e] = v;
                    if (trace_h != nullptr) {
                        trace_h[e] = v;
                    }
                } else {
                    v = h_dst[e];
                }
#pragma unroll
                for (int mm = 0; mm < M_T; ++mm) {
                    if (mm == m) {
                        ss[mm] += (double) __fmul_rn(v, v);
                    }
                }
            }
        }
    }
    const int warp = t / 32;
    const int lane = t % 32;
#pragma unroll
    for (int m = 0; m < M_T; ++m) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
        }
        if (lane == 0) {
            s.rms_part[warp * 2 + m] = ss[m];
        }
    }
    named_barrier_sync(1, kStepConsumers);
    if (t < M) {
        double tot = 0.0;
        for (int w = 0; w < kStepConsumerWarps; ++w) {
            tot += s.rms_part[w * 2 + t];
        }
        const float mean = (float) (tot / (double) H);
        s.rms_scale[t]   = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, a.eps)));
    }
    named_barrier_sync(1, kStepConsumers);
}

// Quantizes K values per token into s.xc / s.xd.  Four lanes per block,
// eight values per lane, so each warp quantizes eight blocks at once.
// src_kind: 0 = normed shared buffer (hsrc * scale * norm), 1 = LL words via
// index map (GQA expansion when map_gqa, else identity).
template <int M_T, int MODE>
__device__ void stage_activations(const StepArgs & a, const Smem & s, int K, int M, int src_kind,
                                  const float * hsrc, const float * norm, const unsigned long long * ll, size_t ll_stride,
                                  bool map_gqa, unsigned epoch, float * trace_x, size_t trace_stride, bool & fail) {
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int NB   = K / kQK;
    const int P    = K / 64;
    const int g4   = lane / 4;
    const int e4   = lane % 4;
    for (int base = warp * 8; base < M * NB; base += kStepConsumerWarps * 8) {
        const int  blk   = base + g4;
        const bool valid = blk < M * NB;
        const int  m     = valid ? blk / NB : 0;
        const int  b     = valid ? blk % NB : 0;
        const int  i0    = b * kQK + e4 * 8;
        float      v[8];
        if (src_kind == 0) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                v[k] = valid ? __fmul_rn(__fmul_rn(hsrc[(size_t) m * K + i0 + k], s.rms_scale[m]), norm[i0 + k])
                             : 0.0f;
            }
        } else {
            const unsigned long long * src[8];
            unsigned long long         w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                int j = i0 + k;
                if (map_gqa) {
                    j = ((j / a.head_dim) / a.group) * a.head_dim + j % a.head_dim;
                }
                src[k] = ll + (size_t) m * ll_stride + j;
                w[k]   = valid ? ld_ll(src[k]) : ((unsigned long long) epoch << 32);
            }
            if (!fail && !ll_settle<8>(a, s, src, w, valid ? 8 : 0, epoch)) {
                fail = true;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                v[k] = valid ? __uint_as_float((unsigned) (w[k] & 0xffffffffu)) : 0.0f;
            }
        }
        const float       am = block_amax<4, 8>(v, e4);
        const QuantParams qp = quant_params<MODE>(am);
        uint32_t          lo = 0, hi = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            lo |= (uint32_t) (quant_code<MODE>(v[k], qp.id) & 0xff) << (8 * k);
            hi |= (uint32_t) (quant_code<MODE>(v[4 + k], qp.id) & 0xff) << (8 * k);
        }
        if (valid) {
            const int pp  = b >> 1;
            const int pos = ((b & 1) << 5) + e4 * 8;
            const int wi  = pos >> 2;  // even
            uint2 *   dst = reinterpret_cast<uint2 *>(s.xc + ((size_t) (m * 4 + (wi >> 2)) * P + pp) * 16 + (wi & 3) * 4);
            *dst          = make_uint2(lo, hi);
            if (e4 == 0) {
                s.xd[m * NB + b] = qp.d;
            }
            if (trace_x != nullptr) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    trace_x[(size_t) m * trace_stride + i0 + k] = v[k];
                }
            }
        }
    }
    named_barrier_sync(1, kStepConsumers);
}

template <int M_T, int MODE>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int G = gridDim.x;
    const int c = blockIdx.x;
    const int M = a.M;
    const int H = a.H;
    const int Kmax = max(max(a.H, a.Q), a.I);

    Smem s;
    s.full        = reinterpret_cast<uint64_t *>(smem);
    s.empty       = s.full + kStepMaxSlots;
    s.epoch       = reinterpret_cast<unsigned *>(smem + 256);
    s.abort_local = reinterpret_cast<int *>(smem + 260);
    s.rms_scale   = reinterpret_cast<float *>(smem + 264);
    s.rms_part    = reinterpret_cast<double *>(smem + 512);
    size_t off    = kStepHeader;
    s.hbuf        = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * H * 4;
    s.h1buf = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * H * 4;
    s.normbuf = reinterpret_cast<float *>(smem + off);
    off += (size_t) H * 4;
    s.ybuf = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * 2 * kStepYMax * 4;
    s.xc = smem + off;
    off += (size_t) M_T * Kmax;
    s.xd = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * (Kmax / kQK) * 4;
    off    = (off + 127) & ~(size_t) 127;
    s.ring = smem + off;
    const int S = a.n_slots;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStepMaxSlots; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kStepConsumerWarps);
        }
        *s.abort_local = 0;
        // launch k (1-based) of this plan: every CTA computes the same k
        *s.epoch = atomicAdd(&a.sync[0], 1u) / (unsigned) G + 1u;
        fence_mbar_init();
    }
    __syncthreads();
    const unsigned epoch = *s.epoch;
    const int      warp  = threadIdx.x / 32;
    const int      lane  = threadIdx.x % 32;

    if (warp == kStepConsumerWarps) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol    = l2_evict_first_policy();
            int            t      = 0;
            bool           stop   = false;
            for (int l = 0; l < a.n_layers && !stop; ++l) {
                Seg segs[5];
                layer_segs(a, l, c, G, segs);
                for (int g = 0; g < 5 && !stop; ++g) {
                    const int nt = seg_tiles(segs[g]);
#ifdef B200Q8_TIMELINE
                    if (a.timeline != nullptr && g != 3) {
                        unsigned long long gt;
                        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt));
                        a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + 4 * l + (g < 3 ? g : 3)) * 8 + 5] = gt;
                    }
#endif
                    for (int k = 0; k < nt; ++k, ++t) {
                        const int sl = t % S;
                        if (t >= S && !mbar_wait_bounded_sleep(&s.empty[sl], ((t / S) - 1) & 1)) {
                            raise_abort(a, s);
                            stop = true;
                            break;
                        }
                        if (*(volatile int *) s.abort_local != 0) {
                            stop = true;
                            break;
                        }
                        const int      r     = k * segs[g].sr;
                        const int      R     = min(segs[g].sr, segs[g].n - r);
                        const uint32_t bytes = (uint32_t) ((size_t) R * segs[g].rb);
                        mbar_arrive_expect_tx(&s.full[sl], bytes);
                        bulk_copy_g2s(s.ring + (size_t) sl * kStepSlotBytes, segs[g].base + (size_t) r * segs[g].rb,
                                      bytes, &s.full[sl], pol);
                    }
                }
            }
            for (int u = max(0, t - S); u < t; ++u) {
                if (!mbar_wait_bounded(&s.full[u % S], (u / S) & 1)) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                }
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int t_id = threadIdx.x;
    // step input: h = x_in + get_rows(table, ids), every CTA for itself
    for (int e = t_id; e < M * H; e += kStepConsumers) {
        const int     m  = e / H;
        const int     k  = e % H;
        const int64_t r  = a.ids[m];
        float         ev = 0.0f;
        if (r >= 0 && r < a.table_rows) {
            const uint8_t * blk = a.table + r * a.rb_h + (k / kQK) * kBlockBytes;
            const float     d   = __half2float(__ushort_as_half((unsigned short) (blk[0] | (blk[1] << 8))));
            ev                  = __fmul_rn((float) (int8_t) blk[2 + k % kQK], d);
        } else if (c == 0 && k == 0) {
            record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
        }
        s.hbuf[e] = __fadd_rn(a.x_in[e], ev);
    }
    named_barrier_sync(1, kStepConsumers);

    const int qkv_dim = a.Q + 2 * a.KV;
    int       t       = 0;      // tile counter, mirrors the producer
    bool      fail    = false;  // this thread saw a timeout or an abort
#ifdef B200Q8_TIMELINE
    long long tl_wait_cycles = 0, tl_dot_cycles = 0;
#endif
    // Consumes the tiles of one weight segment.  A warp whose wait runs out
    // stops consuming (and stops arriving) but still reaches every barrier.
    auto consume = [&](const Seg & sg, int K, int yoff) {
        const int NB = K / kQK;
        const int P  = K / 64;
        const int nt = seg_tiles(sg);
        for (int k = 0; k < nt; ++k, ++t) {
            if (fail) {
                continue;
            }
            const int sl = t % S;
#ifdef B200Q8_TIMELINE
            const long long c0 = clock64();
#endif
            if (!mbar_wait_bounded(&s.full[sl], (t / S) & 1)) {
                raise_abort(a, s);
                fail = true;
                continue;
            }
#ifdef B200Q8_TIMELINE
            const long long c1 = clock64();
#endif
            const int r = k * sg.sr;
            const int R = min(sg.sr, sg.n - r);
            dot_tile_rows<M_T>(s.ring + (size_t) sl * kStepSlotBytes, R, sg.rb, P, NB, s.xc, s.xd, M, warp, lane,
                               kStepConsumerWarps, [&](int rr, int m, float acc) {
                                   s.ybuf[m * 2 * kStepYMax + yoff + r + rr] = acc;
                               });
            __syncwarp();
#ifdef B200Q8_TIMELINE
            const long long c2 = clock64();
            tl_wait_cycles += c1 - c0;
            tl_dot_cycles += c2 - c1;
#endif
            if (lane == 0) {
                mbar_arrive(&s.empty[sl]);
            }
        }
    };
    auto trace = [&](int l, int which) -> float * {
        return a.trace ? a.trace + (size_t) l * a.trace_layer + a.trace_off[which] : nullptr;
    };
    const size_t llm = (size_t) a.ll_m;  // token stride of the LL buffers

    for (int l = 0; l < a.n_layers; ++l) {
        const StepLayerDev &       L    = a.layers[l];
        unsigned long long * const ll_v = a.ll + (size_t) l * a.ll_layer;
        unsigned long long * const ll_o = ll_v + llm * a.KV;
        unsigned long long * const ll_s = ll_o + llm * a.H;
        unsigned long long * const ll_d = ll_s + llm * a.I;
        Seg                        segs[5];
        layer_segs(a, l, c, G, segs);
        const Part pq = part(qkv_dim, G, c);
        const Part po = part(a.H, G, c);
        const Part pg = part(a.I, G, c);

        // ---- qkv = W_qkv * Q(rms_norm(h) * norm_in), h = h1 + d(l-1)
        TL(4 * l + 0, 0);
        const unsigned long long * prev_d = l > 0 ? a.ll + (size_t) (l - 1) * a.ll_layer + llm * (a.KV + a.H + a.I)
                                                  : nullptr;
        residual_and_rms<M_T>(a, s, prev_d, s.h1buf, s.hbuf, M, epoch, (l > 0 && c == 0) ? trace(l - 1, 9) : nullptr,
                              L.norm_in, fail);
        TL(4 * l + 0, 1);
        stage_activations<M_T, MODE>(a, s, H, M, 0, s.hbuf, s.normbuf, nullptr, 0, false, epoch,
                                     c == 0 ? trace(l, 0) : nullptr, (size_t) H, fail);
        TL(4 * l + 0, 2);
        consume(segs[0], H, 0);
        TL(4 * l + 0, 3);
        TL_CYC(4 * l + 0);
        if (consumers_any(fail || aborted(a, s))) {
            break;
        }
        TL(4 * l + 0, 4);
        {
            float * tq = trace(l, 1);
            for (int e = t_id; e < M * pq.n; e += kStepConsumers) {
                const int   m   = e / pq.n;
                const int   i   = e % pq.n;
                const int   row = pq.r0 + i;
                const float v   = s.ybuf[m * 2 * kStepYMax + i];
                if (row >= a.Q + a.KV) {
                    st_ll(ll_v + (size_t) m * a.KV + (row - a.Q - a.KV), v, epoch);
                }
                if (tq) {
                    tq[(size_t) m * qkv_dim + row] = v;
                }
            }
        }
        // ---- o = W_o * Q(attend(v)); attention over one cached position
        TL(4 * l + 1, 0);
        stage_activations<M_T, MODE>(a, s, a.Q, M, 1, nullptr, nullptr, ll_v, (size_t) a.KV, true, epoch,
                                     c == 0 ? trace(l, 2) : nullptr, (size_t) a.Q, fail);
        TL(4 * l + 1, 2);
        consume(segs[1], a.Q, 0);
        TL(4 * l + 1, 3);
        TL_CYC(4 * l + 1);
        if (consumers_any(fail || aborted(a, s))) {
            break;
        }
        TL(4 * l + 1, 4);
        {
            float * to = trace(l, 3);
            for (int e = t_id; e < M * po.n; e += kStepConsumers) {
                const int   m = e / po.n;
                const int   i = e % po.n;
                const float v = s.ybuf[m * 2 * kStepYMax + i];
                st_ll(ll_o + (size_t) m * a.H + po.r0 + i, v, epoch);
                if (to) {
                    to[(size_t) m * a.H + po.r0 + i] = v;
                }
            }
        }
        // ---- g|u = W_gate|W_up * Q(rms_norm(h1) * norm_post), h1 = h + o
        TL(4 * l + 2, 0);
        residual_and_rms<M_T>(a, s, ll_o, s.hbuf, s.h1buf, M, epoch, c == 0 ? trace(l, 4) : nullptr, L.norm_post,
                              fail);
        TL(4 * l + 2, 1);
        stage_activations<M_T, MODE>(a, s, H, M, 0, s.h1buf, s.normbuf, nullptr, 0, false, epoch,
                                     c == 0 ? trace(l, 5) : nullptr, (size_t) H, fail);
        TL(4 * l + 2, 2);
        consume(segs[2], H, 0);
        consume(segs[3], H, kStepYMax);
        TL(4 * l + 2, 3);
        TL_CYC(4 * l + 2);
        if (consumers_any(fail || aborted(a, s))) {
            break;
        }
        TL(4 * l + 2, 4);
        {
            float * tgu = trace(l, 6);
            float * ts  = trace(l, 7);
            for (int e = t_id; e < M * pg.n; e += kStepConsumers) {
                const int   m  = e / pg.n;
                const int   i  = e % pg.n;
                const float gv = s.ybuf[m * 2 * kStepYMax + i];
                const float uv = s.ybuf[m * 2 * kStepYMax + kStepYMax + i];
                const float sv = __fmul_rn(silu_f32(gv), uv);
                st_ll(ll_s + (size_t) m * a.I + pg.r0 + i, sv, epoch);
                if (tgu) {
                    tgu[(size_t) m * 2 * a.I + pg.r0 + i]       = gv;
                    tgu[(size_t) m * 2 * a.I + a.I + pg.r0 + i] = uv;
                }
                if (ts) {
                    ts[(size_t) m * a.I + pg.r0 + i] = sv;
                }
            }
        }
        // ---- d = W_down * Q(s)
        TL(4 * l + 3, 0);
        stage_activations<M_T, MODE>(a, s, a.I, M, 1, nullptr, nullptr, ll_s, (size_t) a.I, false, epoch, nullptr,
                                     0, fail);
        TL(4 * l + 3, 2);
        consume(segs[4], a.I, 0);
        TL(4 * l + 3, 3);
        TL_CYC(4 * l + 3);
        if (consumers_any(fail || aborted(a, s))) {
            break;
        }
        TL(4 * l + 3, 4);
        {
            float *    td   = trace(l, 8);
            const bool last = l == a.n_layers - 1;
            for (int e = t_id; e < M * po.n; e += kStepConsumers) {
                const int   m   = e / po.n;
                const int   i   = e % po.n;
                const int   row = po.r0 + i;
                const float v   = s.ybuf[m * 2 * kStepYMax + i];
                if (last) {
                    a.h_out[(size_t) m * H + row] = __fadd_rn(s.h1buf[m * H + row], v);
                } else {
                    st_ll(ll_d + (size_t) m * a.H + row, v, epoch);
                }
                if (td) {
                    td[(size_t) m * a.H + row] = v;
                }
            }
        }
    }
}

}  // namespace

size_t decode_step_smem_bytes(const StepArgs & a, int mt, int & n_slots) {
    const int Kmax = std::max(std::max(a.H, a.Q), a.I);
    size_t    off  = kStepHeader;
    off += (size_t) mt * a.H * 4 * 2;
    off += (size_t) a.H * 4;
    off += (size_t) mt * 2 * kStepYMax * 4;
    off += (size_t) mt * Kmax;
    off += (size_t) mt * (Kmax / kQK) * 4;
    off                   = (off + 127) & ~(size_t) 127;
    const size_t limit    = 227 * 1024;
    if (off + kStepSlotBytes * 2 > limit) {
        n_slots = 0;
        return 0;
    }
    n_slots = (int) std::min<size_t>(kStepMaxSlots, (limit - off) / kStepSlotBytes);
    return off + (size_t) n_slots * kStepSlotBytes;
}

bool decode_step_supported(const StepArgs & a, int G) {
    if (a.M < 1 || a.M > 2 || a.H % 256 || a.Q % 256 || a.I % 256 || a.KV % 32) {
        return false;
    }
    // every CTA's slice of one op must fit the output staging buffer
    const int qkv = a.Q + 2 * a.KV;
    if ((qkv + G - 1) / G > 2 * kStepYMax || (a.I + G - 1) / G > kStepYMax || (a.H + G - 1) / G > kStepYMax) {
        return false;
    }
    if (a.rb_i > (size_t) kStepSlotBytes || a.rb_q > (size_t) kStepSlotBytes || a.rb_h > (size_t) kStepSlotBytes) {
        return false;
    }
    int slots = 0;
    return decode_step_smem_bytes(a, a.M <= 1 ? 1 : 2, slots) > 0 && slots >= 2;
}

cudaError_t launch_decode_step(StepArgs a, int G, cudaStream_t stream) {
    const int mt   = a.M <= 1 ? 1 : 2;
    int       slots = 0;
    const size_t smem = decode_step_smem_bytes(a, mt, slots);
    a.n_slots         = slots;
    void (*fn)(const StepArgs) = nullptr;
    switch (a.mode) {
        case B200Q8_QUANT_CPU_X86: fn = mt == 1 ? decode_step_kernel<1, B200Q8_QUANT_CPU_X86> : decode_step_kernel<2, B200Q8_QUANT_CPU_X86>; break;
        case B200Q8_QUANT_CPU_ARM: fn = mt == 1 ? decode_step_kernel<1, B200Q8_QUANT_CPU_ARM> : decode_step_kernel<2, B200Q8_QUANT_CPU_ARM>; break;
        default: fn = mt == 1 ? decode_step_kernel<1, B200Q8_QUANT_REF> : decode_step_kernel<2, B200Q8_QUANT_REF>; break;
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) {
        return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) G);
    cfg.blockDim           = dim3(kStepThreads);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id             = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs              = attr;
    cfg.numAttrs           = 1;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace b200q8
