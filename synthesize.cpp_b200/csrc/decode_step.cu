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

constexpr int kStepConsumerWarps = 12;
constexpr int kStepConsumers     = kStepConsumerWarps * 32;
constexpr int kStepThreads       = kStepConsumers + 32;
constexpr int kStepSlotBytes     = 16384;
constexpr int kStepMaxSlots      = 16;
constexpr int kStepYMax          = 64;  // rows one CTA produces in one op (per token)
constexpr int kStepHeader        = 2048;
// Tokens per launch.  The kernel's token loops are written for any M_T (the
// tokens' elements and blocks are flat ranges), and it was measured with 4
// and 8 token slots: 0.968 / 1.880 ms per step at M = 4 / 8, against 0.755 /
// 0.757 ms for the per-op tensor-core GEMM chain, whose MMAs take 8 tokens at
// once.  From M = 3 on the chain runs that path, and the step keeps 1 and 2.
constexpr int kStepMaxM          = 2;

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
#else
#define TL(op, ev) ((void) 0)
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
    int t = 0;
    for (int r = 0; r < s.n; r += s.sr) {
        ++t;
    }
    return t;
}

// Token facts the attention CTAs keep for the whole launch (header words).
struct AttTok {
    int pos[2];
    int slot[2];
    int ok[2];
};

struct Smem {
    uint64_t * full;
    uint64_t * empty;
    unsigned * epoch;
    int *      abort_local;
    double *   rms_part;   // [kStepConsumerWarps][M_T] (header room for 12 warps x 8 tokens)
    float *    rms_scale;  // unused slot kept for the header layout
    float *    hbuf;       // [M_T][H]
    float *    h1buf;      // [M_T][H]
    float *    normbuf;    // [H] the RMS-norm weight of the current norm op
    float *    ybuf;       // [M_T][2*kStepYMax]
    uint8_t *  xc[2];      // staged codes [M_T][Kmax], double buffered by op parity
    float *    xd[2];      // staged scales [M_T][Kmax/32]
    float *    att;        // attention scratch (attention steps): q, 2 k, 2 v rows, per-warp partials
    AttTok *   tok;        // attention steps: positions and slots of the launch's tokens
    uint8_t *  ring;
    double     inv_h;      // 1 / H when H is a power of two, else 0
};

// Floats of attention scratch: q [hd], k and v of up to 2 in-launch tokens
// [2][hd] each, per-warp weighted V [warps][hd], per-warp max and sum, the
// layer's q_norm and k_norm [hd] each, and per token of the launch the RoPE
// cos and sin at its position [2][hd] (cos at i, sin at hd/2 + i).
__host__ __device__ constexpr size_t att_scratch_floats(int hd) {
    return (size_t) hd * (1 + 2 + 2 + kStepConsumerWarps) + 2 * kStepConsumerWarps + 2 * (size_t) hd + 2 * (size_t) hd;
}

// Offsets (floats) in the attention scratch of q_norm / k_norm and of the
// RoPE table.
__host__ __device__ constexpr size_t att_norm_offset(int hd) {
    return (size_t) hd * (1 + 2 + 2 + kStepConsumerWarps) + 2 * kStepConsumerWarps;
}
__host__ __device__ constexpr size_t att_rope_offset(int hd) {
    return att_norm_offset(hd) + 2 * (size_t) hd;
}


// This CTA's row slices and tile sizes, the same for every layer; computed
// once per launch (each holds runtime divisions).
struct Plan {
    Part pq, ph, pi;       // rows of q|k|v, of H (o and down), of I (gate and up)
    int  sr_h, sr_q, sr_i;  // rows per 16 KiB slot for K = H, Q, I
};

__device__ __forceinline__ Plan make_plan(const StepArgs & a, int c, int G) {
    Plan p;
    p.pq   = part(a.Q + 2 * a.KV, G, c);
    p.ph   = part(a.H, G, c);
    p.pi   = part(a.I, G, c);
    p.sr_h = max(1, (int) (kStepSlotBytes / a.rb_h));
    p.sr_q = max(1, (int) (kStepSlotBytes / a.rb_q));
    p.sr_i = max(1, (int) (kStepSlotBytes / a.rb_i));
    return p;
}

// The 5 weight segments of layer l for this CTA, in streaming order:
// qkv, o, gate, up, down.
__device__ __forceinline__ void layer_segs(const StepArgs & a, const Plan & p, int l, Seg (&segs)[5]) {
    const StepLayerDev & L = a.layers[l];
    segs[0] = { L.w_qkv + (size_t) p.pq.r0 * a.rb_h, a.rb_h, p.pq.n, p.sr_h };
    segs[1] = { L.w_o + (size_t) p.ph.r0 * a.rb_q, a.rb_q, p.ph.n, p.sr_q };
    segs[2] = { L.w_gate + (size_t) p.pi.r0 * a.rb_h, a.rb_h, p.pi.n, p.sr_h };
    segs[3] = { L.w_up + (size_t) p.pi.r0 * a.rb_h, a.rb_h, p.pi.n, p.sr_h };
    segs[4] = { L.w_down + (size_t) p.ph.r0 * a.rb_i, a.rb_i, p.ph.n, p.sr_i };
}

// This CTA's rows of the output head.
__device__ __forceinline__ Seg head_seg(const StepArgs & a, const Plan & p, int c, int G) {
    const Part pv = part(a.vocab, G, c);
    return { a.head + (size_t) pv.r0 * a.rb_h, a.rb_h, pv.n, p.sr_h };
}

// The global abort word holds the epoch of the launch that raised it, so an
// abort left by an earlier launch of the same plan does not stop this one.
__device__ __forceinline__ bool aborted(const StepArgs & a, const Smem & s) {
    return *(volatile int *) s.abort_local != 0 || *(volatile unsigned *) &a.sync[1] == *(volatile unsigned *) s.epoch;
}

__device__ void raise_abort(const StepArgs & a, const Smem & s) {
    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
    *(volatile int *) s.abort_local = 1;
    atomicExch(&a.sync[1], *(volatile unsigned *) s.epoch);
}

// This CTA's own stop flag (set by raise_abort and stop_producer).  The
// barriers between ops check only this: another CTA's abort reaches this one
// through the global word, which every bounded wait polls, so a barrier need
// not pay an L2 round trip for it.
__device__ __forceinline__ bool local_stop(const Smem & s) {
    return *(volatile int *) s.abort_local != 0;
}

// Consumers that stop early tell their producer, which then stops waiting
// for slots to be released.
__device__ __forceinline__ void stop_producer(const Smem & s) {
    if (threadIdx.x == 0) {
        *(volatile int *) s.abort_local = 1;
    }
}

// Reads n LL words (this thread's share, already loaded in w[]) until all
// carry `epoch`.  Returns false on timeout/abort.
template <int N>
__device__ __forceinline__ bool ll_settle_one(const StepArgs & a, const Smem & s,
                                              const unsigned long long * const (&src)[N], unsigned long long (&w)[N],
                                              int n, unsigned epoch) {
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

template <int N>
__device__ __forceinline__ bool ll_settle(const StepArgs & a, const Smem & s, const unsigned long long * const (&src)[N],
                                          unsigned long long (&w)[N], int n, unsigned epoch) {
    if (N > 4) {  // the staggered second reads would not fit the registers
        return ll_settle_one<N>(a, s, src, w, n, epoch);
    }
    unsigned pend = 0;  // words not yet seen with this launch's epoch
#pragma unroll
    for (int i = 0; i < N; ++i) {
        if (i < n && (unsigned) (w[i] >> 32) != epoch) {
            pend |= 1u << i;
        }
    }
    if (pend == 0) {
        return true;
    }
    // Two reads of each pending word stay in flight, the second started
    // kPollStagger cycles after the first, so a word that lands is seen about
    // half a round trip sooner than with one read at a time.  Landed words go
    // to val (a register a read is still headed for is never written over).
    constexpr long long kPollStagger = 300;
    unsigned long long  val[N];
    unsigned long long  r1[N], r2[N];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        val[i] = w[i];
        r1[i]  = w[i];
    }
    const long long start = clock64();
    while (clock64() - start < kPollStagger) {
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
        r2[i] = (pend >> i) & 1u ? ld_ll(src[i]) : 0ull;
    }
    for (unsigned iter = 0;; ++iter) {
        // the pending words' first reads (r1 holds the caller's reads at first)
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if (((pend >> i) & 1u) && (unsigned) (r1[i] >> 32) == epoch) {
                val[i] = r1[i];
                pend &= ~(1u << i);
            }
        }
        if (pend == 0) {
            break;
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if ((pend >> i) & 1u) {
                r1[i] = ld_ll(src[i]);
            }
        }
        // their second reads
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if (((pend >> i) & 1u) && (unsigned) (r2[i] >> 32) == epoch) {
                val[i] = r2[i];
                pend &= ~(1u << i);
            }
        }
        if (pend == 0) {
            break;
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if ((pend >> i) & 1u) {
                r2[i] = ld_ll(src[i]);
            }
        }
        if (clock64() - start > kWaitLimitCycles) {
            return false;
        } else if ((iter & 255u) == 255u && aborted(a, s)) {
            // the global abort word costs an L2 round trip: look rarely
            return false;
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
        w[i] = val[i];
    }
    return true;
}

// Phase A of a norm stage: h_dst[m][i] = h_src[m][i] + published delta[m][i]
// for all i < H (delta read as LL words; delta == nullptr: h_dst already
// holds the values), accumulating sum of squares per token.  Then the
// per-token RMS scale, returned in scale_out (every thread gets it).
template <int M_T>
__device__ void residual_and_rms(const StepArgs & a, const Smem & s, const unsigned long long * delta,
                                 const float * h_src, float * h_dst, int M, unsigned epoch, float * trace_h,
                                 const float * norm, bool & fail, float (&scale_out)[M_T]) {
    const int H = a.H;
    const int t = threadIdx.x;
    // The norm weight is loaded into registers now and stored to shared
    // memory after the wait for the previous op's outputs, which hides its L2
    // latency (a store right behind the load would stall on it).
    constexpr int kNormRegs = 8;  // widths up to 8 * kStepConsumers
    float         nreg[kNormRegs];
#pragma unroll
    for (int k = 0; k < kNormRegs; ++k) {
        const int i = t + k * kStepConsumers;
        nreg[k]     = i < H ? norm[i] : 0.0f;
    }
    for (int i = t + kNormRegs * kStepConsumers; i < H; i += kStepConsumers) {
        s.normbuf[i] = norm[i];
    }
    double    ss[M_T];
#pragma unroll
    for (int m = 0; m < M_T; ++m) {
        ss[m] = 0.0;
    }
    // The M tokens' H values are one flat range of M * H elements (element
    // i = m * H + e), taken kPer per thread per pass.  (Token by token
    // measured slower at M = 1; issuing a pass's reads before the previous
    // pass settles measured slower too: the extra registers spill in the
    // several-token kernels.)
    constexpr int kPer   = 4;  // elements in flight per thread per pass
    const int     total  = M * H;
    const int     lg_h   = (H & (H - 1)) == 0 ? __ffs(H) - 1 : -1;
    const int     stride = kStepConsumers * kPer;
    // a pass's words: the first one's address (the others follow at the
    // consumer-count stride) and the kPer words read so far
    auto load = [&](int base, const unsigned long long *& p0, unsigned long long (&w)[kPer], int & n) {
        n  = 0;
        p0 = delta != nullptr ? delta + base + t : nullptr;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = base + i * kStepConsumers + t;
            w[i]        = 0;
            if (e < total) {
                n = i + 1;
                if (delta != nullptr) {
                    w[i] = ld_ll(p0 + i * kStepConsumers);
                }
            }
        }
    };
    const unsigned long long * p0 = nullptr;
    unsigned long long         w[kPer];
    int                        n = 0;
    load(0, p0, w, n);
    for (int base = 0; base < total; base += stride) {
        if (delta != nullptr && !fail) {
            const unsigned long long * src[kPer];
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                src[i] = p0 + (i < n ? i * kStepConsumers : 0);
            }
            if (!ll_settle<kPer>(a, s, src, w, n, epoch)) {
                raise_abort(a, s);  // records the timeout; other CTAs stop at their next check
                fail = true;
            }
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = base + i * kStepConsumers + t;
            if (e < total) {
                const int m = M_T == 1 ? 0 : lg_h >= 0 ? e >> lg_h : e / H;
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
        if (base + stride < total) {  // the next pass's reads go out once this one is done
            load(base + stride, p0, w, n);
        }
    }
#pragma unroll
    for (int k = 0; k < kNormRegs; ++k) {
        const int i = t + k * kStepConsumers;
        if (i < H) {
            s.normbuf[i] = nreg[k];
        }
    }
    const int warp = t >> 5;
    const int lane = t & 31;
#pragma unroll
    for (int m = 0; m < M_T; ++m) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
        }
        if (lane == 0) {
            s.rms_part[warp * M_T + m] = ss[m];
        }
    }
    named_barrier_sync(1, kStepConsumers);
    // every thread sums the per-warp partials in the same order (no second
    // barrier needed to hand the scale around)
#pragma unroll
    for (int m = 0; m < M_T; ++m) {
        double tot = 0.0;
        for (int w = 0; w < kStepConsumerWarps; ++w) {
            tot += s.rms_part[w * M_T + m];
        }
        // dividing by a power of two is multiplying by its exact reciprocal
        const float mean = (float) (s.inv_h != 0.0 ? tot * s.inv_h : tot / (double) H);
        scale_out[m]     = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, a.eps)));
    }
}

// Quantizes K values per token of the normed shared buffer (hsrc * scale *
// norm) into the staging buffer xc/xd (chunk-major layout of tile_dot.cuh).
// LPB lanes per block, 32/LPB consecutive values per lane; the caller picks
// LPB so that every block of a token is staged in one round.  Ends with the
// consumer barrier, which also ORs every thread's failure flag: returns true
// when the step must stop.
template <int M_T, int MODE, int LPB>
__device__ bool stage_activations_t(const StepArgs & a, const Smem & s, int K, int M, const float * hsrc,
                                    const float * norm, const float (&scale)[M_T], float * trace_x,
                                    size_t trace_stride, uint8_t * xc, float * xd, bool & fail) {
    constexpr int E    = 32 / LPB;  // values per lane
    constexpr int BPW  = 32 / LPB;  // blocks per warp per round
    const int     warp = threadIdx.x >> 5;
    const int     lane = threadIdx.x & 31;
    const int     NB   = K >> 5;
    const int     NSB  = K >> 8;
    const int     gb   = lane / LPB;  // block within the warp's BPW
    const int     eb   = lane % LPB;  // values E*eb .. E*eb+E-1 of the block
    // the M tokens' blocks are one flat range (token m's block b is m * NB + b),
    // so the tokens share the rounds
    const int     MNB  = M * NB;
    for (int base = warp * BPW; base < MNB; base += kStepConsumerWarps * BPW) {
        const int   bf    = base + gb;
        const bool  valid = bf < MNB;
        const int   m     = M_T == 1 || !valid ? 0 : bf / NB;
        const int   b     = valid ? bf - m * NB : 0;
        const int   i0    = b * kQK + eb * E;
        float       sc    = scale[0];
#pragma unroll
        for (int mm = 1; mm < M_T; ++mm) {
            sc = m == mm ? scale[mm] : sc;
        }
        float       v[E];
        // 128-bit loads (both buffers and i0 are 16-byte aligned): a lane's
        // values are 16 bytes apart from its neighbour's, and scalar loads at
        // that stride would conflict four ways
#pragma unroll
        for (int q = 0; q < E / 4; ++q) {
            const float4 h4 = *reinterpret_cast<const float4 *>(hsrc + (size_t) m * K + i0 + 4 * q);
            const float4 n4 = *reinterpret_cast<const float4 *>(norm + i0 + 4 * q);
            v[4 * q]        = __fmul_rn(__fmul_rn(h4.x, sc), n4.x);
            v[4 * q + 1]    = __fmul_rn(__fmul_rn(h4.y, sc), n4.y);
            v[4 * q + 2]    = __fmul_rn(__fmul_rn(h4.z, sc), n4.z);
            v[4 * q + 3]    = __fmul_rn(__fmul_rn(h4.w, sc), n4.w);
        }
#pragma unroll
        for (int k = 0; k < E; ++k) {
            v[k] = valid ? v[k] : 0.0f;
        }
        const float       am = block_amax<LPB, E>(v, eb);
        const QuantParams qp = quant_params<MODE>(am);
        uint32_t          words[E / 4];
#pragma unroll
        for (int q = 0; q < E / 4; ++q) {
            words[q] = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                words[q] |= (uint32_t) (quant_code<MODE>(v[4 * q + k], qp.id) & 0xff) << (8 * k);
            }
        }
        if (valid) {
            const int pos = ((b & 7) << 5) + eb * E;  // E consecutive codes stay inside one 16-byte chunk
            uint8_t * dst = xc + sb_code_offset(m, K, NSB, b >> 3, pos);
            if (E == 4) {
                *reinterpret_cast<uint32_t *>(dst) = words[0];
            } else if (E == 8) {
                *reinterpret_cast<uint2 *>(dst) = make_uint2(words[0], words[1]);
            } else {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(words[0], words[1], words[2], words[3 % (E / 4)]);
            }
            if (eb == 0) {
                xd[m * NB + b] = qp.d;
            }
            if (trace_x != nullptr) {
#pragma unroll
                for (int k = 0; k < E; ++k) {
                    trace_x[(size_t) m * trace_stride + i0 + k] = v[k];
                }
            }
        }
    }
    return consumers_any(fail || local_stop(s));
}

// Quantizes K values per token read from LL words (ll + m * ll_stride) into
// xc/xd.  Lane eb of a block's LPB lanes holds the block's values eb + LPB*k,
// so at every load the lanes of a warp read whole 32-byte sectors (a lane
// holding consecutive values would make each load touch a sector per lane).
// With lg_rep > 0 (the single cached position's GQA expansion) the source
// holds K >> lg_rep values, a kv head per 1 << lg_rep query heads: each source
// block is waited for and quantized once and stored at every query-head
// position that reads it.  Ends with the consumer barrier, which also ORs
// every thread's failure flag: returns true when the step must stop.
template <int M_T, int MODE, int LPB>
__device__ bool stage_ll_t(const StepArgs & a, const Smem & s, int K, int M, const unsigned long long * ll,
                           size_t ll_stride, int lg_rep, unsigned epoch, float * trace_x, size_t trace_stride,
                           uint8_t * xc, float * xd, bool & fail) {
    constexpr int E    = 32 / LPB;  // values per lane
    constexpr int BPW  = 32 / LPB;  // blocks per warp per round
    const int     warp = threadIdx.x >> 5;
    const int     lane = threadIdx.x & 31;
    const int     NB   = K >> 5;
    const int     NSB  = K >> 8;
    const int     NBs  = NB >> lg_rep;  // source blocks
    const int     gb   = lane / LPB;
    const int     eb   = lane % LPB;
    for (int m = 0; m < M; ++m)
    for (int base = warp * BPW; base < NBs; base += kStepConsumerWarps * BPW) {
        const int                  b     = base + gb;
        const bool                 valid = b < NBs;
        const unsigned long long * row   = ll + (size_t) m * ll_stride + (size_t) (valid ? b : 0) * kQK + eb;
        const unsigned long long * src[E];
        unsigned long long         w[E];
#pragma unroll
        for (int k = 0; k < E; ++k) {
            src[k] = row + LPB * k;
            w[k]   = valid ? ld_ll(src[k]) : ((unsigned long long) epoch << 32);
        }
        if (!fail && !ll_settle<E>(a, s, src, w, valid ? E : 0, epoch)) {
            raise_abort(a, s);
            fail = true;
        }
        float v[E];
#pragma unroll
        for (int k = 0; k < E; ++k) {
            v[k] = valid ? __uint_as_float((unsigned) (w[k] & 0xffffffffu)) : 0.0f;
        }
        const float       am = block_amax<LPB, E, true>(v, eb);
        const QuantParams qp = quant_params<MODE>(am);
        uint8_t           code[E];
#pragma unroll
        for (int k = 0; k < E; ++k) {
            code[k] = (uint8_t) (quant_code<MODE>(v[k], qp.id) & 0xff);
        }
        if (valid) {
            for (int r = 0; r < (1 << lg_rep); ++r) {
                int db = b;  // destination block of replica r
                if (lg_rep > 0) {
                    const int j  = b << 5;  // first source index of the block
                    const int hk = j >> a.lg_head_dim;
                    db = ((((hk << lg_rep) + r) << a.lg_head_dim) | (j & ((1 << a.lg_head_dim) - 1))) >> 5;
                }
#pragma unroll
                for (int k = 0; k < E; ++k) {
                    xc[sb_code_offset(m, K, NSB, db >> 3, ((db & 7) << 5) + eb + LPB * k)] = code[k];
                }
                if (eb == 0) {
                    xd[m * NB + db] = qp.d;
                }
                if (trace_x != nullptr) {
#pragma unroll
                    for (int k = 0; k < E; ++k) {
                        trace_x[(size_t) m * trace_stride + (size_t) db * kQK + eb + LPB * k] = v[k];
                    }
                }
            }
        }
    }
    return consumers_any(fail || local_stop(s));
}

// Lanes per block by one token's blocks: 8 up to 4 * kStepConsumerWarps
// blocks, then 4, then 2; the M tokens' blocks form one flat range taken in
// as many rounds as it needs (one lane group per block keeps the per-lane
// chains short: one round of all tokens with fewer lanes per block measured
// slower).  src_kind 0 stages the normed shared buffer (stage_activations_t),
// 1 LL words (stage_ll_t; map_gqa: the source holds the kv heads of the GQA
// expansion).
template <int M_T, int MODE>
__device__ bool stage_activations(const StepArgs & a, const Smem & s, int K, int M, int src_kind, const float * hsrc,
                                  const float * norm, const float (&scale)[M_T], const unsigned long long * ll,
                                  size_t ll_stride, bool map_gqa, unsigned epoch, float * trace_x, size_t trace_stride,
                                  uint8_t * xc, float * xd, bool & fail) {
    if (src_kind == 1) {
        // lanes per block by one token's source blocks: a lane keeps at most 8
        // words (4 where they fit) pending, further tokens take further rounds
        const int lg_rep = map_gqa ? a.lg_group : 0;
        const int NBs    = (K >> 5) >> lg_rep;
        if (NBs <= kStepConsumerWarps * 4) {
            return stage_ll_t<M_T, MODE, 8>(a, s, K, M, ll, ll_stride, lg_rep, epoch, trace_x, trace_stride, xc, xd,
                                            fail);
        }
        if (NBs <= kStepConsumerWarps * 8) {
            return stage_ll_t<M_T, MODE, 4>(a, s, K, M, ll, ll_stride, lg_rep, epoch, trace_x, trace_stride, xc, xd,
                                            fail);
        }
        return stage_ll_t<M_T, MODE, 2>(a, s, K, M, ll, ll_stride, lg_rep, epoch, trace_x, trace_stride, xc, xd, fail);
    }
    const int NB = K >> 5;  // one token's blocks (further tokens take further rounds)
    if (NB <= kStepConsumerWarps * 4) {
        return stage_activations_t<M_T, MODE, 8>(a, s, K, M, hsrc, norm, scale, trace_x, trace_stride, xc, xd, fail);
    }
    if (NB <= kStepConsumerWarps * 8) {
        return stage_activations_t<M_T, MODE, 4>(a, s, K, M, hsrc, norm, scale, trace_x, trace_stride, xc, xd, fail);
    }
    return stage_activations_t<M_T, MODE, 2>(a, s, K, M, hsrc, norm, scale, trace_x, trace_stride, xc, xd, fail);
}

// The tiles of one op occupy consecutive ring slots in streaming order: tile
// i sits in slot (sl0 + i) mod S and was filled in round ph0, flipped once per
// wrap of the ring.
__device__ __forceinline__ int tile_slot(int sl0, int S, int i) {
    int q = sl0 + i;
    while (q >= S) {
        q -= S;
    }
    return q;
}

__device__ __forceinline__ uint32_t tile_phase(int sl0, uint32_t ph0, int S, int i) {
    int      q = sl0 + i;
    uint32_t p = ph0;
    while (q >= S) {
        q -= S;
        p ^= 1u;
    }
    return p;
}

// The tiles of an op still held when consume_op returns: [a0, a1) and
// [b0, b1) of the op's tile indices, counted from slot sl0.
struct Release {
    int sl0 = 0;
    int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
};

// Hands the op's held slots back to the producer.  Called by every consumer
// after the consumer barrier that ends the op (so every warp is done with the
// slots, whose data each saw land): one thread arrives for all consumer warps
// at once, while the others go on to the next op's inputs.
__device__ __forceinline__ void release_tiles(const Smem & s, int S, const Release & r) {
    if (threadIdx.x == kStepConsumers - 32) {  // lane 0 of the last consumer warp
        for (int i = r.a0; i < r.a1; ++i) {
            mbar_arrive_count(&s.empty[tile_slot(r.sl0, S, i)], kStepConsumerWarps);
        }
        for (int i = r.b0; i < r.b1; ++i) {
            mbar_arrive_count(&s.empty[tile_slot(r.sl0, S, i)], kStepConsumerWarps);
        }
    }
}

// One op's tile geometry and ring position, worked out (and its first
// round's tiles waited for) by plan_op before the op's inputs are: none of it
// depends on them, and a CTA always has time to spare while the previous op's
// outputs travel.
struct OpRun {
    int      sl0;     // slot of the op's first tile
    uint32_t ph0;     // its fill round mod 2
    int      nt;      // tiles of the op
    int      seg1;    // first tile of segment 1
    int      n_r;     // tiles per segment (pair ops) or all tiles
    int      per_rd;  // tile pairs per round (pair ops larger than the ring)
    int      lgs;     // log2 of the lanes per row group (~1 half-superblock per lane)
};

// Plans the op on segs[0..nseg) (pair_units: two equal segments consumed as
// row pairs) at ring position sl / ph, advances sl / ph past its tiles and
// waits for the tiles of its first round: lane i of each warp waits for tile
// i, so the round is checked in one go.  Sets fail (warp-uniform) when a wait
// timed out or the op is beyond the tile table.
__device__ __forceinline__ OpRun plan_op(const StepArgs & a, const Smem & s, int S, int & sl, uint32_t & ph,
                                         const Seg * segs, int nseg, bool pair_units, int K, int lane, bool & fail) {
    constexpr int kMaxOpTiles = 16;
    OpRun         o;
    o.sl0  = sl;
    o.ph0  = ph;
    o.nt   = 0;
    o.seg1 = 0;
    for (int g = 0; g < nseg; ++g) {
        if (g == 1) {
            o.seg1 = o.nt;
        }
        o.nt += seg_tiles(segs[g]);
    }
    sl       = tile_slot(o.sl0, S, o.nt);  // the ring position after this op's tiles
    ph       = tile_phase(o.sl0, o.ph0, S, o.nt);
    o.n_r    = pair_units ? o.seg1 : o.nt;
    o.per_rd = pair_units && 2 * o.n_r > S ? min(o.n_r, S - o.n_r) : o.n_r;
    o.lgs    = min(5, 32 - __clz(2 * (K >> 8) - 1));
    // an op with no rows in this CTA (narrow shapes) has nothing to wait for;
    // an op beyond the tile table is refused by decode_step_supported, and is
    // recorded as an internal error should it get here
    const bool too_big = o.nt > kMaxOpTiles || (o.nt > 0 && o.per_rd < 1);
    if (too_big && lane == 0) {
        record_device_error((unsigned) B200Q8_ERR_INTERNAL);
    }
    const int k1   = min(o.n_r, o.per_rd);
    const int nin  = (pair_units ? 2 : 1) * k1;
    bool      rbad = false;
    if (!fail && !too_big && lane < nin) {
        const int ti = lane < k1 ? lane : o.seg1 + (lane - k1);
        if (!mbar_wait_bounded(&s.full[tile_slot(o.sl0, S, ti)], tile_phase(o.sl0, o.ph0, S, ti))) {
            raise_abort(a, s);
            rbad = true;
        }
    }
    rbad = __any_sync(0xffffffffu, rbad);
    fail = fail || rbad || too_big;
    return o;
}

// Consumes all tiles of the op planned in o over all consumer warps.  The
// op's rows come from segs[0..nseg) in streaming order; with pair_units the
// op has two segments of equal length (gate, up) and unit u is the row pair
// (seg0 row u, seg1 row u), computed by one lane group so that SwiGLU can be
// applied before publishing.  Otherwise nseg == 1 and unit u is row u.
// publish(u, acc0, acc1) is called by lane 0 of the unit's group.  The first
// round's tiles were waited for by plan_op.  The slots of the op's last
// round are left held and described in rel: the caller releases them with
// release_tiles after the op's consumer barrier.
template <int M_T, typename Pub>
__device__ __forceinline__ void consume_op(const StepArgs & a, const Smem & s, int S, const OpRun & o,
                                           const Seg * segs, bool pair_units, int K, int M, int warp, int lane,
                                           const uint8_t * xc, const float * xd, bool & fail, int op, Release & rel,
                                           Pub && publish) {
    rel     = Release();
    rel.sl0 = o.sl0;
#ifdef B200Q8_TIMELINE
    const long long tc0 = clock64();
#endif
    // The op is consumed in rounds of tiles.  A single-segment op, or a pair
    // op whose tiles all fit the ring, is one round.  A pair op (gate, up)
    // too large for the ring takes R tile pairs per round, R = S - n_r with
    // n_r tiles per segment: the last fill the first tile round needs reuses
    // the slot of a fill from an earlier op, and each later round's last fill
    // reuses a slot an earlier round released, so the producer never waits on
    // a slot the consumers still hold.
    bool bad = fail;  // warp-uniform
#ifdef B200Q8_TIMELINE
    const long long tc1 = clock64();
    long long       tc_pub = 0;
#endif
    const int      NSB    = K >> 8;  // superblocks per row
    const int      NB     = K >> 5;
    const int      GS     = 1 << o.lgs;
    const int      gpw    = 32 >> o.lgs;  // groups per warp
    const int      ngroup = kStepConsumerWarps * gpw;
    const int      gl     = lane & (GS - 1);
    const bool     split  = pair_units && o.lgs <= 4;  // two groups of a pair unit fit one warp
    const uint32_t xc_s   = smem_addr(xc);
    const uint32_t xd_s   = smem_addr(xd);
    const uint32_t ring_s = smem_addr(s.ring);
    int            k0     = 0;
    for (; k0 < o.n_r && !bad; k0 += o.per_rd) {
        const int k1  = min(o.n_r, k0 + o.per_rd);
        const int nin = (pair_units ? 2 : 1) * (k1 - k0);  // tiles of this round
        auto      tile = [&](int i) { return i < k1 - k0 ? k0 + i : o.seg1 + k0 + (i - (k1 - k0)); };
        if (k0 > 0) {  // a later round of a pair op larger than the ring
            bool rbad = false;
            if (lane < nin) {
                const int ti = tile(lane);
                if (!mbar_wait_bounded(&s.full[tile_slot(o.sl0, S, ti)], tile_phase(o.sl0, o.ph0, S, ti))) {
                    raise_abort(a, s);
                    rbad = true;
                }
            }
            rbad = __any_sync(0xffffffffu, rbad);
            if (rbad) {
                bad  = true;
                fail = true;
                break;
            }
        }
        const int u_lo = pair_units ? k0 * segs[0].sr : 0;
        const int u_hi = pair_units ? min(segs[0].n, k1 * segs[0].sr) : segs[0].n;
        auto row_addr = [&](int g, int r) -> uint32_t {
            int ti = g ? o.seg1 : 0;
            while (r >= segs[g].sr) {
                r -= segs[g].sr;
                ++ti;
            }
            return ring_s + (uint32_t) (tile_slot(o.sl0, S, ti) * kStepSlotBytes) + (uint32_t) (r * segs[g].rb);
        };
        if (split) {
            // a pair op's two rows of a unit go to two neighbouring lane groups
            // (gate row: even group, up row: odd group): twice the lanes of one
            // group per unit, half the work per lane; the up row's sum joins
            // the gate row's by a shuffle before the publish
            for (int ub = u_lo + warp * (gpw >> 1); ub < u_hi; ub += ngroup >> 1) {  // warp-uniform
                const int  u      = ub + (lane >> (o.lgs + 1));
                const int  seg    = (lane >> o.lgs) & 1;
                const bool active = u < u_hi;
                float      acc0[M_T], acc1[M_T];
#pragma unroll
                for (int m = 0; m < M_T; ++m) {
                    acc0[m] = 0.0f;
                }
                if (active) {
                    // the segment's fields by select (a runtime index into segs would put it in local memory)
                    const int    sr = seg ? segs[1].sr : segs[0].sr;
                    const size_t rb = seg ? segs[1].rb : segs[0].rb;
                    int          ti = seg ? o.seg1 : 0;
                    int          r  = u;
                    while (r >= sr) {
                        r -= sr;
                        ++ti;
                    }
                    const uint32_t addr =
                        ring_s + (uint32_t) (tile_slot(o.sl0, S, ti) * kStepSlotBytes) + (uint32_t) (r * rb);
                    dot_row_half<M_T>(addr, NSB, NB, K, gl, GS, xc_s, xd_s, M, acc0);
                }
                group_reduce<M_T>(acc0, GS);
#pragma unroll
                for (int m = 0; m < M_T; ++m) {
                    acc1[m] = __shfl_down_sync(0xffffffffu, acc0[m], GS);
                }
#ifdef B200Q8_TIMELINE
                const long long tp0 = clock64();
#endif
                if (active && seg == 0 && gl == 0) {
                    publish(u, acc0, acc1);
                }
#ifdef B200Q8_TIMELINE
                __syncwarp();
                tc_pub += clock64() - tp0;
#endif
            }
        } else {
            for (int ub = u_lo + warp * gpw; ub < u_hi; ub += ngroup) {  // warp-uniform
                const int  u      = ub + (lane >> o.lgs);
                const bool active = u < u_hi;
                float      acc0[M_T], acc1[M_T];
#pragma unroll
                for (int m = 0; m < M_T; ++m) {
                    acc0[m] = 0.0f;
                    acc1[m] = 0.0f;
                }
                if (active) {
                    dot_row_half<M_T>(row_addr(0, u), NSB, NB, K, gl, GS, xc_s, xd_s, M, acc0);
                    if (pair_units) {
                        dot_row_half<M_T>(row_addr(1, u), NSB, NB, K, gl, GS, xc_s, xd_s, M, acc1);
                    }
                }
                group_reduce<M_T>(acc0, GS);
                if (pair_units) {
                    group_reduce<M_T>(acc1, GS);
                }
#ifdef B200Q8_TIMELINE
                const long long tp0 = clock64();
#endif
                if (active && gl == 0) {
                    publish(u, acc0, acc1);
                }
#ifdef B200Q8_TIMELINE
                __syncwarp();
                tc_pub += clock64() - tp0;
#endif
            }
        }
        if (k1 >= o.n_r) {
            break;  // the last round: its tiles stay held for release_tiles
        }
        // a later round follows: this round's slots go back to the producer
        // once every warp is done with them (their data was seen to land)
        __syncwarp();
        if (lane == 0) {
            for (int i = 0; i < nin; ++i) {
                mbar_arrive(&s.empty[tile_slot(o.sl0, S, tile(i))]);
            }
        }
    }
    __syncwarp();
#ifdef B200Q8_TIMELINE
    if (threadIdx.x == 0 && a.timeline != nullptr) {
        const long long tc2 = clock64();
        // [6] = tile waits, [7] = dot + reduce, packed with publish in the high half
        a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + op) * 8 + 6] = (unsigned long long) (tc1 - tc0);
        a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + op) * 8 + 7] =
            (unsigned long long) (tc2 - tc1 - tc_pub) | ((unsigned long long) tc_pub << 32);
    }
#endif
    // A slot whose copy may still be in flight must not be handed back to the
    // producer (it then times out instead, and drains before it exits): after
    // a failure nothing is released.
    if (!bad) {
        rel.a0 = k0;  // the last round's first tile of segment 0
        rel.a1 = o.n_r;
        if (pair_units) {
            rel.b0 = o.seg1 + k0;
            rel.b1 = o.nt;
        }
    }
}

// Qwen3's per-head RMS norm then NEOX RoPE for one head held by one warp:
// lane holds elements lane + 32 e (e < E), so the NEOX pair (i, i + hd/2)
// is (x[e], x[e + E/2]) of one lane.  The same arithmetic as
// qk_rope_cache_kernel (attention.cu): fp64 sum of fp32 squares, scale
// 1/sqrtf(mean + eps), (x * scale) * w, then the rotation by cs (cos and
// sin of the angles at the token's position, from rope_table).

// cos and sin of the RoPE angles of position pos, for i < hd/2: the angle
// recurrence theta_0 = pos, theta_{i+1} = theta_i * base^(-2/hd) in fp32 (as
// qk_rope_cache_kernel computes it), then cosf / sinf.  cs[i] = cos,
// cs[hd/2 + i] = sin.
__device__ __forceinline__ void rope_entry(float * cs, int hd, int i, int pos, float theta_base) {
    const float ts    = powf(theta_base, __fdiv_rn(-2.0f, (float) hd));
    float       theta = (float) pos;
    for (int k = 0; k < i; ++k) {
        theta = __fmul_rn(theta, ts);
    }
    cs[i]          = cosf(theta);
    cs[hd / 2 + i] = sinf(theta);
}
template <int E>
__device__ __forceinline__ void warp_head_norm_rope(float (&x)[E], const float * w, float eps, const float * cs,
                                                    int lane) {
    constexpr int hd = 32 * E;
    double        ss = 0.0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        ss += (double) __fmul_rn(x[e], x[e]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
    }
    const float mean  = (float) (ss / (double) hd);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
#pragma unroll
    for (int e = 0; e < E; ++e) {
        x[e] = __fmul_rn(__fmul_rn(x[e], scale), w[lane + 32 * e]);
    }
#pragma unroll
    for (int e = 0; e < E / 2; ++e) {
        const int   i  = lane + 32 * e;
        const float c  = cs[i];
        const float sn = cs[hd / 2 + i];
        const float x0 = x[e];
        const float x1 = x[e + E / 2];
        x[e]           = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        x[e + E / 2]   = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
}

// Waits for this lane's E LL words of one head (elements lane + 32 e) and
// returns their values.
template <int E>
__device__ __forceinline__ bool ll_head(const StepArgs & a, const Smem & s, const unsigned long long * base, int lane,
                                        unsigned epoch, float (&x)[E]) {
    const unsigned long long * src[E];
    unsigned long long         w[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        src[e] = base + lane + 32 * e;
        w[e]   = ld_ll(src[e]);
    }
    const bool ok = ll_settle<E>(a, s, src, w, E, epoch);
#pragma unroll
    for (int e = 0; e < E; ++e) {
        x[e] = __uint_as_float((unsigned) (w[e] & 0xffffffffu));
    }
    return ok;
}

// Waits for this lane's words of one kv head's k and v together.
template <int E>
__device__ __forceinline__ bool ll_head_kv(const StepArgs & a, const Smem & s, const unsigned long long * kbase,
                                           const unsigned long long * vbase, int lane, unsigned epoch, float (&k)[E],
                                           float (&v)[E]) {
    const unsigned long long * src[2 * E];
    unsigned long long         w[2 * E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        src[e]     = kbase + lane + 32 * e;
        src[E + e] = vbase + lane + 32 * e;
    }
#pragma unroll
    for (int i = 0; i < 2 * E; ++i) {
        w[i] = ld_ll(src[i]);
    }
    const bool ok = ll_settle<2 * E>(a, s, src, w, 2 * E, epoch);
#pragma unroll
    for (int e = 0; e < E; ++e) {
        k[e] = __uint_as_float((unsigned) (w[e] & 0xffffffffu));
        v[e] = __uint_as_float((unsigned) (w[E + e] & 0xffffffffu));
    }
    return ok;
}

// The attention of one (query head h, token m) inside the step, by this
// CTA's consumer warps (src/arch/qwen3-tts/operations.cpp:86-135): q and the
// kv head's k are RMS-normed and rotated at their positions; the token's k
// and v go to its cache row (written by the group's first query head); the
// softmax runs over cached positions 0..pos, where positions of tokens of the
// same slot in this launch come from their freshly computed rows, never from
// the cache (another CTA may still be writing them).  Per-warp online
// softmax, fixed-order merge; the head's output is published as LL words.
template <int E>
__device__ void attention_phase(const StepArgs & a, const Smem & s, int l, const unsigned long long * ll_qkv,
                                unsigned long long * ll_att, size_t qkv_dim, int h, int m, int M, unsigned epoch,
                                bool & fail) {
    constexpr int hd    = 32 * E;
    const int     warp  = threadIdx.x >> 5;
    const int     lane  = threadIdx.x & 31;
    const int     kvh   = h >> a.lg_group;
    const int     pos   = s.tok->pos[m];
    const int     slot  = s.tok->slot[m];
    const bool    ok    = s.tok->ok[m] != 0;
    float *       sq    = s.att;
    float *       kr    = sq + hd;          // [2][hd]
    float *       vr    = kr + 2 * hd;      // [2][hd]
    float *       wo    = vr + 2 * hd;      // [warps][hd]
    float *       wm    = wo + kStepConsumerWarps * hd;
    float *       wl    = wm + kStepConsumerWarps;
    const float * qn    = wl + kStepConsumerWarps;
    const float * kn    = qn + hd;
    const float * cs    = kn + hd;          // [2][hd]
    // tokens of this launch whose rows this token reads: same slot, position <= pos
    int in_m[2] = { 0, 0 }, in_pos[2] = { -1, -1 }, n_in = 0;
    for (int t = 0; t < M && ok; ++t) {
        const int pt = s.tok->pos[t];
        const int st = s.tok->slot[t];
        if (s.tok->ok[t] && st == slot && pt <= pos && n_in < 2) {
            in_m[n_in]   = t;
            in_pos[n_in] = pt;
            ++n_in;
        }
    }
    const size_t layer_rows = (size_t) a.n_cache_slots * a.n_ctx;
    const size_t cache_row0 = ((size_t) l * layer_rows + (size_t) (ok ? slot : 0) * a.n_ctx) * a.KV + (size_t) kvh * hd;
    if (!ok) {
        if (h == 0 && threadIdx.x == 0) {
            record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
        }
    } else if (warp == 0) {
        float x[E];
        if (!ll_head<E>(a, s, ll_qkv + (size_t) m * qkv_dim + (size_t) h * hd, lane, epoch, x)) {
            fail = true;
        }
        warp_head_norm_rope<E>(x, qn, a.eps, cs + m * hd, lane);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            sq[lane + 32 * e] = x[e];
        }
    } else if (warp <= n_in) {
        const int t   = in_m[warp - 1];
        float     k[E], v[E];
        const unsigned long long * row = ll_qkv + (size_t) t * qkv_dim;
        const bool good = ll_head_kv<E>(a, s, row + a.Q + (size_t) kvh * hd, row + a.Q + a.KV + (size_t) kvh * hd,
                                        lane, epoch, k, v);
        if (!good) {
            fail = true;
        }
        warp_head_norm_rope<E>(k, kn, a.eps, cs + t * hd, lane);
        const bool writer = t == m && (h & ((1 << a.lg_group) - 1)) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            kr[(warp - 1) * hd + lane + 32 * e] = k[e];
            vr[(warp - 1) * hd + lane + 32 * e] = v[e];
            if (writer && good) {
                a.k_cache[cache_row0 + (size_t) pos * a.KV + lane + 32 * e] = k[e];
                a.v_cache[cache_row0 + (size_t) pos * a.KV + lane + 32 * e] = v[e];
            }
        }
    }
    if (fail) {
        raise_abort(a, s);
    }
    if (consumers_any(fail)) {  // every consumer takes the same decision
        fail = true;
        return;
    }
    // Online softmax over this warp's positions: a group of LPP = hd/16 lanes
    // takes one position (lane gl of the group holds elements 16 gl .. 16 gl
    // + 15, read as four 16-byte words), so a warp covers 32/LPP positions per
    // round and every warp is busy even for a short prefix.
    constexpr int LPP  = hd / 16;
    constexpr int PPW  = 32 / LPP;
    const int     grp  = lane / LPP;
    const int     gl   = lane % LPP;
    const float   scale = __fdiv_rn(1.0f, sqrtf((float) hd));
    float         mx = -INFINITY, lsum = 0.0f, o[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        o[e] = 0.0f;
    }
    const int npos = ok ? pos + 1 : 0;
    float     qv[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        qv[e] = sq[16 * gl + e];
    }
    for (int base = warp * PPW; base < npos; base += kStepConsumerWarps * PPW) {  // warp-uniform
        const int  j      = base + grp;
        const bool active = j < npos;
        const float * kj;
        const float * vj;
        if (!active || j == in_pos[0]) {  // n_in >= 1 whenever npos > 0: the token's own position
            kj = kr;
            vj = vr;
        } else if (n_in > 1 && j == in_pos[1]) {
            kj = kr + hd;
            vj = vr + hd;
        } else {
            kj = a.k_cache + cache_row0 + (size_t) j * a.KV;
            vj = a.v_cache + cache_row0 + (size_t) j * a.KV;
        }
        const float4 * k4 = reinterpret_cast<const float4 *>(kj + 16 * gl);
        const float4 * v4 = reinterpret_cast<const float4 *>(vj + 16 * gl);
        float4         kk[4], vv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            kk[q] = k4[q];
            vv[q] = v4[q];
        }
        float dot = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            dot = __fmaf_rn(qv[4 * q + 0], kk[q].x, dot);
            dot = __fmaf_rn(qv[4 * q + 1], kk[q].y, dot);
            dot = __fmaf_rn(qv[4 * q + 2], kk[q].z, dot);
            dot = __fmaf_rn(qv[4 * q + 3], kk[q].w, dot);
        }
#pragma unroll
        for (int off = LPP / 2; off > 0; off >>= 1) {
            dot += __shfl_xor_sync(0xffffffffu, dot, off);
        }
        if (active) {
            const float sc = __fmul_rn(dot, scale);
            const float nm = fmaxf(mx, sc);
            const float f  = expf(mx - nm);  // 0 on the group's first position (mx = -inf)
            const float p  = expf(sc - nm);
            lsum           = __fmaf_rn(lsum, f, p);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                o[4 * q + 0] = __fmaf_rn(o[4 * q + 0], f, __fmul_rn(p, vv[q].x));
                o[4 * q + 1] = __fmaf_rn(o[4 * q + 1], f, __fmul_rn(p, vv[q].y));
                o[4 * q + 2] = __fmaf_rn(o[4 * q + 2], f, __fmul_rn(p, vv[q].z));
                o[4 * q + 3] = __fmaf_rn(o[4 * q + 3], f, __fmul_rn(p, vv[q].w));
            }
            mx = nm;
        }
    }
    // merge the warp's groups (butterfly over the lanes holding the same elements)
#pragma unroll
    for (int off = LPP; off < 32; off <<= 1) {
        const float omx = __shfl_xor_sync(0xffffffffu, mx, off);
        const float ol  = __shfl_xor_sync(0xffffffffu, lsum, off);
        const float nm  = fmaxf(mx, omx);
        const float f1  = mx == -INFINITY ? 0.0f : expf(mx - nm);
        const float f2  = omx == -INFINITY ? 0.0f : expf(omx - nm);
        lsum            = __fmaf_rn(lsum, f1, __fmul_rn(ol, f2));
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float oo = __shfl_xor_sync(0xffffffffu, o[e], off);
            o[e]           = __fmaf_rn(o[e], f1, __fmul_rn(oo, f2));
        }
        mx = nm;
    }
    if (lane == 0) {
        wm[warp] = mx;
        wl[warp] = lsum;
    }
    if (grp == 0) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            wo[warp * hd + 16 * gl + e] = o[e];
        }
    }
    named_barrier_sync(1, kStepConsumers);
    if (threadIdx.x < hd) {
        const int d  = threadIdx.x;
        float     M_ = -INFINITY;
        for (int w = 0; w < kStepConsumerWarps; ++w) {
            M_ = fmaxf(M_, wm[w]);
        }
        float L = 0.0f, acc = 0.0f;
        for (int w = 0; w < kStepConsumerWarps; ++w) {
            if (wm[w] != -INFINITY) {
                const float f = expf(wm[w] - M_);
                L             = __fmaf_rn(wl[w], f, L);
                acc           = __fmaf_rn(wo[w * hd + d], f, acc);
            }
        }
        st_ll(ll_att + (size_t) m * a.Q + (size_t) h * hd + d, npos > 0 ? __fdiv_rn(acc, L) : 0.0f, epoch);
    }
}

// ATTN: the reference's attention over the KV cache (a.attn), else the
// single cached position; a compile-time switch so the benchmark step's
// kernel carries none of the attention code.
template <int M_T, int MODE, bool ATTN>
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
    s.rms_part    = reinterpret_cast<double *>(smem + 1024);
    s.tok         = reinterpret_cast<AttTok *>(smem + 1024 + 8 * kStepConsumerWarps * 8);
    size_t off    = kStepHeader;
    s.hbuf        = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * H * 4;
    s.h1buf = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * H * 4;
    s.normbuf = reinterpret_cast<float *>(smem + off);
    off += (size_t) H * 4;
    s.ybuf = reinterpret_cast<float *>(smem + off);
    off += (size_t) M_T * 2 * kStepYMax * 4;
    for (int i = 0; i < 2; ++i) {
        s.xc[i] = smem + off;
        off += (size_t) M_T * Kmax;
        s.xd[i] = reinterpret_cast<float *>(smem + off);
        off += (size_t) M_T * (Kmax / kQK) * 4;
    }
    s.att = reinterpret_cast<float *>(smem + off);
    if (ATTN) {
        off += att_scratch_floats(a.head_dim) * 4;
    }
    off    = (off + 127) & ~(size_t) 127;
    s.ring  = smem + off;
    s.inv_h = (H & (H - 1)) == 0 ? 1.0 / (double) H : 0.0;
    const int S = a.n_slots;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStepMaxSlots; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kStepConsumerWarps);
        }
        *s.abort_local = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int      warp  = threadIdx.x >> 5;
    const int      lane  = threadIdx.x & 31;
    const Plan     plan  = make_plan(a, c, G);

    if (warp == kStepConsumerWarps) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol     = l2_evict_first_policy();
            int            t       = 0;  // tiles issued
            int            sl      = 0;  // slot of tile t
            uint32_t       ph      = 0;  // fill round of slot sl, mod 2
            bool           stop    = false;
            for (int l = 0; l <= a.n_layers && !stop; ++l) {
                Seg segs[5];
                int nsegs = 5;
                if (l < a.n_layers) {
                    layer_segs(a, plan, l, segs);
                } else if (a.head != nullptr) {  // the output head after the last layer
                    segs[0] = head_seg(a, plan, c, G);
                    nsegs   = 1;
                } else {
                    break;
                }
                for (int g = 0; g < nsegs && !stop; ++g) {
#ifdef B200Q8_TIMELINE
                    if (a.timeline != nullptr && g != 3 && l < a.n_layers) {
                        unsigned long long gt;
                        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt));
                        a.timeline[((size_t) blockIdx.x * (4 * a.n_layers) + 4 * l + (g < 3 ? g : 3)) * 8 + 5] = gt;
                    }
#endif
                    for (int r = 0; r < segs[g].n; r += segs[g].sr) {
                        // slot sl was last filled in round ph^1: wait until it was released
                        // (or the consumers stopped, which they signal through abort_local)
                        if (t >= S && !mbar_wait_bounded_or_flag(&s.empty[sl], ph ^ 1u, s.abort_local)) {
                            if (*(volatile int *) s.abort_local == 0) {
                                raise_abort(a, s);
                            }
                            stop = true;
                            break;
                        }
                        if (*(volatile int *) s.abort_local != 0) {
                            stop = true;
                            break;
                        }
                        const int      R     = min(segs[g].sr, segs[g].n - r);
                        const uint32_t bytes = (uint32_t) ((size_t) R * segs[g].rb);
                        mbar_arrive_expect_tx(&s.full[sl], bytes);
                        bulk_copy_g2s(s.ring + (size_t) sl * kStepSlotBytes, segs[g].base + (size_t) r * segs[g].rb,
                                      bytes, &s.full[sl], pol);
                        ++t;
                        if (++sl == S) {
                            sl = 0;
                            ph ^= 1u;
                        }
                    }
                }
            }
            // never leave with a copy in flight into this CTA's shared memory
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
    if (t_id == 0) {
        // launch k (1-based) of this plan: every CTA computes the same k.  Taken
        // here, not before the CTA barrier above, so that the producer's first
        // copies do not wait for the atomic's round trip; the consumers read it
        // after their barrier below, and the producer only on a timeout.
        *s.epoch = atomicAdd(&a.sync[0], 1u) / (unsigned) G + 1u;
    }
    // step input: h = x_in + get_rows(table, ids), every CTA for itself
    // (either term may be absent: ids == nullptr or x_in == nullptr)
    for (int m = 0; m < M; ++m) {
        const int64_t r     = a.ids != nullptr ? a.ids[m] : -1;
        const bool    in_tb = r >= 0 && r < a.table_rows;
        if (a.ids != nullptr && !in_tb && c == 0 && t_id == 0) {
            record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
        }
        for (int k = t_id; k < H; k += kStepConsumers) {
            float ev = 0.0f;
            if (in_tb) {
                const uint8_t * blk = a.table + r * a.rb_h + (k >> 5) * kBlockBytes;
                const float     d   = __half2float(__ushort_as_half((unsigned short) (blk[0] | (blk[1] << 8))));
                ev                  = __fmul_rn((float) (int8_t) blk[2 + (k & 31)], d);
            }
            s.hbuf[m * H + k] = a.ids == nullptr  ? a.x_in[(size_t) m * H + k]
                                : a.x_in == nullptr ? ev
                                                    : __fadd_rn(a.x_in[(size_t) m * H + k], ev);
        }
    }
    // attention: the tokens' positions and slots, and (attention CTAs) the
    // RoPE cos / sin at each token's position, once per launch
    const bool att_cta = ATTN && c < (a.Q >> a.lg_head_dim) * M;
    if (ATTN) {
        if (t_id < 2) {
            int p = 0, sl = 0, okv = 0;
            if (t_id < M) {
                p   = a.pos[t_id];
                sl  = a.slots ? a.slots[t_id] : t_id;
                okv = p >= 0 && p < a.n_ctx && sl >= 0 && sl < a.n_cache_slots;
            }
            s.tok->pos[t_id]  = p;
            s.tok->slot[t_id] = sl;
            s.tok->ok[t_id]   = okv;
        }
        if (att_cta) {
            const int hd = a.head_dim;
            for (int idx = t_id; idx < M * (hd / 2); idx += kStepConsumers) {
                const int m = idx / (hd / 2);
                const int p = a.pos[m];
                rope_entry(s.att + att_rope_offset(hd) + (size_t) m * hd, hd, idx % (hd / 2),
                           p >= 0 && p < a.n_ctx ? p : 0, a.rope_theta);
            }
        }
    }
    named_barrier_sync(1, kStepConsumers);
    const unsigned epoch = *s.epoch;

    const int qkv_dim = a.Q + 2 * a.KV;
    int       sl      = 0;      // slot of the next tile, mirrors the producer
    uint32_t  ph      = 0;      // its fill round mod 2
    bool      fail    = false;  // this thread saw a timeout or an abort
    auto trace = [&](int l, int which) -> float * {
        return a.trace ? a.trace + (size_t) l * a.trace_layer + a.trace_off[which] : nullptr;
    };
    const size_t llm = (size_t) a.ll_m;  // token stride of the LL buffers
    const Part   pq  = plan.pq;
    const Part   po  = plan.ph;
    const Part   pg  = plan.pi;
    bool         stopped = false;
    Release      rel;      // the slots the last op still holds

    for (int l = 0; l < a.n_layers; ++l) {
        const StepLayerDev &       L    = a.layers[l];
        unsigned long long * const ll_qkv = a.ll + (size_t) l * a.ll_layer;
        unsigned long long * const ll_att = ll_qkv + llm * qkv_dim;
        unsigned long long * const ll_o   = ll_att + llm * a.Q;
        unsigned long long * const ll_s   = ll_o + llm * a.H;
        unsigned long long * const ll_d   = ll_s + llm * a.I;
        Seg                        segs[5];
        layer_segs(a, plan, l, segs);
        // attention CTAs: this layer's q_norm | k_norm (2 * head_dim <= 512
        // values), loaded now and stored to shared memory after the qkv op, so
        // that no thread stalls on the loads
        float qkn[2] = { 0.0f, 0.0f };
        if (ATTN && att_cta) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int i = t_id + k * kStepConsumers;
                if (i < 2 * a.head_dim) {
                    qkn[k] = i < a.head_dim ? L.q_norm[i] : L.k_norm[i - a.head_dim];
                }
            }
        }

        // Staged activations alternate between two buffers op by op.
        float no_scale[M_T];
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
            no_scale[m] = 1.0f;
        }
        float scale[M_T];
        // ---- qkv = W_qkv * Q(rms_norm(h) * norm_in), h = h1 + d(l-1); v published
        TL(4 * l + 0, 0);
        const unsigned long long * prev_d =
            l > 0 ? a.ll + (size_t) (l - 1) * a.ll_layer + llm * (qkv_dim + a.Q + a.H + a.I) : nullptr;
        const OpRun o_qkv = plan_op(a, s, S, sl, ph, &segs[0], 1, false, H, lane, fail);
        residual_and_rms<M_T>(a, s, prev_d, s.h1buf, s.hbuf, M, epoch, (l > 0 && c == 0) ? trace(l - 1, 9) : nullptr,
                              L.norm_in, fail, scale);
        TL(4 * l + 0, 1);
        if (stage_activations<M_T, MODE>(a, s, H, M, 0, s.hbuf, s.normbuf, scale, nullptr, 0, false, epoch,
                                         c == 0 ? trace(l, 0) : nullptr, (size_t) H, s.xc[0], s.xd[0], fail)) {
            stop_producer(s);
            stopped = true;
            break;
        }
        TL(4 * l + 0, 2);
        {
            float * tq = trace(l, 1);
            consume_op<M_T>(a, s, S, o_qkv, &segs[0], false, H, M, warp, lane, s.xc[0], s.xd[0], fail, 4 * l + 0, rel,
                            [&](int u, const float (&y)[M_T], const float (&)[M_T]) {
                                const int row = pq.r0 + u;
#pragma unroll
                                for (int m = 0; m < M_T; ++m) {
                                    if (m < M) {
                                        if (ATTN || row >= a.Q + a.KV) {
                                            st_ll(ll_qkv + (size_t) m * qkv_dim + row, y[m], epoch);
                                        }
                                        if (tq) {
                                            tq[(size_t) m * qkv_dim + row] = y[m];
                                        }
                                    }
                                }
                            });
        }
        TL(4 * l + 0, 3);
        if (ATTN && att_cta) {  // read by the attention phase, after the barrier below
            float * qk = s.att + att_norm_offset(a.head_dim);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int i = t_id + k * kStepConsumers;
                if (i < 2 * a.head_dim) {
                    qk[i] = qkn[k];
                }
            }
        }
        // park warps that are done until the whole op is: a warp polling the
        // next op's inputs would steal issue slots from warps still computing
        if (consumers_any(fail || local_stop(s))) {
            stop_producer(s);
            stopped = true;
            break;
        }
        release_tiles(s, S, rel);
        // ---- attention: one CTA per (query head, token) publishes the head's output
        if (ATTN) {
            const int n_head = a.Q >> a.lg_head_dim;
            if (c < n_head * M) {
                TL(4 * l + 1, 4);
                const int hh = c % n_head, mm = c / n_head;
                switch (a.head_dim) {
                    case 64: attention_phase<2>(a, s, l, ll_qkv, ll_att, qkv_dim, hh, mm, M, epoch, fail); break;
                    case 128: attention_phase<4>(a, s, l, ll_qkv, ll_att, qkv_dim, hh, mm, M, epoch, fail); break;
                    default: attention_phase<8>(a, s, l, ll_qkv, ll_att, qkv_dim, hh, mm, M, epoch, fail); break;
                }
                if (consumers_any(fail || local_stop(s))) {
                    stop_producer(s);
                    stopped = true;
                    break;
                }
                TL(4 * l + 1, 1);
            }
        }
        // ---- o = W_o * Q(attend); attention over the cache, or over one cached position; o published
        TL(4 * l + 1, 0);
        const unsigned long long * o_src = ATTN ? ll_att : ll_qkv + a.Q + a.KV;
        const OpRun o_o = plan_op(a, s, S, sl, ph, &segs[1], 1, false, a.Q, lane, fail);
        if (stage_activations<M_T, MODE>(a, s, a.Q, M, 1, nullptr, nullptr, no_scale, o_src,
                                         ATTN ? (size_t) a.Q : (size_t) qkv_dim, !ATTN, epoch,
                                         c == 0 ? trace(l, 2) : nullptr, (size_t) a.Q, s.xc[1], s.xd[1], fail)) {
            stop_producer(s);
            stopped = true;
            break;
        }
        TL(4 * l + 1, 2);
        {
            float * to = trace(l, 3);
            consume_op<M_T>(a, s, S, o_o, &segs[1], false, a.Q, M, warp, lane, s.xc[1], s.xd[1], fail, 4 * l + 1, rel,
                            [&](int u, const float (&y)[M_T], const float (&)[M_T]) {
#pragma unroll
                                for (int m = 0; m < M_T; ++m) {
                                    if (m < M) {
                                        st_ll(ll_o + (size_t) m * a.H + po.r0 + u, y[m], epoch);
                                        if (to) {
                                            to[(size_t) m * a.H + po.r0 + u] = y[m];
                                        }
                                    }
                                }
                            });
        }
        TL(4 * l + 1, 3);
        // park warps that are done until the whole op is: a warp polling the
        // next op's inputs would steal issue slots from warps still computing
        if (consumers_any(fail || local_stop(s))) {
            stop_producer(s);
            stopped = true;
            break;
        }
        release_tiles(s, S, rel);
        // ---- g|u = W_gate|W_up * Q(rms_norm(h1) * norm_post), h1 = h + o; s = silu(g)*u published
        TL(4 * l + 2, 0);
        const OpRun o_gu = plan_op(a, s, S, sl, ph, &segs[2], 2, true, H, lane, fail);
        residual_and_rms<M_T>(a, s, ll_o, s.hbuf, s.h1buf, M, epoch, c == 0 ? trace(l, 4) : nullptr, L.norm_post,
                              fail, scale);
        TL(4 * l + 2, 1);
        if (stage_activations<M_T, MODE>(a, s, H, M, 0, s.h1buf, s.normbuf, scale, nullptr, 0, false, epoch,
                                         c == 0 ? trace(l, 5) : nullptr, (size_t) H, s.xc[0], s.xd[0], fail)) {
            stop_producer(s);
            stopped = true;
            break;
        }
        TL(4 * l + 2, 2);
        {
            float * tgu = trace(l, 6);
            float * ts  = trace(l, 7);
            consume_op<M_T>(a, s, S, o_gu, &segs[2], true, H, M, warp, lane, s.xc[0], s.xd[0], fail, 4 * l + 2, rel,
                            [&](int u, const float (&g)[M_T], const float (&up)[M_T]) {
#pragma unroll
                                for (int m = 0; m < M_T; ++m) {
                                    if (m < M) {
                                        const float sv = __fmul_rn(silu_f32(g[m]), up[m]);
                                        st_ll(ll_s + (size_t) m * a.I + pg.r0 + u, sv, epoch);
                                        if (tgu) {
                                            tgu[(size_t) m * 2 * a.I + pg.r0 + u]       = g[m];
                                            tgu[(size_t) m * 2 * a.I + a.I + pg.r0 + u] = up[m];
                                        }
                                        if (ts) {
                                            ts[(size_t) m * a.I + pg.r0 + u] = sv;
                                        }
                                    }
                                }
                            });
        }
        TL(4 * l + 2, 3);
        // park warps that are done until the whole op is: a warp polling the
        // next op's inputs would steal issue slots from warps still computing
        if (consumers_any(fail || local_stop(s))) {
            stop_producer(s);
            stopped = true;
            break;
        }
        release_tiles(s, S, rel);
        // ---- d = W_down * Q(s); d published (the last layer writes h_out = h1 + d)
        TL(4 * l + 3, 0);
        const OpRun o_d = plan_op(a, s, S, sl, ph, &segs[4], 1, false, a.I, lane, fail);
        if (stage_activations<M_T, MODE>(a, s, a.I, M, 1, nullptr, nullptr, no_scale, ll_s, (size_t) a.I, false,
                                         epoch, nullptr, 0, s.xc[1], s.xd[1], fail)) {
            stop_producer(s);
            stopped = true;
            break;
        }
        TL(4 * l + 3, 2);
        {
            float *    td   = trace(l, 8);
            const bool last = l == a.n_layers - 1;
            consume_op<M_T>(a, s, S, o_d, &segs[4], false, a.I, M, warp, lane, s.xc[1], s.xd[1], fail, 4 * l + 3, rel,
                            [&](int u, const float (&y)[M_T], const float (&)[M_T]) {
                                const int row = po.r0 + u;
#pragma unroll
                                for (int m = 0; m < M_T; ++m) {
                                    if (m < M) {
                                        if (last && a.head == nullptr) {
                                            a.h_out[(size_t) m * H + row] = __fadd_rn(s.h1buf[m * H + row], y[m]);
                                        } else {
                                            st_ll(ll_d + (size_t) m * a.H + row, y[m], epoch);
                                        }
                                        if (td) {
                                            td[(size_t) m * a.H + row] = y[m];
                                        }
                                    }
                                }
                            });
        }
        TL(4 * l + 3, 3);
        // park warps that are done until the whole op is: a warp polling the
        // next op's inputs would steal issue slots from warps still computing
        if (consumers_any(fail || local_stop(s))) {
            stop_producer(s);
            stopped = true;
            break;
        }
        release_tiles(s, S, rel);
    }
    if (stopped || fail || a.head == nullptr) {
        return;
    }
    // ---- output: h = h1 + d (CTA 0 writes h_out), hidden = rms_norm(h) * out_norm
    // (CTA 0 writes hidden_out), logits = head * Q(hidden)
    {
        const unsigned long long * last_d =
            a.ll + (size_t) (a.n_layers - 1) * a.ll_layer + llm * (qkv_dim + a.Q + a.H + a.I);
        float      scale[M_T];
        const Seg  hs     = head_seg(a, plan, c, G);
        const Part pv     = part(a.vocab, G, c);
        const OpRun o_h   = plan_op(a, s, S, sl, ph, &hs, 1, false, H, lane, fail);
        residual_and_rms<M_T>(a, s, last_d, s.h1buf, s.hbuf, M, epoch, c == 0 ? a.h_out : nullptr, a.out_norm, fail,
                              scale);
        if (stage_activations<M_T, MODE>(a, s, H, M, 0, s.hbuf, s.normbuf, scale, nullptr, 0, false, epoch,
                                         c == 0 ? a.hidden_out : nullptr, (size_t) H, s.xc[0], s.xd[0], fail)) {
            stop_producer(s);
            return;
        }
        consume_op<M_T>(a, s, S, o_h, &hs, false, H, M, warp, lane, s.xc[0], s.xd[0], fail, 0, rel,
                        [&](int u, const float (&y)[M_T], const float (&)[M_T]) {
#pragma unroll
                            for (int m = 0; m < M_T; ++m) {
                                if (m < M) {
                                    a.logits[(size_t) m * a.vocab + pv.r0 + u] = y[m];
                                }
                            }
                        });
        if (consumers_any(fail || local_stop(s))) {
            stop_producer(s);
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
    off += 2 * (size_t) mt * Kmax;
    off += 2 * (size_t) mt * (Kmax / kQK) * 4;
    if (a.attn) {
        off += att_scratch_floats(a.head_dim) * 4;
    }
    off                   = (off + 127) & ~(size_t) 127;
    const size_t limit    = 227 * 1024;
    if (off + kStepSlotBytes * 2 > limit) {
        n_slots = 0;
        return 0;
    }
    n_slots = (int) std::min<size_t>(kStepMaxSlots, (limit - off) / kStepSlotBytes);
    return off + (size_t) n_slots * kStepSlotBytes;
}

// Token slots of the kernel instance that runs M tokens (1 or 2).
int step_mt(int M) {
    return M <= 1 ? 1 : 2;
}

bool decode_step_supported(const StepArgs & a, int G) {
    if (a.M < 1 || a.M > kStepMaxM || a.M > a.ll_m || a.H % 256 || a.Q % 256 || a.I % 256 || a.KV % 32) {
        return false;
    }
    if ((1 << a.lg_head_dim) != a.head_dim || (1 << a.lg_group) != a.group) {
        return false;  // the GQA expansion uses shifts
    }
    // every CTA's slice of one op must fit the output staging buffer
    const int qkv = a.Q + 2 * a.KV;
    if ((qkv + G - 1) / G > 2 * kStepYMax || (a.I + G - 1) / G > kStepYMax || (a.H + G - 1) / G > kStepYMax) {
        return false;
    }
    if (a.rb_i > (size_t) kStepSlotBytes || a.rb_q > (size_t) kStepSlotBytes || a.rb_h > (size_t) kStepSlotBytes) {
        return false;
    }
    // attention: one CTA per (query head, token); a warp holds a head in
    // lanes of head_dim/32 elements whose NEOX pairs stay in one lane, and
    // head_dim/16 lanes share a cached position (head_dim 64, 128 or 256)
    if (a.attn && ((a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) || (a.Q / a.head_dim) * a.M > G ||
                   a.pos == nullptr || a.k_cache == nullptr || a.v_cache == nullptr || !(a.rope_theta > 0.0f))) {
        return false;
    }
    if (a.head != nullptr && (a.vocab < 1 || (a.vocab + G - 1) / G > kStepYMax || a.logits == nullptr ||
                              a.hidden_out == nullptr || a.out_norm == nullptr)) {
        return false;
    }
    int slots = 0;
    if (decode_step_smem_bytes(a, step_mt(a.M), slots) == 0 || slots < 2) {
        return false;
    }
    // consume_op holds all tiles of one op at once: they must fit the ring
    auto tiles = [&](int rows_total, size_t rb) {
        const int rows = (rows_total + G - 1) / G;
        const int sr   = std::max(1, (int) (kStepSlotBytes / rb));
        return (rows + sr - 1) / sr;
    };
    // (the gate/up pair op is consumed in rounds: it needs one slot more than
    // its tiles per segment, and both segments' tiles within consume_op's table)
    const int worst = std::max(std::max(tiles(qkv, a.rb_h), tiles(a.H, a.rb_q)),
                               std::max(tiles(a.H, a.rb_i), a.head != nullptr ? tiles(a.vocab, a.rb_h) : 0));
    const int gu    = tiles(a.I, a.rb_h);
    return worst <= std::min(slots, 16) && gu + 1 <= slots && 2 * gu <= 16;
}

namespace {
using StepFn = void (*)(const StepArgs);

template <int MODE>
StepFn pick_step_kernel_m(int mt, bool attn) {
    if (attn) {
        return mt == 1 ? decode_step_kernel<1, MODE, true> : decode_step_kernel<2, MODE, true>;
    }
    return mt == 1 ? decode_step_kernel<1, MODE, false> : decode_step_kernel<2, MODE, false>;
}

StepFn pick_step_kernel(int mode, int mt, bool attn) {
    switch (mode) {
        case B200Q8_QUANT_CPU_X86: return pick_step_kernel_m<B200Q8_QUANT_CPU_X86>(mt, attn);
        case B200Q8_QUANT_CPU_ARM: return pick_step_kernel_m<B200Q8_QUANT_CPU_ARM>(mt, attn);
        default: return pick_step_kernel_m<B200Q8_QUANT_REF>(mt, attn);
    }
}
}  // namespace

// The largest M (0, 1 or 2) up to which one CTA of the step kernel fits on an
// SM with its shared memory (the cooperative launch needs every CTA resident
// at once).
int decode_step_max_m(const StepArgs & a) {
    int best = 0;
    for (int mt = 1; mt <= kStepMaxM; mt *= 2) {
        int          slots = 0;
        const size_t smem  = decode_step_smem_bytes(a, mt, slots);
        StepFn       fn    = pick_step_kernel(a.mode, mt, a.attn != 0);
        if (smem == 0 || slots < 2 ||
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess) {
            cudaGetLastError();
            break;
        }
        int blocks = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, kStepThreads, smem) != cudaSuccess || blocks < 1) {
            cudaGetLastError();
            break;
        }
        best = mt;
    }
    return best;
}

cudaError_t launch_decode_step(StepArgs a, int G, cudaStream_t stream) {
    const int mt   = step_mt(a.M);
    int       slots = 0;
    const size_t smem = decode_step_smem_bytes(a, mt, slots);
    a.n_slots         = slots;
    StepFn fn = pick_step_kernel(a.mode, mt, a.attn != 0);
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
    e                      = cudaLaunchKernelEx(&cfg, fn, a);
    if (e != cudaSuccess) {
        cudaGetLastError();  // a failed launch must not surface in the caller's next check
    }
    return e;
}

}  // namespace b200q8
