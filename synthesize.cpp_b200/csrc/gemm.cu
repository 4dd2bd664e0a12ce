// gemm.cu -- Q8_0 x F32 MUL_MAT for M > 8 tokens on int8 tensor cores (sm_100a).
//
// y[m][n] = sum_b fp32(dw[n,b]) * fp32(dx[m,b]) * sum_{i<32} qw[n,32b+i] * qx[m,32b+i]
//
// One Q8_0 block is exactly the K = 32 of one mma.sync.m16n8k32 s8 x s8 -> s32,
// so each MMA yields the exact int32 block sums of a 16-row x 8-token tile.
// The scale differs per block, so every block sum is rescaled in fp32: the
// MMA accumulates onto the bias 0x4B400000 (the float 1.5 * 2^23), which turns
// the int32 result into a float bit pattern (|sum| <= 32*128*128 < 2^22), and
// the rescale is three packed f32x2 instructions per pair of outputs -- no
// int->float conversions.
//
// Activations are quantized once per call ("staged") into records of one
// 256-wide K chunk for a chunk of tm tokens: tm rows of 256 code bytes whose
// 16-byte units are XOR-swizzled by token, then the chunk's 8 x tm fp32
// scales.  A CTA works on units of (token chunk, RB weight rows, all of K):
// each 256-wide K chunk of the unit's weight rows (one 2-D tiled TMA load of
// a 272-byte x RB-row box through a tensor map over the standard Q8_0 rows)
// and the matching activation record (one 1-D bulk copy) land in one
// shared-memory slot of a ring, so weights and activations stream together
// and every byte is loaded once per unit.  Eight consumer warps
// split the unit into 16-row tiles x block subsets of the chunk; partial sums
// over K are combined through shared memory in a fixed order, so results are
// deterministic.  When the units of a small-M call leave SMs idle, and the
// caller gives room for it, a unit takes only a range of the K chunks
// (split-K): its partial sums go through L2 and the last of a block's splits
// to finish adds them in split order, again independent of arrival order.
// Copies are never multicast.
#include "common.cuh"
#include "kernels.h"
#include "mma_tile.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

namespace b200q8 {
namespace {

constexpr int   kGemmConsumerWarps = 8;
constexpr int   kGemmThreads       = (kGemmConsumerWarps + 1) * 32;
constexpr int   kGemmMaxSlots      = 6;
constexpr int   kGemmSmemLimit     = 224 * 1024;
constexpr int   kChunkBlocks       = 8;                           // Q8_0 blocks per K chunk
constexpr int   kChunkRowBytes     = kChunkBlocks * kBlockBytes;  // 272: one weight row of a chunk
constexpr int   kRecTokenBytes     = kChunkBlocks * kQK + kChunkBlocks * 4;  // 288: codes + scales
constexpr int   kMaxTokenChunk     = 64;
constexpr int   kGemmMaxM          = 65536;  // tokens per call (chunks of <= 64)
constexpr int   kGemmSplitMaxTG    = 2;      // split-K only for token chunks of <= 16

// 2-D tiled TMA load of the box at (x, y) of `map` into this CTA's shared
// memory (128-byte aligned), completing on `bar`.  x counts 2-byte elements
// and is a multiple of 8 (16-byte aligned); rows past the tensor read as 0.
// Never multicast.
__device__ __forceinline__ void tma_load_2d(void * dst_smem, const CUtensorMap * map, int x, int y, uint64_t * bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst_smem)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Byte offset of code byte i (0..31) of block j (0..7) of token t inside a
// record: 16-byte unit (2j + i/16) is XOR-swizzled by 2*(t % 8), so the eight
// tokens a B-fragment load touches fall in eight different bank groups.
__host__ __device__ __forceinline__ int rec_code_offset(int t, int j, int i) {
    const int unit = (2 * j + (i >> 4)) ^ ((t & 7) << 1);
    return t * (kChunkBlocks * kQK) + unit * 16 + (i & 15);
}


#ifdef B200Q8_TIMELINE
// Analysis builds only: globaltimer stamps per (launch slot, CTA, event) of
// the GEMM and stage kernels; slots are assigned on the host at launch (or
// capture) time.
constexpr int kTlSlots = 256, kTlCtas = 256;
__device__ unsigned long long g_tl[kTlSlots * kTlCtas * 8];
__device__ __forceinline__ void tl_stamp(int slot, int ev) {
    unsigned long long g;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g));
    if (slot >= 0 && slot < kTlSlots && blockIdx.x < kTlCtas) {
        g_tl[((size_t) slot * kTlCtas + blockIdx.x) * 8 + ev] = g;
    }
}
static int  g_tl_next = 0;
static char g_tl_kind[kTlSlots];
int tl_take(char kind) {
    const int s = g_tl_next++;
    if (s < kTlSlots) {
        g_tl_kind[s] = kind;
    }
    return s;
}
#define GTL(ev) tl_stamp(a.tl_slot, ev)
#else
#define GTL(ev) ((void) 0)
#endif

struct GemmArgs {
    const uint8_t * w;
    size_t          row_bytes;
    int             K, N, M;
    const uint8_t * xrec;  // staged activations
    float *         y;
    size_t          y_stride;  // floats between tokens
    int             tm;        // tokens per chunk (multiple of 8, <= 64)
    int             n_tc;      // token chunks
    int             rb;        // weight rows per unit (16, 32, 64 or 128)
    int             n_rb;      // row blocks = ceil(N / rb)
    int             n_units;   // n_tc * n_rb * ksplit
    int             n_slots;
    int             tl_slot;   // timeline builds only
    // split-K (ksplit > 1): unit u takes K chunks [kz * kc_n, (kz + 1) * kc_n)
    // of its rows and tokens; partial sums go to part [ksplit][M][N], and the
    // last of a (tokens, rows) block's ksplit units to finish (counted in
    // cnt[tc * n_rb + rb], which it sets back to 0) adds the partials in split
    // order 0, 1, ... and writes y, so results do not depend on arrival order.
    int             ksplit;
    int             kc_n;      // K chunks per unit
    float *         part;
    unsigned *      cnt;
};

// TG: token groups of 8 in a token chunk (tm = 8 * TG); SPLITK: the
// instance can split K (it does when a.ksplit > 1).  Only the small token
// chunks that use split-K carry its code.
template <int TG, bool SPLITK>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_q8_0_kernel(const GemmArgs a, const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *     full       = reinterpret_cast<uint64_t *>(smem);
    uint64_t *     empty      = full + kGemmMaxSlots;
    volatile int * abort_flag = reinterpret_cast<volatile int *>(smem + 2 * kGemmMaxSlots * 8);
    float *        red        = reinterpret_cast<float *>(smem + 128);  // K-subset partials
    const int      red_bytes  = kGemmConsumerWarps * 32 * TG * 4 * 4;
    uint8_t *      ring       = smem + 128 + red_bytes;

    const int    warp      = threadIdx.x >> 5;
    const int    lane      = threadIdx.x & 31;
    const int    n_kc      = a.K >> 8;
    const int    S         = a.n_slots;
    const int    w_bytes   = a.rb * kChunkRowBytes;
    const int    slot      = w_bytes + a.tm * kRecTokenBytes;
    const int    rec_bytes = a.tm * kRecTokenBytes;
    const int    G         = gridDim.x;

    if (threadIdx.x == 0) {
        GTL(0);
        for (int i = 0; i < kGemmMaxSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kGemmConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kGemmConsumerWarps) {
        // Producer warp (lane 0 issues): weights are constant, so the first
        // S slots' weights stream before the wait on the kernel that wrote
        // the activations.
        const uint64_t wpol     = a.n_tc == 1 ? l2_evict_first_policy() : l2_evict_last_policy();
        const uint64_t xpol     = l2_evict_last_policy();
        const int      my_units = (a.n_units - (int) blockIdx.x + G - 1) / G;
        const int      kc_n     = SPLITK ? a.kc_n : n_kc;
        const int      total    = my_units * kc_n;
        // fill i = the (i % kc_n)-th chunk of the CTA's unit i / kc_n; it uses slot i % S
        auto issue_w = [&](int i, int si) {
            const int ui = i / kc_n;
            const int u  = (int) blockIdx.x + ui * G;
            const int kz = SPLITK ? u / (a.n_tc * a.n_rb) : 0;
            const int ut = u - kz * (a.n_tc * a.n_rb);
            const int kc = kz * kc_n + (i - ui * kc_n);
            const int tc = ut / a.n_rb;
            const int r0 = (ut - tc * a.n_rb) * a.rb;
            if (lane == 0) {
                // the box counts in full, rows past N included (they read as 0)
                mbar_arrive_expect_tx(&full[si], (uint32_t) (w_bytes + rec_bytes));
                tma_load_2d(ring + (size_t) si * slot, &wmap, kc * (kChunkRowBytes / 2), r0, &full[si], wpol);
            }
        };
        auto issue_x = [&](int i, int si) {
            const int ui = i / kc_n;
            const int u  = (int) blockIdx.x + ui * G;
            const int kz = SPLITK ? u / (a.n_tc * a.n_rb) : 0;
            const int kc = kz * kc_n + (i - ui * kc_n);
            const int tc = (u - kz * (a.n_tc * a.n_rb)) / a.n_rb;
            if (lane == 0) {
                bulk_copy_g2s(ring + (size_t) si * slot + w_bytes, a.xrec + ((size_t) tc * n_kc + kc) * rec_bytes,
                              (uint32_t) rec_bytes, &full[si], xpol);
            }
        };
        // Weights are constant: the first S fills' weights stream before the
        // wait on the kernel that wrote the activations.
        const int pre = min(S, total);
        for (int i = 0; i < pre; ++i) {
            issue_w(i, i);
        }
        if (lane == 0) GTL(1);
        pdl_wait_primary();
        if (lane == 0) GTL(2);
        for (int i = 0; i < pre; ++i) {
            issue_x(i, i);
        }
        int      s     = pre == S ? 0 : pre;
        uint32_t ph    = pre == S ? 1 : 0;
        int      fills = pre;
        for (int i = pre; i < total; ++i) {
            bool ok = true;
            if (lane == 0) {
                // gives up early when a consumer already failed (abort_flag)
                ok = mbar_wait_bounded_or_flag(&empty[s], ph ^ 1, const_cast<const int *>(abort_flag));
                if (!ok) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                    *abort_flag = 1;
                }
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
                break;
            }
            issue_w(i, s);
            issue_x(i, s);
            ++fills;
            if (++s == S) {
                s = 0;
                ph ^= 1;
            }
        }
        // never leave with copies in flight: wait for the last S fills
        if (lane == 0) {
            int      ws  = s;
            uint32_t wph = ph;
            for (int i = 0; i < min(fills, S); ++i) {
                if (--ws < 0) {
                    ws = S - 1;
                    wph ^= 1;
                }
                if (!mbar_wait_bounded(&full[ws], wph)) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                }
            }
            GTL(6);
        }
        return;
    }

    // consumer roles: 16-row tile rt of the unit, block subset ks of each chunk
    const int rt_n = a.rb >> 4;
    const int ks_n = kChunkBlocks / rt_n;  // 8 warps = rt_n row tiles x ks_n block subsets
    const int rt   = warp % rt_n;
    const int ks   = warp / rt_n;
    const int j0   = ks * rt_n;            // this warp's blocks of each chunk: j0 .. j0 + rt_n - 1
    const int j1   = j0 + rt_n;
    const int g    = lane >> 2;
    const int tq   = lane & 3;
    const float2 nbias    = make_float2(-kMmaBiasF, -kMmaBiasF);
    const int    cbias[4] = { kMmaBias, kMmaBias, kMmaBias, kMmaBias };
    float4 *     red4  = reinterpret_cast<float4 *>(red);

    int      s    = 0;
    uint32_t ph   = 0;
    bool     fail = false;
    // Every consumer warp runs the same trip counts and reaches the same
    // barriers whatever happens; a failed wait only skips work.
    // split-K: set when this CTA finished a block's last split
    volatile unsigned * last_s = reinterpret_cast<volatile unsigned *>(smem + 2 * kGemmMaxSlots * 8 + 4);
    const int           kc_n   = SPLITK ? a.kc_n : n_kc;
    const bool          split  = SPLITK && a.ksplit > 1;
    for (int u = blockIdx.x; u < a.n_units; u += G) {
        const int kz   = SPLITK ? u / (a.n_tc * a.n_rb) : 0;
        const int ut   = u - kz * (a.n_tc * a.n_rb);
        const int tc   = ut / a.n_rb;
        const int r0   = (ut - tc * a.n_rb) * a.rb;
        const int rows = min(a.rb, a.N - r0);
        const int tok0 = tc * a.tm;
        float2    acc[TG][2];
#pragma unroll
        for (int i = 0; i < TG; ++i) {
            acc[i][0] = make_float2(0.0f, 0.0f);
            acc[i][1] = make_float2(0.0f, 0.0f);
        }
        for (int kc = 0; kc < kc_n; ++kc) {
            if (!fail && !mbar_wait_bounded(&full[s], ph)) {
                record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                *abort_flag = 1;
                fail        = true;
            }
            fail = __any_sync(0xffffffffu, fail);  // mma.sync needs the whole warp
#ifdef B200Q8_TIMELINE
            if (threadIdx.x == 0 && kc == 0 && u == (int) blockIdx.x) GTL(3);
#endif
            if (!fail) {
                const uint8_t * wt    = ring + (size_t) s * slot;
                const uint8_t * row_a = wt + (rt * 16 + g) * kChunkRowBytes;
                const uint8_t * row_b = row_a + 8 * kChunkRowBytes;
                const uint8_t * xc    = wt + w_bytes;
                const float *   xsc   = reinterpret_cast<const float *>(xc + TG * 8 * kChunkBlocks * kQK);
#pragma unroll
                for (int j = 0; j < kChunkBlocks; ++j) {
                    if (j >= j0 && j < j1) {  // warp-uniform
                        uint2 wa, wb;
                        ld_w8(j, row_a, tq, wa);
                        ld_w8(j, row_b, tq, wb);
                        const uint32_t A[4] = { wa.x, wb.x, wa.y, wb.y };
                        const float    da   = __half2float(*reinterpret_cast<const __half *>(row_a + j * kBlockBytes));
                        const float    db   = __half2float(*reinterpret_cast<const __half *>(row_b + j * kBlockBytes));
                        uint2  bv[TG];
                        float2 xv[TG];
#pragma unroll
                        for (int tg = 0; tg < TG; ++tg) {
                            const int unit = (2 * j + (tq >> 1)) ^ (g << 1);
                            bv[tg]         = *reinterpret_cast<const uint2 *>(
                                xc + (tg * 8 + g) * (kChunkBlocks * kQK) + unit * 16 + (tq & 1) * 8);
                            xv[tg] = *reinterpret_cast<const float2 *>(xsc + j * (TG * 8) + tg * 8 + 2 * tq);
                        }
                        int D[TG][4];
#pragma unroll
                        for (int tg = 0; tg < TG; ++tg) {
                            mma_s8(D[tg], A, bv[tg], cbias);
                        }
                        const float2 da2 = make_float2(da, da);
                        const float2 db2 = make_float2(db, db);
#pragma unroll
                        for (int tg = 0; tg < TG; ++tg) {
                            const float2 s01 =
                                __fadd2_rn(make_float2(__int_as_float(D[tg][0]), __int_as_float(D[tg][1])), nbias);
                            const float2 s23 =
                                __fadd2_rn(make_float2(__int_as_float(D[tg][2]), __int_as_float(D[tg][3])), nbias);
                            acc[tg][0] = __ffma2_rn(s01, __fmul2_rn(da2, xv[tg]), acc[tg][0]);
                            acc[tg][1] = __ffma2_rn(s23, __fmul2_rn(db2, xv[tg]), acc[tg][1]);
                        }
                    }
                }
            }
            __syncwarp();
            // a slot is handed back only after its data was seen to land
            if (lane == 0 && !fail) {
                mbar_arrive(&empty[s]);
            }
            if (++s == S) {
                s = 0;
                ph ^= 1;
            }
        }
        if (threadIdx.x == 0) GTL(4);
        // Combine the block subsets of each row tile in a fixed order
        // (subset 0 + 1 + ...); the ks_n warps of a row tile share the token
        // groups of the combine and the stores.
        auto store = [&](int tg, float4 v) {
            const int ra = rt * 16 + g;
            const int c0 = tg * 8 + 2 * tq;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int tok = tok0 + c0 + q;
                if (tok < a.M) {
                    // split-K: this unit's partial sums, added up by the block's last split
                    float * dst = split ? a.part + ((size_t) kz * a.M + tok) * a.N + r0
                                               : a.y + (size_t) tok * a.y_stride + r0;
                    if (ra < rows) {
                        dst[ra] = q ? v.y : v.x;
                    }
                    if (ra + 8 < rows) {
                        dst[ra + 8] = q ? v.w : v.z;
                    }
                }
            }
        };
        if (ks_n > 1) {
#pragma unroll
            for (int tg = 0; tg < TG; ++tg) {
                red4[(warp * TG + tg) * 32 + lane] = make_float4(acc[tg][0].x, acc[tg][0].y, acc[tg][1].x, acc[tg][1].y);
            }
            named_barrier_sync(1, kGemmConsumerWarps * 32);
            const bool ok = !fail && *abort_flag == 0;
#pragma unroll
            for (int tg = 0; tg < TG; ++tg) {
                if (tg % ks_n == ks) {
                    float4 v = red4[(rt * TG + tg) * 32 + lane];
                    for (int k2 = 1; k2 < ks_n; ++k2) {
                        const float4 o = red4[((rt + k2 * rt_n) * TG + tg) * 32 + lane];
                        v.x += o.x;
                        v.y += o.y;
                        v.z += o.z;
                        v.w += o.w;
                    }
                    if (ok) {
                        store(tg, v);
                    }
                }
            }
            named_barrier_sync(1, kGemmConsumerWarps * 32);
        } else if (!fail && *abort_flag == 0) {
#pragma unroll
            for (int tg = 0; tg < TG; ++tg) {
                store(tg, make_float4(acc[tg][0].x, acc[tg][0].y, acc[tg][1].x, acc[tg][1].y));
            }
        }
        if (split) {
            // every consumer's partial stores reach the device before the count
            __threadfence();
            named_barrier_sync(1, kGemmConsumerWarps * 32);
            unsigned * const cnt = a.cnt + (size_t) tc * a.n_rb + (ut - tc * a.n_rb);
            if (threadIdx.x == 0) {
                *last_s = atomicAdd(cnt, 1u) == (unsigned) (a.ksplit - 1) ? 1u : 0u;
                __threadfence();
            }
            named_barrier_sync(1, kGemmConsumerWarps * 32);
            if (*last_s) {
                // all splits of this (tokens, rows) block have landed: add them in split order
                // kU elements per thread per pass, their loads issued together
                constexpr int kU     = 4;
                constexpr int kT     = kGemmConsumerWarps * 32;
                const bool    ok     = !fail && *abort_flag == 0;
                const size_t  plane  = (size_t) a.M * a.N;
                const int     n_elem = a.tm * a.rb;
                for (int i0 = threadIdx.x; i0 < n_elem; i0 += kU * kT) {
                    float  v[kU];
                    size_t off[kU], yoff[kU];
                    bool   in[kU];
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const int i   = i0 + q * kT;
                        const int t   = i / a.rb;
                        const int r   = i - t * a.rb;
                        const int tok = tok0 + t;
                        in[q]         = i < n_elem && tok < a.M && r < rows;
                        off[q]        = (size_t) tok * a.N + r0 + r;
                        yoff[q]       = (size_t) tok * a.y_stride + r0 + r;
                        v[q]          = in[q] ? __ldcg(a.part + off[q]) : 0.0f;
                    }
                    for (int k2 = 1; k2 < a.ksplit; ++k2) {
#pragma unroll
                        for (int q = 0; q < kU; ++q) {
                            if (in[q]) {
                                v[q] += __ldcg(a.part + off[q] + (size_t) k2 * plane);
                            }
                        }
                    }
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        if (in[q] && ok) {
                            a.y[yoff[q]] = v[q];
                        }
                    }
                }
                if (threadIdx.x == 0) {
                    *cnt = 0u;  // ready for the next launch
                }
            }
            named_barrier_sync(1, kGemmConsumerWarps * 32);
        }
    }
    if (threadIdx.x == 0) GTL(5);
    if (threadIdx.x == 32 * (kGemmConsumerWarps - 1)) GTL(7);
}

// Stage one token's GEMM input: one CTA per token, each thread holds E
// groups of 4 consecutive values (8 threads per Q8_0 block).  kind:
// 0 = rms_norm(a [+ b]) * norm (a + b also written to sum_out),
// 1 = GQA expansion of a (query head h reads KV head h / group),
// 2 = silu(a) * b, 3 = a.
// The value is quantized and written into the token's staged records; the
// fp32 value itself goes to trace when given.
struct StageArgs {
    int           kind;
    const float * a;
    const float * b;
    size_t        ab_stride;
    float *       sum_out;
    size_t        sum_stride;
    const float * norm;
    float         eps;
    int           K;
    int           head_dim;
    int           group;
    float *       trace;
    size_t        trace_stride;
    uint8_t *     xrec;
    int           tm;
    int           tl_slot;  // timeline builds only
};

template <int MODE, int E>
__global__ void __launch_bounds__(1024) stage_rows_kernel(const StageArgs s) {
    __shared__ double part[32];
    __shared__ float  scale_s;
#ifdef B200Q8_TIMELINE
    const StageArgs & a = s;
    if (threadIdx.x == 0) GTL(0);
#endif
    pdl_launch_dependents();
    const int t  = threadIdx.x;
    const int T  = blockDim.x;
    const int K4 = s.K >> 2;
    // The norm weights are constant: load them before the wait on the kernel
    // that wrote this op's input, so their latency overlaps it.
    float4 nv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int f = t + e * T;
        nv[e]       = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        if (s.kind == 0 && f < K4) {
            const float * np = s.norm + 4 * f;  // caller's pointer: only 4-byte alignment is assumed
            nv[e]            = make_float4(np[0], np[1], np[2], np[3]);
        }
    }
    pdl_wait_primary();
#ifdef B200Q8_TIMELINE
    if (threadIdx.x == 0) GTL(1);
#endif
    const int     m    = blockIdx.x;
    const float * am   = s.a + (size_t) m * s.ab_stride;
    const float * bm   = s.b ? s.b + (size_t) m * s.ab_stride : nullptr;
    float4        v[E];
    double        ss = 0.0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int f = t + e * T;
        v[e]        = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (f < K4) {
            if (s.kind == 0) {
                float4 x = reinterpret_cast<const float4 *>(am)[f];
                if (bm) {
                    const float4 y = reinterpret_cast<const float4 *>(bm)[f];
                    x              = make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z),
                                                 __fadd_rn(x.w, y.w));
                }
                if (s.sum_out) {
                    reinterpret_cast<float4 *>(s.sum_out + (size_t) m * s.sum_stride)[f] = x;
                }
                ss += (double) __fmul_rn(x.x, x.x);
                ss += (double) __fmul_rn(x.y, x.y);
                ss += (double) __fmul_rn(x.z, x.z);
                ss += (double) __fmul_rn(x.w, x.w);
                v[e] = x;
            } else if (s.kind == 1) {
                const int i    = 4 * f;
                const int head = i / s.head_dim;
                v[e] = *reinterpret_cast<const float4 *>(am + (head / s.group) * s.head_dim + (i - head * s.head_dim));
            } else if (s.kind == 2) {
                const float4 x = reinterpret_cast<const float4 *>(am)[f];
                const float4 y = reinterpret_cast<const float4 *>(bm)[f];
                v[e] = make_float4(__fmul_rn(silu_f32(x.x), y.x), __fmul_rn(silu_f32(x.y), y.y),
                                   __fmul_rn(silu_f32(x.z), y.z), __fmul_rn(silu_f32(x.w), y.w));
            } else {
                const float * row = am;
                v[e] = make_float4(row[4 * f], row[4 * f + 1], row[4 * f + 2], row[4 * f + 3]);
            }
        }
    }
    if (s.kind == 0) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, off);
        }
        if ((t & 31) == 0) {
            part[t >> 5] = ss;
        }
        __syncthreads();
        if (t == 0) {
            double tot = 0.0;
            for (int w = 0; w < (T >> 5); ++w) {
                tot += part[w];
            }
            const float mean = (float) (tot / (double) s.K);
            scale_s          = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, s.eps)));
        }
        __syncthreads();
        const float sc = scale_s;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int f = t + e * T;
            if (f < K4) {
                v[e] = make_float4(__fmul_rn(__fmul_rn(v[e].x, sc), nv[e].x), __fmul_rn(__fmul_rn(v[e].y, sc), nv[e].y),
                                   __fmul_rn(__fmul_rn(v[e].z, sc), nv[e].z), __fmul_rn(__fmul_rn(v[e].w, sc), nv[e].w));
            }
        }
    }
    // quantize: the 8 threads of a block are 8 consecutive lanes
    const int      n_kc = s.K >> 8;
    const int      tc   = m / s.tm;
    const int      tt   = m - tc * s.tm;
    const int      li   = t & 7;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int         f     = t + e * T;
        const bool        valid = f < K4;
        float             vv[4] = { v[e].x, v[e].y, v[e].z, v[e].w };
        const float       amx   = block_amax<8, 4>(vv, li);
        const QuantParams qp    = quant_params<MODE>(amx);
        if (valid) {
            const int blk = f >> 3;          // Q8_0 block
            const int kc  = blk >> 3;        // K chunk
            const int j   = blk & 7;         // block within the chunk
            uint8_t * rec = s.xrec + ((size_t) tc * n_kc + kc) * (size_t) (s.tm * kRecTokenBytes);
            const uint32_t q = (uint32_t) (quant_code<MODE>(vv[0], qp.id) & 0xff) |
                               ((uint32_t) (quant_code<MODE>(vv[1], qp.id) & 0xff) << 8) |
                               ((uint32_t) (quant_code<MODE>(vv[2], qp.id) & 0xff) << 16) |
                               ((uint32_t) (quant_code<MODE>(vv[3], qp.id) & 0xff) << 24);
            *reinterpret_cast<uint32_t *>(rec + rec_code_offset(tt, j, 4 * li)) = q;
            if (li == 0) {
                reinterpret_cast<float *>(rec + s.tm * kChunkBlocks * kQK)[j * s.tm + tt] = qp.d;
            }
            if (s.trace) {
                reinterpret_cast<float4 *>(s.trace + (size_t) m * s.trace_stride)[f] = v[e];
            }
        }
    }
#ifdef B200Q8_TIMELINE
    __syncthreads();
    if (threadIdx.x == 0) GTL(2);
#endif
}

__global__ void residual_rows_kernel(const float * __restrict__ a, const float * __restrict__ b, size_t ab_stride,
                                     float * __restrict__ out, size_t out_stride, int K) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const int m = blockIdx.x;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        out[(size_t) m * out_stride + i] = __fadd_rn(a[(size_t) m * ab_stride + i], b[(size_t) m * ab_stride + i]);
    }
}

template <typename F, typename... Args>
cudaError_t launch_pdl(F fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = grid;
    cfg.blockDim           = block;
    cfg.dynamicSmemBytes   = smem;
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

// threads per stage CTA and groups of 4 per thread for a row of K values
void stage_shape(int K, int * threads, int * e) {
    const int k4 = K / 4;
    *e           = (k4 + 1023) / 1024;
    *threads     = ((k4 + *e - 1) / *e + 31) / 32 * 32;
}

template <int MODE>
cudaError_t launch_stage_mode(const StageArgs & s, int64_t M, cudaStream_t stream, bool pdl) {
    int threads, e;
    stage_shape(s.K, &threads, &e);
    switch (e) {
        case 1: return launch_pdl(stage_rows_kernel<MODE, 1>, dim3((unsigned) M), dim3(threads), 0, stream, pdl, s);
        case 2: return launch_pdl(stage_rows_kernel<MODE, 2>, dim3((unsigned) M), dim3(threads), 0, stream, pdl, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_stage(const StageArgs & s, int64_t M, int mode, cudaStream_t stream, bool pdl) {
    if (s.K % 256 != 0 || s.K > 8192 || M < 1) {
        return cudaErrorInvalidValue;
    }
    switch (mode) {
        case B200Q8_QUANT_CPU_X86: return launch_stage_mode<B200Q8_QUANT_CPU_X86>(s, M, stream, pdl);
        case B200Q8_QUANT_CPU_ARM: return launch_stage_mode<B200Q8_QUANT_CPU_ARM>(s, M, stream, pdl);
        default: return launch_stage_mode<B200Q8_QUANT_REF>(s, M, stream, pdl);
    }
}

size_t gemm_slot_bytes(int rb, int tm) {
    return (size_t) rb * kChunkRowBytes + (size_t) tm * kRecTokenBytes;
}

size_t gemm_fixed_bytes(int tg) {
    return 128 + (size_t) kGemmConsumerWarps * 32 * tg * 4 * 4;
}

// cuTensorMapEncodeTiled from the driver, through the runtime (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *                          p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            p = nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// Q8_0 rows viewed as a 2-D tensor of 2-byte elements: row_bytes / 2 wide,
// N high; box = one 256-wide K chunk (136 elements = 272 bytes) x rb rows.
bool encode_weight_map(CUtensorMap * map, const uint8_t * w, size_t row_bytes, int64_t N, int rb) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) {
        return false;
    }
    const cuuint64_t dims[2]    = { (cuuint64_t) (row_bytes / 2), (cuuint64_t) N };
    const cuuint64_t strides[1] = { (cuuint64_t) row_bytes };
    const cuuint32_t box[2]     = { (cuuint32_t) (kChunkRowBytes / 2), (cuuint32_t) rb };
    const cuuint32_t estr[2]    = { 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// token groups of 8 per chunk: the kernel's template argument
int gemm_tg(int tm) {
    return tm / 8;
}

template <int TG, bool SPLITK>
cudaError_t launch_gemm_tg(const GemmArgs & a, const CUtensorMap & wmap, int grid, size_t smem, cudaStream_t stream,
                           bool pdl) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_q8_0_kernel<TG, SPLITK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    return e != cudaSuccess ? e
                            : launch_pdl(gemm_q8_0_kernel<TG, SPLITK>, dim3((unsigned) grid), dim3(kGemmThreads), smem, stream,
                                         pdl, a, wmap);
}

}  // namespace

GemmChunking gemm_chunking(int64_t M) {
    GemmChunking c;
    c.n_tc = (int) ((M + kMaxTokenChunk - 1) / kMaxTokenChunk);
    if (c.n_tc < 1) {
        c.n_tc = 1;
    }
    const int64_t per = (M + c.n_tc - 1) / c.n_tc;
    c.tm              = (int) ((per + 7) / 8 * 8);
    return c;
}

cudaError_t launch_stage_rows(int kind, const float * a, const float * b, size_t ab_stride, float * sum_out,
                              size_t sum_stride, const float * norm, float eps, int K, int head_dim, int group,
                              float * trace, size_t trace_stride, int64_t M, int mode, uint8_t * xrec,
                              cudaStream_t stream, bool pdl) {
    StageArgs s    = {};
    s.kind         = kind;
    s.a            = a;
    s.b            = b;
    s.ab_stride    = ab_stride;
    s.sum_out      = sum_out;
    s.sum_stride   = sum_stride;
    s.norm         = norm;
    s.eps          = eps;
    s.K            = K;
    s.head_dim     = head_dim;
    s.group        = group;
    s.trace        = trace;
    s.trace_stride = trace_stride;
    s.xrec         = xrec;
    s.tm           = gemm_chunking(M).tm;
#ifdef B200Q8_TIMELINE
    s.tl_slot = tl_take('s');
#else
    s.tl_slot = -1;
#endif
    return launch_stage(s, M, mode, stream, pdl);
}

cudaError_t launch_residual_rows(const float * a, const float * b, size_t ab_stride, float * out, size_t out_stride,
                                 int K, int64_t M, cudaStream_t stream, bool pdl) {
    return launch_pdl(residual_rows_kernel, dim3((unsigned) M), dim3(256), 0, stream, pdl, a, b, ab_stride, out,
                      out_stride, K);
}

size_t gemm_workspace_bytes(int64_t K, int64_t M) {
    const GemmChunking c = gemm_chunking(M);
    return (size_t) c.n_tc * (size_t) (K / 256) * (size_t) c.tm * kRecTokenBytes;
}

bool gemm_supported(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, int64_t M) {
    // K % 256: whole 272-byte chunks, 16-byte aligned in every row
    if (M < 1 || M > kGemmMaxM || N < 16 || N > (int64_t) 1 << 30 || K < 256 || K % 256 != 0 || K > 8192 ||
        row_bytes % 16 != 0 || row_bytes < (size_t) (K / kQK) * kBlockBytes ||
        (reinterpret_cast<uintptr_t>(w) % 16) != 0) {
        return false;
    }
    const GemmChunking c = gemm_chunking(M);
    return gemm_fixed_bytes(gemm_tg(c.tm)) + 2 * gemm_slot_bytes(16, c.tm) <= (size_t) kGemmSmemLimit;
}

cudaError_t launch_gemm_staged(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const uint8_t * xrec,
                               int64_t M, float * y, size_t y_stride, cudaStream_t stream, int sm_count, bool pdl,
                               const GemmSplit * split) {
    const GemmChunking c = gemm_chunking(M);
    GemmArgs           a = {};
    a.w                  = w;
    a.row_bytes          = row_bytes;
    a.K                  = (int) K;
    a.N                  = (int) N;
    a.M                  = (int) M;
    a.xrec               = xrec;
    a.y                  = y;
    a.y_stride           = y_stride;
    a.tm                 = c.tm;
    a.n_tc               = c.n_tc;
#ifdef B200Q8_TIMELINE
    a.tl_slot = tl_take('g');
#else
    a.tl_slot = -1;
#endif
    const int tg         = gemm_tg(c.tm);
    const size_t fixed   = gemm_fixed_bytes(tg);
    // Rows per unit: fewer, larger units share each activation record among
    // more rows; more units fill more SMs.  Cost ~ units per CTA x (rows +
    // a fixed share for the record and the unit's combine step).
    int    best_rb   = 16;
    double best_cost = 1e300;
    for (int rb = 16; rb <= 128 && rb <= N; rb *= 2) {
        if (fixed + 2 * gemm_slot_bytes(rb, c.tm) > (size_t) kGemmSmemLimit) {
            break;
        }
        const int64_t units = (int64_t) c.n_tc * ((N + rb - 1) / rb);
        const int64_t waves = (units + sm_count - 1) / sm_count;
        const double  cost  = (double) waves * (rb + 24);
        if (cost < best_cost) {
            best_cost = cost;
            best_rb   = rb;
        }
    }
    a.rb             = best_rb;
    a.n_rb           = (int) ((N + a.rb - 1) / a.rb);
    a.n_units        = a.n_tc * a.n_rb;
    // split-K when the units leave SMs idle: the largest split of the K chunks
    // (a divisor of them) whose units still fit in one wave, given room for
    // the partials and the counters.  Only for token chunks of <= 16: on
    // larger chunks (M = 32 and 64 measured) the partials' round trip through
    // L2 and the serial combine cost more than the idle SMs.
    const int n_kc = (int) (K >> 8);
    a.ksplit       = 1;
    for (int d = 2; split != nullptr && tg <= kGemmSplitMaxTG && d <= n_kc; ++d) {
        if (n_kc % d == 0 && (int64_t) a.n_units * d <= sm_count &&
            (size_t) d * (size_t) M * (size_t) N <= split->part_floats &&
            (size_t) a.n_units <= split->n_cnt) {
            a.ksplit = d;
        }
    }
    a.kc_n    = n_kc / a.ksplit;
    a.part    = a.ksplit > 1 ? split->part : nullptr;
    a.cnt     = a.ksplit > 1 ? split->cnt : nullptr;
    a.n_units = a.n_tc * a.n_rb * a.ksplit;
    const size_t slot = gemm_slot_bytes(a.rb, c.tm);
    a.n_slots        = (int) std::min<size_t>(kGemmMaxSlots, ((size_t) kGemmSmemLimit - fixed) / slot);
    if (a.n_slots < 2) {
        return cudaErrorInvalidValue;
    }
    const size_t smem = fixed + (size_t) a.n_slots * slot;
    const int    grid = std::min(a.n_units, sm_count);
    CUtensorMap  wmap;
    if (!encode_weight_map(&wmap, w, row_bytes, N, a.rb)) {
        return cudaErrorInvalidValue;
    }
    // TG 1 and 2 run the split-capable instances whether or not this call
    // splits: measured faster at M <= 16 than the plain ones, for every op
    static_assert(kGemmSplitMaxTG == 2, "split-capable instances: TG 1 and 2");
    switch (tg) {
        case 1: return launch_gemm_tg<1, true>(a, wmap, grid, smem, stream, pdl);
        case 2: return launch_gemm_tg<2, true>(a, wmap, grid, smem, stream, pdl);
        case 3: return launch_gemm_tg<3, false>(a, wmap, grid, smem, stream, pdl);
        case 4: return launch_gemm_tg<4, false>(a, wmap, grid, smem, stream, pdl);
        case 5: return launch_gemm_tg<5, false>(a, wmap, grid, smem, stream, pdl);
        case 6: return launch_gemm_tg<6, false>(a, wmap, grid, smem, stream, pdl);
        case 7: return launch_gemm_tg<7, false>(a, wmap, grid, smem, stream, pdl);
        case 8: return launch_gemm_tg<8, false>(a, wmap, grid, smem, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const float * x, size_t x_stride,
                        int64_t M, float * y, size_t y_stride, int mode, void * workspace, cudaStream_t stream,
                        int sm_count) {
    uint8_t *   xrec = static_cast<uint8_t *>(workspace);
    cudaError_t e    = launch_stage_rows(3, x, nullptr, x_stride, nullptr, 0, nullptr, 0.0f, (int) K, 1, 1, nullptr, 0,
                                         M, mode, xrec, stream, false);
    if (e != cudaSuccess) {
        return e;
    }
    return launch_gemm_staged(w, row_bytes, K, N, xrec, M, y, y_stride, stream, sm_count, true);
}

}  // namespace b200q8

#ifdef B200Q8_TIMELINE
// Copies the stamps and the slot kinds ('g' GEMM, 's' stage) and restarts slot numbering.
extern "C" int b200q8_gemm_timeline(unsigned long long * host, size_t n, char * kinds, int reset) {
    using namespace b200q8;
    const size_t have = (size_t) kTlSlots * kTlCtas * 8;
    int          rc   = 0;
    if (host != nullptr) {
        rc = cudaMemcpyFromSymbol(host, g_tl, sizeof(unsigned long long) * (n < have ? n : have)) == cudaSuccess ? 0 : 1;
    }
    if (kinds != nullptr) {
        for (int i = 0; i < kTlSlots; ++i) {
            kinds[i] = i < g_tl_next ? g_tl_kind[i] : 0;
        }
    }
    if (reset) {
        g_tl_next = 0;
    }
    return rc;
}
#endif
