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
// each 256-wide K chunk of the unit's weight rows (RB 1-D copies of 272
// bytes, one per row) and the matching activation record (one copy) land in
// one shared-memory slot of a ring, so weights and activations stream
// together and every byte is loaded once per unit.  Eight consumer warps
// split the unit into 16-row tiles x block subsets of the chunk; partial sums
// over K are combined through shared memory in a fixed order, so results are
// deterministic.  Copies are never multicast.
#include "common.cuh"
#include "kernels.h"

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
constexpr int   kMmaBias           = 0x4B400000;  // float 12582912.0f
constexpr float kMmaBiasF          = 12582912.0f;

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Byte offset of code byte i (0..31) of block j (0..7) of token t inside a
// record: 16-byte unit (2j + i/16) is XOR-swizzled by 2*(t % 8), so the eight
// tokens a B-fragment load touches fall in eight different bank groups.
__host__ __device__ __forceinline__ int rec_code_offset(int t, int j, int i) {
    const int unit = (2 * j + (i >> 4)) ^ ((t & 7) << 1);
    return t * (kChunkBlocks * kQK) + unit * 16 + (i & 15);
}

// The 8 code bytes 8*tq .. 8*tq+7 of block j of a staged weight row (34-byte
// blocks, so only 2-byte aligned; the alignment class depends on j alone).
// Lanes load 8 consecutive bytes rather than the two 4-byte groups of the
// standard fragment: A and B use the same permutation of k, so every MMA
// still sums exactly the products of matching codes.
template <int J>
__device__ __forceinline__ uint2 lds_w8(uint32_t row, int tq) {
    const uint32_t off = (uint32_t) (J * kBlockBytes + 2 + 8 * tq);
    uint2          r;
    if ((off & 7) == 0) {
        const uint64_t v = lds_u64(row + off);
        r.x              = (uint32_t) v;
        r.y              = (uint32_t) (v >> 32);
    } else if ((off & 3) == 0) {
        r.x = lds_u32(row + off);
        r.y = lds_u32(row + off + 4);
    } else if (((off - 2) & 7) == 0) {
        const uint64_t v  = lds_u64(row + off - 2);
        const uint32_t w2 = lds_u32(row + off + 6);
        r.x               = __byte_perm((uint32_t) v, (uint32_t) (v >> 32), 0x5432);
        r.y               = __byte_perm((uint32_t) (v >> 32), w2, 0x5432);
    } else {
        const uint32_t w0 = lds_u32(row + off - 2);
        const uint64_t v  = lds_u64(row + off + 2);
        r.x               = __byte_perm(w0, (uint32_t) v, 0x5432);
        r.y               = __byte_perm((uint32_t) v, (uint32_t) (v >> 32), 0x5432);
    }
    return r;
}

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
    int             n_units;   // n_tc * n_rb
    int             n_slots;
};

// TG: token groups of 8 a warp can hold (>= tm / 8).
template <int TG>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_q8_0_kernel(const GemmArgs a) {
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
        // Producer warp: lane 0 arms each slot, then all lanes issue the row
        // copies.  Weights are constant, so the first S slots' weights stream
        // before the wait on the kernel that wrote the activations.
        const uint64_t wpol     = a.n_tc == 1 ? l2_evict_first_policy() : l2_evict_last_policy();
        const uint64_t xpol     = l2_evict_last_policy();
        const int      my_units = (a.n_units - (int) blockIdx.x + G - 1) / G;
        const int      total    = my_units * n_kc;
        // fill i = chunk kc of the CTA's unit i / n_kc; it uses slot i % S
        auto issue_w = [&](int i, int si) {
            const int ui   = i / n_kc;
            const int kc   = i - ui * n_kc;
            const int u    = (int) blockIdx.x + ui * G;
            const int tc   = u / a.n_rb;
            const int r0   = (u - tc * a.n_rb) * a.rb;
            const int rows = min(a.rb, a.N - r0);
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[si], (uint32_t) (rows * kChunkRowBytes + rec_bytes));
            }
            __syncwarp();
            uint8_t * dst = ring + (size_t) si * slot;
            for (int r = lane; r < rows; r += 32) {
                bulk_copy_g2s(dst + (size_t) r * kChunkRowBytes,
                              a.w + (size_t) (r0 + r) * a.row_bytes + (size_t) kc * kChunkRowBytes,
                              (uint32_t) kChunkRowBytes, &full[si], wpol);
            }
        };
        auto issue_x = [&](int i, int si) {
            const int ui = i / n_kc;
            const int kc = i - ui * n_kc;
            const int tc = ((int) blockIdx.x + ui * G) / a.n_rb;
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
        pdl_wait_primary();
        for (int i = 0; i < pre; ++i) {
            issue_x(i, i);
        }
        int      s     = pre == S ? 0 : pre;
        uint32_t ph    = pre == S ? 1 : 0;
        int      fills = pre;
        for (int i = pre; i < total; ++i) {
            bool ok = true;
            if (lane == 0) {
                ok = mbar_wait_bounded_sleep(&empty[s], ph ^ 1);
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
        }
        return;
    }

    // consumer roles: 16-row tile rt of the unit, block subset ks of each chunk
    const int rt_n  = a.rb >> 4;
    const int ks_n  = kChunkBlocks / rt_n > 0 ? kChunkBlocks / rt_n : 1;  // K subsets (8 warps = rt_n x ks_n)
    const int rt    = warp % rt_n;
    const int ks    = warp / rt_n;
    const int j0    = ks * (kChunkBlocks / ks_n);
    const int j1    = j0 + kChunkBlocks / ks_n;
    const int g     = lane >> 2;
    const int tq    = lane & 3;
    const int n_tg  = a.tm >> 3;
    const uint32_t ring_s = smem_addr(ring);
    const float2   biasf  = make_float2(kMmaBiasF, kMmaBiasF);

    int      s    = 0;
    uint32_t ph   = 0;
    bool     fail = false;
    // Every consumer warp runs the same trip counts and reaches the same
    // barriers whatever happens; a failed wait only skips work.
    for (int u = blockIdx.x; u < a.n_units; u += G) {
        const int tc   = u / a.n_rb;
        const int r0   = (u - tc * a.n_rb) * a.rb;
        const int rows = min(a.rb, a.N - r0);
        const int tok0 = tc * a.tm;
        float2    acc[TG][2];
#pragma unroll
        for (int i = 0; i < TG; ++i) {
            acc[i][0] = make_float2(0.0f, 0.0f);
            acc[i][1] = make_float2(0.0f, 0.0f);
        }
        for (int kc = 0; kc < n_kc; ++kc) {
            if (!fail && !mbar_wait_bounded(&full[s], ph)) {
                record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                *abort_flag = 1;
                fail        = true;
            }
            fail = __any_sync(0xffffffffu, fail);  // mma.sync needs the whole warp
            if (!fail) {
                const uint32_t wt    = ring_s + (uint32_t) (s * slot);
                const uint32_t row_a = wt + (uint32_t) ((rt * 16 + g) * kChunkRowBytes);
                const uint32_t row_b = row_a + 8 * kChunkRowBytes;
                const uint32_t xc    = wt + (uint32_t) w_bytes;
                const uint32_t xsc   = xc + (uint32_t) (a.tm * kChunkBlocks * kQK);
#pragma unroll
                for (int j = 0; j < kChunkBlocks; ++j) {
                    if (j >= j0 && j < j1) {
                        uint2 wa, wb;
                        switch (j) {
                            case 0: wa = lds_w8<0>(row_a, tq); wb = lds_w8<0>(row_b, tq); break;
                            case 1: wa = lds_w8<1>(row_a, tq); wb = lds_w8<1>(row_b, tq); break;
                            case 2: wa = lds_w8<2>(row_a, tq); wb = lds_w8<2>(row_b, tq); break;
                            case 3: wa = lds_w8<3>(row_a, tq); wb = lds_w8<3>(row_b, tq); break;
                            case 4: wa = lds_w8<4>(row_a, tq); wb = lds_w8<4>(row_b, tq); break;
                            case 5: wa = lds_w8<5>(row_a, tq); wb = lds_w8<5>(row_b, tq); break;
                            case 6: wa = lds_w8<6>(row_a, tq); wb = lds_w8<6>(row_b, tq); break;
                            default: wa = lds_w8<7>(row_a, tq); wb = lds_w8<7>(row_b, tq); break;
                        }
                        const uint32_t A[4] = { wa.x, wb.x, wa.y, wb.y };
                        const float    da   = __half2float(__ushort_as_half(
                            (unsigned short) lds_u16(row_a + (uint32_t) (j * kBlockBytes))));
                        const float db = __half2float(__ushort_as_half(
                            (unsigned short) lds_u16(row_b + (uint32_t) (j * kBlockBytes))));
                        const float2 da2 = make_float2(da, da);
                        const float2 db2 = make_float2(db, db);
#pragma unroll
                        for (int tg = 0; tg < TG; ++tg) {
                            if (tg < n_tg) {
                                const int      t    = tg * 8 + g;
                                const int      unit = (2 * j + (tq >> 1)) ^ (g << 1);
                                const uint64_t bv =
                                    lds_u64(xc + (uint32_t) (t * (kChunkBlocks * kQK) + unit * 16 + (tq & 1) * 8));
                                const uint32_t B[2] = { (uint32_t) bv, (uint32_t) (bv >> 32) };
                                const float2   x2 =
                                    lds_f2(xsc + (uint32_t) ((j * a.tm + tg * 8 + 2 * tq) * 4));
                                int D[4] = { kMmaBias, kMmaBias, kMmaBias, kMmaBias };
                                mma_s8(D, A, B);
                                const float2 s01 = __fadd2_rn(
                                    make_float2(__int_as_float(D[0]), __int_as_float(D[1])),
                                    make_float2(-biasf.x, -biasf.y));
                                const float2 s23 = __fadd2_rn(
                                    make_float2(__int_as_float(D[2]), __int_as_float(D[3])),
                                    make_float2(-biasf.x, -biasf.y));
                                acc[tg][0] = __ffma2_rn(s01, __fmul2_rn(da2, x2), acc[tg][0]);
                                acc[tg][1] = __ffma2_rn(s23, __fmul2_rn(db2, x2), acc[tg][1]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[s]);
            }
            if (++s == S) {
                s = 0;
                ph ^= 1;
            }
        }
        // combine the block subsets in a fixed order (subset 0 adds 1, 2, ...)
        if (ks_n > 1) {
            if (ks != 0) {
                float4 * mine = reinterpret_cast<float4 *>(red) + (size_t) (warp * TG) * 32 + lane;
#pragma unroll
                for (int tg = 0; tg < TG; ++tg) {
                    if (tg < n_tg) {
                        mine[tg * 32] = make_float4(acc[tg][0].x, acc[tg][0].y, acc[tg][1].x, acc[tg][1].y);
                    }
                }
            }
            named_barrier_sync(1, kGemmConsumerWarps * 32);
            if (ks == 0) {
                for (int k2 = 1; k2 < ks_n; ++k2) {
                    const float4 * o =
                        reinterpret_cast<const float4 *>(red) + (size_t) ((warp + k2 * rt_n) * TG) * 32 + lane;
#pragma unroll
                    for (int tg = 0; tg < TG; ++tg) {
                        if (tg < n_tg) {
                            const float4 v = o[tg * 32];
                            acc[tg][0].x += v.x;
                            acc[tg][0].y += v.y;
                            acc[tg][1].x += v.z;
                            acc[tg][1].y += v.w;
                        }
                    }
                }
            }
            named_barrier_sync(1, kGemmConsumerWarps * 32);
        }
        if (ks == 0 && !fail && *abort_flag == 0) {
            const int ra = rt * 16 + g;
#pragma unroll
            for (int tg = 0; tg < TG; ++tg) {
                if (tg < n_tg) {
                    const int c0 = tg * 8 + 2 * tq;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int tok = tok0 + c0 + q;
                        if (c0 + q < a.tm && tok < a.M) {
                            float * dst = a.y + (size_t) tok * a.y_stride + r0;
                            if (ra < rows) {
                                dst[ra] = q ? acc[tg][0].y : acc[tg][0].x;
                            }
                            if (ra + 8 < rows) {
                                dst[ra + 8] = q ? acc[tg][1].y : acc[tg][1].x;
                            }
                        }
                    }
                }
            }
        }
    }
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
};

template <int MODE, int E>
__global__ void __launch_bounds__(1024) stage_rows_kernel(const StageArgs s) {
    __shared__ double part[32];
    __shared__ float  scale_s;
    pdl_launch_dependents();
    pdl_wait_primary();
    const int     m    = blockIdx.x;
    const int     t    = threadIdx.x;
    const int     T    = blockDim.x;
    const int     K4   = s.K >> 2;
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
                const float * np = s.norm + 4 * f;  // caller's pointer: only 4-byte alignment is assumed
                const float4  nv = make_float4(np[0], np[1], np[2], np[3]);
                v[e]            = make_float4(__fmul_rn(__fmul_rn(v[e].x, sc), nv.x), __fmul_rn(__fmul_rn(v[e].y, sc), nv.y),
                                              __fmul_rn(__fmul_rn(v[e].z, sc), nv.z), __fmul_rn(__fmul_rn(v[e].w, sc), nv.w));
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

int gemm_tg(int tm) {
    const int n_tg = tm / 8;
    return n_tg <= 2 ? 2 : n_tg <= 4 ? 4 : 8;
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
    if (M < 1 || M > 1024 || N < 1 || N > (int64_t) 1 << 30 || K < 256 || K % 256 != 0 || K > 8192 ||
        row_bytes % 16 != 0 || row_bytes < (size_t) (K / kQK) * kBlockBytes ||
        (reinterpret_cast<uintptr_t>(w) % 16) != 0) {
        return false;
    }
    const GemmChunking c = gemm_chunking(M);
    return gemm_fixed_bytes(gemm_tg(c.tm)) + 2 * gemm_slot_bytes(16, c.tm) <= (size_t) kGemmSmemLimit;
}

cudaError_t launch_gemm_staged(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const uint8_t * xrec,
                               int64_t M, float * y, size_t y_stride, cudaStream_t stream, int sm_count, bool pdl) {
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
    const int tg         = gemm_tg(c.tm);
    const size_t fixed   = gemm_fixed_bytes(tg);
    // Rows per unit: fewer, larger units share each activation record among
    // more rows; more units fill more SMs.  Cost ~ units per CTA x (rows +
    // a fixed share for the record and the unit's combine step).
    int    best_rb   = 16;
    double best_cost = 1e300;
    for (int rb = 16; rb <= 128; rb *= 2) {
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
    const size_t slot = gemm_slot_bytes(a.rb, c.tm);
    a.n_slots        = (int) std::min<size_t>(kGemmMaxSlots, ((size_t) kGemmSmemLimit - fixed) / slot);
    if (a.n_slots < 2) {
        return cudaErrorInvalidValue;
    }
    const size_t smem = fixed + (size_t) a.n_slots * slot;
    const int    grid = std::min(a.n_units, sm_count);
    cudaError_t  e;
    switch (tg) {
        case 2:
            e = cudaFuncSetAttribute(gemm_q8_0_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            return e != cudaSuccess ? e
                                    : launch_pdl(gemm_q8_0_kernel<2>, dim3((unsigned) grid), dim3(kGemmThreads), smem,
                                                 stream, pdl, a);
        case 4:
            e = cudaFuncSetAttribute(gemm_q8_0_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            return e != cudaSuccess ? e
                                    : launch_pdl(gemm_q8_0_kernel<4>, dim3((unsigned) grid), dim3(kGemmThreads), smem,
                                                 stream, pdl, a);
        default:
            e = cudaFuncSetAttribute(gemm_q8_0_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            return e != cudaSuccess ? e
                                    : launch_pdl(gemm_q8_0_kernel<8>, dim3((unsigned) grid), dim3(kGemmThreads), smem,
                                                 stream, pdl, a);
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
