// gemm.cu -- Q8_0 x F32 MUL_MAT for M > 8 tokens on int8 tensor cores (sm_100a).
//
// y[m][n] = sum_b fp32(dw[n,b]) * fp32(dx[m,b]) * sum_{i<32} qw[n,32b+i] * qx[m,32b+i]
//
// One Q8_0 block is exactly the K = 32 of one mma.sync.m16n8k32 s8 x s8 -> s32,
// so each MMA yields the exact int32 block sums of a 16-row x 8-token tile,
// which are rescaled by dw*dx in fp32 registers (the scale differs per block,
// so the int32 accumulator cannot span blocks).  Weights are the 16-row A
// operand, streamed per 16-row tile through a shared-memory ring by 1-D bulk
// copies (never multicast); activations are quantized once per call into the
// workspace (codes plane [M][K] + fp32 scale plane [M][K/32]) and read as B
// fragments through the L1/L2.  Eight consumer warps split the token groups
// of 8 and, when there are few tokens, the K range; partial sums over K are
// combined through shared memory in a fixed order, so results are
// deterministic.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace b200q8 {
namespace {

constexpr int kGemmConsumerWarps = 8;
constexpr int kGemmThreads       = (kGemmConsumerWarps + 1) * 32;
constexpr int kGemmMaxSlots      = 4;
constexpr int kGemmSmemLimit     = 220 * 1024;

// Activations -> codes plane + fp32 scale plane (warp per block).
template <int MODE>
__global__ void __launch_bounds__(256) quantize_planes_kernel(const float * __restrict__ x, size_t x_stride, int64_t M,
                                                              int64_t NB, int8_t * __restrict__ codes,
                                                              float * __restrict__ scales) {
    const int     warp = threadIdx.x >> 5;
    const int     lane = threadIdx.x & 31;
    const int64_t step = (int64_t) gridDim.x * 8;
    for (int64_t i = (int64_t) blockIdx.x * 8 + warp; i < M * NB; i += step) {
        const int64_t     m     = i / NB;
        const int64_t     b     = i - m * NB;
        const float       v     = x[m * x_stride + b * kQK + lane];
        float             vv[1] = { v };
        const float       am    = block_amax<32, 1>(vv, lane);
        const QuantParams qp    = quant_params<MODE>(am);
        codes[(m * NB + b) * kQK + lane] = (int8_t) quant_code<MODE>(v, qp.id);
        if (lane == 0) {
            scales[m * NB + b] = qp.d;
        }
    }
}

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// 4 code bytes at byte offset `off` (2-byte aligned) of a shared-memory row.
__device__ __forceinline__ uint32_t lds_u32_at(uint32_t row, int off) {
    const uint32_t base = row + (uint32_t) (off & ~3);
    if ((off & 3) == 0) {
        return lds_u32(base);
    }
    return __byte_perm(lds_u32(base), lds_u32(base + 4), 0x5432);
}

struct GemmArgs {
    const uint8_t * w;
    size_t          row_bytes;
    int             K, N, M;
    const int8_t *  codes;   // [M][K]
    const float *   scales;  // [M][K/32]
    float *         y;
    size_t          y_stride;  // floats between tokens
    int             slot_bytes;
    int             n_slots;
    int             tg_per_warp;  // token groups of 8 handled per warp (looped)
    int             ksplit;       // warps sharing one token-group set, splitting K
};

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_q8_0_kernel(const GemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *     full       = reinterpret_cast<uint64_t *>(smem);
    uint64_t *     empty      = full + kGemmMaxSlots;
    volatile int * abort_flag = reinterpret_cast<volatile int *>(smem + 128);
    float *        red        = reinterpret_cast<float *>(smem + 256);  // K-split partials
    const int      red_floats = kGemmConsumerWarps * 32 * 4 * 4;       // per warp: 4 tg x 4 values x 32 lanes
    uint8_t *      ring       = smem + ((256 + red_floats * 4 + 127) & ~127);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int NB   = a.K >> 5;
    // this CTA's 16-row tiles
    const int n_rt  = (a.N + 15) >> 4;
    const int G     = gridDim.x;
    const int base  = n_rt / G;
    const int rem   = n_rt % G;
    const int rt0   = blockIdx.x * base + min((int) blockIdx.x, rem);
    const int nrt   = base + ((int) blockIdx.x < rem ? 1 : 0);
    const int S     = a.n_slots;

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
        // weights are constant: they may stream in before the previous kernel ends
        if (lane == 0) {
            const uint64_t pol    = l2_evict_first_policy();
            int            issued = 0;
            for (int t = 0; t < nrt; ++t) {
                const int s = t % S;
                if (t >= S && !mbar_wait_bounded_sleep(&empty[s], ((t / S) - 1) & 1)) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) {
                    break;
                }
                const int      r0    = (rt0 + t) * 16;
                const int      rows  = min(16, a.N - r0);
                const uint32_t bytes = (uint32_t) (rows * a.row_bytes);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_copy_g2s(ring + (size_t) s * a.slot_bytes, a.w + (size_t) r0 * a.row_bytes, bytes, &full[s], pol);
                ++issued;
            }
            for (int t = max(0, issued - S); t < issued; ++t) {
                if (!mbar_wait_bounded(&full[t % S], (t / S) & 1)) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                }
            }
        }
        return;
    }

    // consumer warp roles: token-group set (tgs) and K slice (ks)
    const int ks    = warp % a.ksplit;
    const int tgs   = warp / a.ksplit;  // token groups tgs*tg_per_warp .. +tg_per_warp
    const int b_per = (NB + a.ksplit - 1) / a.ksplit;
    const int b0    = ks * b_per;
    const int b1    = min(NB, b0 + b_per);
    const int g     = lane >> 2;
    const int tq    = lane & 3;
    const uint32_t ring_s = smem_addr(ring);

    pdl_wait_primary();  // activations come from the previous kernel
    // Every consumer warp runs the same loop trip counts and reaches the same
    // named barriers whatever happens: a timed-out wait or a token group past
    // M only skips work, it never leaves the loop early.
    bool fail = false;
    for (int t = 0; t < nrt; ++t) {
        const int s = t % S;
        if (!fail && !mbar_wait_bounded(&full[s], (t / S) & 1)) {
            record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
            *abort_flag = 1;
            fail        = true;
        }
        fail = __any_sync(0xffffffffu, fail);  // mma.sync needs the whole warp: decide per warp
        const int      r0     = (rt0 + t) * 16;
        const int      rows   = min(16, a.N - r0);
        const uint32_t tile   = ring_s + (uint32_t) (s * a.slot_bytes);
        const int      ra     = min(g, rows - 1);      // clamp rows past N (results discarded)
        const int      rb     = min(g + 8, rows - 1);
        const uint32_t row_a  = tile + (uint32_t) (ra * a.row_bytes);
        const uint32_t row_b  = tile + (uint32_t) (rb * a.row_bytes);
        for (int tgi = 0; tgi < a.tg_per_warp; ++tgi) {
            const int     tg     = tgs * a.tg_per_warp + tgi;
            const int     n0     = tg * 8;
            const bool    work   = !fail && n0 < a.M;          // warp-uniform
            const int     tok    = min(n0 + g, a.M - 1);      // B column this lane loads
            const int     tok0   = n0 + 2 * tq;                // D columns this lane owns
            const int8_t *xrow   = a.codes + (size_t) tok * a.K;
            const float * sc0    = a.scales + (size_t) min(tok0, a.M - 1) * NB;
            const float * sc1    = a.scales + (size_t) min(tok0 + 1, a.M - 1) * NB;
            float         acc[4] = { 0.f, 0.f, 0.f, 0.f };
            // Eight blocks per step: all of their activation fragments and
            // scales are requested from L2 before the first MMA, so the loads
            // overlap instead of costing one L2 round trip per block.
            for (int bb = b0; work && bb < b1; bb += 8) {
                const int nb8 = min(8, b1 - bb);
                uint32_t  Bf[8][2];
                float     x0s[8], x1s[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int b = bb + (j < nb8 ? j : 0);
                    Bf[j][0]    = __ldg(reinterpret_cast<const uint32_t *>(xrow + b * kQK + 4 * tq));
                    Bf[j][1]    = __ldg(reinterpret_cast<const uint32_t *>(xrow + b * kQK + 16 + 4 * tq));
                    x0s[j]      = __ldg(sc0 + b);
                    x1s[j]      = __ldg(sc1 + b);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (j < nb8) {
                        const int b   = bb + j;
                        const int off = b * kBlockBytes + 2;
                        uint32_t  A[4];
                        A[0] = lds_u32_at(row_a, off + 4 * tq);
                        A[1] = lds_u32_at(row_b, off + 4 * tq);
                        A[2] = lds_u32_at(row_a, off + 16 + 4 * tq);
                        A[3] = lds_u32_at(row_b, off + 16 + 4 * tq);
                        int            D[4] = { 0, 0, 0, 0 };
                        const uint32_t Bj[2] = { Bf[j][0], Bf[j][1] };
                        mma_s8(D, A, Bj);
                        const uint32_t wa = lds_u32(row_a + (uint32_t) ((b * kBlockBytes) & ~3));
                        const uint32_t wb = lds_u32(row_b + (uint32_t) ((b * kBlockBytes) & ~3));
                        const float    da = __half2float(__ushort_as_half(
                            (unsigned short) (((b * kBlockBytes) & 3) ? (wa >> 16) : (wa & 0xffffu))));
                        const float db = __half2float(__ushort_as_half(
                            (unsigned short) (((b * kBlockBytes) & 3) ? (wb >> 16) : (wb & 0xffffu))));
                        acc[0] = __fmaf_rn((float) D[0], __fmul_rn(da, x0s[j]), acc[0]);
                        acc[1] = __fmaf_rn((float) D[1], __fmul_rn(da, x1s[j]), acc[1]);
                        acc[2] = __fmaf_rn((float) D[2], __fmul_rn(db, x0s[j]), acc[2]);
                        acc[3] = __fmaf_rn((float) D[3], __fmul_rn(db, x1s[j]), acc[3]);
                    }
                }
            }
            // combine the K slices in a fixed order: slice 0 adds 1..ksplit-1
            if (a.ksplit > 1) {
                float * mine = red + ((size_t) (warp * 4 + tgi) * 32 + lane) * 4;
                if (ks != 0) {
                    mine[0] = acc[0];
                    mine[1] = acc[1];
                    mine[2] = acc[2];
                    mine[3] = acc[3];
                }
                named_barrier_sync(1, kGemmConsumerWarps * 32);
                if (ks == 0) {
                    for (int k2 = 1; k2 < a.ksplit; ++k2) {
                        const float * o = red + ((size_t) ((warp + k2) * 4 + tgi) * 32 + lane) * 4;
                        acc[0] += o[0];
                        acc[1] += o[1];
                        acc[2] += o[2];
                        acc[3] += o[3];
                    }
                }
                named_barrier_sync(1, kGemmConsumerWarps * 32);
            }
            if (ks == 0 && work) {
                const int rA = r0 + g;
                const int rB = r0 + g + 8;
                if (tok0 < a.M) {
                    if (g < rows) a.y[(size_t) tok0 * a.y_stride + rA] = acc[0];
                    if (g + 8 < rows) a.y[(size_t) tok0 * a.y_stride + rB] = acc[2];
                }
                if (tok0 + 1 < a.M) {
                    if (g < rows) a.y[(size_t) (tok0 + 1) * a.y_stride + rA] = acc[1];
                    if (g + 8 < rows) a.y[(size_t) (tok0 + 1) * a.y_stride + rB] = acc[3];
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty[s]);
        }
    }
}

// Per-token prologue of the batched step: one CTA per token builds that
// token's fp32 input of the next MUL_MAT and quantizes it into the code and
// scale planes the GEMM reads.  kind: 0 = RMS norm of (a [+ b]) (the sum is
// also written to sum_out when given), 1 = GQA expansion of a, 2 = silu(a)*b.
template <int MODE>
__global__ void __launch_bounds__(256) stage_rows_kernel(int kind, const float * __restrict__ a, const float * __restrict__ b,
                                                         size_t ab_stride, float * __restrict__ sum_out,
                                                         size_t sum_stride, const float * __restrict__ norm, float eps,
                                                         int K, int head_dim, int group, float * __restrict__ trace,
                                                         size_t trace_stride, int8_t * __restrict__ codes,
                                                         float * __restrict__ scales) {
    __shared__ float  xs[8192];
    __shared__ double part[8];
    __shared__ float  scale_s;
    pdl_launch_dependents();
    pdl_wait_primary();
    const int     m    = blockIdx.x;
    const int     t    = threadIdx.x;
    const float * am   = a + (size_t) m * ab_stride;
    const float * bm   = b ? b + (size_t) m * ab_stride : nullptr;
    double        ss   = 0.0;
    for (int i = t; i < K; i += 256) {
        float v;
        if (kind == 0) {
            v = bm ? __fadd_rn(am[i], bm[i]) : am[i];
            if (sum_out) {
                sum_out[(size_t) m * sum_stride + i] = v;
            }
            ss += (double) __fmul_rn(v, v);
        } else if (kind == 1) {
            const int head = i / head_dim;
            v              = am[(head / group) * head_dim + i % head_dim];
        } else {
            v = __fmul_rn(silu_f32(am[i]), bm[i]);
        }
        xs[i] = v;
    }
    if (kind == 0) {
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
            for (int w = 0; w < 8; ++w) {
                tot += part[w];
            }
            const float mean = (float) (tot / (double) K);
            scale_s          = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
        }
        __syncthreads();
        const float sc = scale_s;
        for (int i = t; i < K; i += 256) {
            xs[i] = __fmul_rn(__fmul_rn(xs[i], sc), norm[i]);
        }
    }
    __syncthreads();
    const int warp = t >> 5;
    const int lane = t & 31;
    const int NB   = K >> 5;
    for (int blk = warp; blk < NB; blk += 8) {
        const float       v     = xs[blk * kQK + lane];
        float             vv[1] = { v };
        const float       amx   = block_amax<32, 1>(vv, lane);
        const QuantParams qp    = quant_params<MODE>(amx);
        codes[((size_t) m * NB + blk) * kQK + lane] = (int8_t) quant_code<MODE>(v, qp.id);
        if (lane == 0) {
            scales[(size_t) m * NB + blk] = qp.d;
        }
        if (trace) {
            trace[(size_t) m * trace_stride + blk * kQK + lane] = v;
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

}  // namespace

cudaError_t launch_stage_rows(int kind, const float * a, const float * b, size_t ab_stride, float * sum_out,
                              size_t sum_stride, const float * norm, float eps, int K, int head_dim, int group,
                              float * trace, size_t trace_stride, int64_t M, int mode, int8_t * codes, float * scales,
                              cudaStream_t stream, bool pdl) {
    if (K > 8192 || K % kQK) {
        return cudaErrorInvalidValue;
    }
    switch (mode) {
        case B200Q8_QUANT_CPU_X86:
            return launch_pdl(stage_rows_kernel<B200Q8_QUANT_CPU_X86>, dim3((unsigned) M), dim3(256), 0, stream, pdl,
                              kind, a, b, ab_stride, sum_out, sum_stride, norm, eps, K, head_dim, group, trace,
                              trace_stride, codes, scales);
        case B200Q8_QUANT_CPU_ARM:
            return launch_pdl(stage_rows_kernel<B200Q8_QUANT_CPU_ARM>, dim3((unsigned) M), dim3(256), 0, stream, pdl,
                              kind, a, b, ab_stride, sum_out, sum_stride, norm, eps, K, head_dim, group, trace,
                              trace_stride, codes, scales);
        default:
            return launch_pdl(stage_rows_kernel<B200Q8_QUANT_REF>, dim3((unsigned) M), dim3(256), 0, stream, pdl, kind,
                              a, b, ab_stride, sum_out, sum_stride, norm, eps, K, head_dim, group, trace, trace_stride,
                              codes, scales);
    }
}

cudaError_t launch_residual_rows(const float * a, const float * b, size_t ab_stride, float * out, size_t out_stride,
                                 int K, int64_t M, cudaStream_t stream, bool pdl) {
    return launch_pdl(residual_rows_kernel, dim3((unsigned) M), dim3(256), 0, stream, pdl, a, b, ab_stride, out,
                      out_stride, K);
}

size_t gemm_workspace_bytes(int64_t K, int64_t M) {
    const size_t codes = (size_t) M * (size_t) K;
    return ((codes + 255) & ~(size_t) 255) + (size_t) M * (size_t) (K / kQK) * 4;
}

bool gemm_supported(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, int64_t M) {
    if (M < 1 || M > 1024 || N < 1 || K < 256 || K % 256 != 0 || row_bytes % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(w) % 16) != 0) {
        return false;
    }
    const size_t slot  = 16 * row_bytes;
    const size_t fixed = (size_t) ((256 + kGemmConsumerWarps * 32 * 4 * 4 * 4 + 127) & ~127);
    return fixed + slot <= (size_t) kGemmSmemLimit;
}

cudaError_t launch_gemm_planes(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const int8_t * codes,
                               const float * scales, int64_t M, float * y, size_t y_stride, cudaStream_t stream,
                               int sm_count, bool pdl) {
    GemmArgs a   = {};
    a.w          = w;
    a.row_bytes  = row_bytes;
    a.K          = (int) K;
    a.N          = (int) N;
    a.M          = (int) M;
    a.codes      = codes;
    a.scales     = scales;
    a.y          = y;
    a.y_stride   = y_stride;
    a.slot_bytes = (int) (16 * row_bytes);
    const int n_tg = (int) ((M + 7) / 8);
    // few tokens: split K across warps; many: loop token groups per warp
    a.ksplit      = n_tg >= kGemmConsumerWarps ? 1 : std::max(1, kGemmConsumerWarps / n_tg);
    while (kGemmConsumerWarps % a.ksplit) {
        --a.ksplit;
    }
    const int sets  = kGemmConsumerWarps / a.ksplit;
    a.tg_per_warp   = (n_tg + sets - 1) / sets;
    if (a.tg_per_warp > 4 && a.ksplit > 1) {
        a.ksplit = 1;
    }
    const size_t fixed = (size_t) ((256 + kGemmConsumerWarps * 32 * 4 * 4 * 4 + 127) & ~127);
    a.n_slots          = (int) std::min<size_t>(kGemmMaxSlots, ((size_t) kGemmSmemLimit - fixed) / a.slot_bytes);
    if (a.n_slots < 1) {
        return cudaErrorInvalidValue;
    }
    const size_t  smem = fixed + (size_t) a.n_slots * a.slot_bytes;
    const int64_t n_rt = (N + 15) / 16;
    const int     grid = (int) std::min<int64_t>(n_rt, sm_count);
    cudaError_t   e    = cudaFuncSetAttribute(gemm_q8_0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) {
        return e;
    }
    return launch_pdl(gemm_q8_0_kernel, dim3((unsigned) grid), dim3(kGemmThreads), smem, stream, pdl, a);
}

void gemm_planes(void * workspace, int64_t K, int64_t M, int8_t ** codes, float ** scales) {
    *codes  = static_cast<int8_t *>(workspace);
    *scales = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) +
                                        (((size_t) M * (size_t) K + 255) & ~(size_t) 255));
}

cudaError_t launch_gemm(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const float * x, size_t x_stride,
                        int64_t M, float * y, size_t y_stride, int mode, void * workspace, cudaStream_t stream,
                        int sm_count) {
    const int64_t NB = K / kQK;
    int8_t *      codes;
    float *       scales;
    gemm_planes(workspace, K, M, &codes, &scales);
    {
        const int64_t warps = M * NB;
        int64_t       ctas  = std::min<int64_t>((warps + 7) / 8, (int64_t) sm_count * 8);
        ctas                = std::max<int64_t>(ctas, 1);
        switch (mode) {
            case B200Q8_QUANT_CPU_X86:
                quantize_planes_kernel<B200Q8_QUANT_CPU_X86><<<(unsigned) ctas, 256, 0, stream>>>(x, x_stride, M, NB,
                                                                                                  codes, scales);
                break;
            case B200Q8_QUANT_CPU_ARM:
                quantize_planes_kernel<B200Q8_QUANT_CPU_ARM><<<(unsigned) ctas, 256, 0, stream>>>(x, x_stride, M, NB,
                                                                                                  codes, scales);
                break;
            default:
                quantize_planes_kernel<B200Q8_QUANT_REF><<<(unsigned) ctas, 256, 0, stream>>>(x, x_stride, M, NB, codes,
                                                                                              scales);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            return e;
        }
    }
    return launch_gemm_planes(w, row_bytes, K, N, codes, scales, M, y, y_stride, stream, sm_count, false);
}

}  // namespace b200q8
