// gemv.cu -- Q8_0 x F32 decode GEMV (M <= 8 tokens) for sm_100a.
//
// y[m][n] = sum_b fp32(dw[n,b]) * fp32(dx[m,b]) * sum_i qw[n,32b+i]*qx[m,32b+i]
//
// This is the arithmetic of ggml-cpu's MUL_MAT for a Q8_0 weight: the F32
// activations are first quantized to Q8_0 (from_float), then every output is
// vec_dot_q8_0_q8_0 of a weight row with a token (reference call sites:
// src/arch/qwen3-tts/operations.cpp:39-41,90-92,142, talker.cpp:45,48,184,
// code-predictor.cpp:79).
//
// Design (HBM-bound; 1.0625 weight bytes per multiply-add at M = 1):
//  * one CTA per SM owns a contiguous, balanced range of weight rows;
//  * a producer warp streams that range into a ring of shared-memory slots
//    with 1-D bulk copies (cp.async.bulk, mbarrier complete_tx, L2
//    evict-first); the slots are whole rows, so a slot is 16-byte aligned
//    whenever K % 256 == 0;
//  * eight consumer warps first quantize the activations into shared memory
//    (bit-exact with the reference quantizer, every CTA redundantly: K <= a
//    few thousand floats read from L2), optionally deriving them from the
//    previous op (RMS norm, GQA expansion, SwiGLU) on the way;
//  * then each weight row is split over a group of lanes by 68-byte block
//    pairs (4-byte aligned): two blocks' codes come out of 17 shared-memory
//    words with byte_perm, dp4a gives each block's exact int32 sum, the
//    fp32 scale product is applied per block and the group reduces with
//    shuffles;
//  * weights are read before griddepcontrol.wait, so in a chain launched with
//    programmatic dependent launch each op's weights stream in while the
//    previous op finishes.
#include "common.cuh"
#include "kernels.h"
#include "tile_dot.cuh"

#include <algorithm>
#include <atomic>

namespace b200q8 {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers     = kConsumerWarps * 32;
constexpr int kGemvThreads   = kConsumers + 32;  // + one producer warp
constexpr int kSlotTarget    = 16384;
constexpr int kMaxSlots      = 6;
constexpr int kSmemLimit     = 112 * 1024;  // two CTAs per SM stay possible
constexpr int kHeaderBytes   = 1024;        // barriers, flags, rms partials

struct Layout {
    int slot_rows;
    int slot_bytes;
    int n_slots;
    int x_codes_bytes;
    int x_scale_bytes;
    int ring_off;
    int smem_bytes;
};

bool make_layout(int K, size_t row_bytes, int rows_per_cta, int mt, Layout & L) {
    if (rows_per_cta < 1 || row_bytes == 0) {
        return false;
    }
    int sr = (int) (kSlotTarget / row_bytes);
    sr     = std::max(sr, 1);
    sr     = std::min(sr, rows_per_cta);
    L.slot_rows      = sr;
    L.slot_bytes     = (int) (sr * row_bytes);
    const int tiles  = (rows_per_cta + sr - 1) / sr;
    L.x_codes_bytes  = mt * K;
    L.x_scale_bytes  = mt * (K / kQK) * 4;
    L.ring_off       = (kHeaderBytes + L.x_codes_bytes + L.x_scale_bytes + 127) & ~127;
    const int budget = kSmemLimit - L.ring_off;
    if (budget < L.slot_bytes) {
        return false;
    }
    L.n_slots    = std::min(std::min(kMaxSlots, tiles), budget / L.slot_bytes);
    L.smem_bytes = L.ring_off + L.n_slots * L.slot_bytes;
    return L.n_slots >= 1;
}

template <int M_T, int MODE, int PRO>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_q8_0_kernel(const GemvParams p, const Layout L) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *     full       = reinterpret_cast<uint64_t *>(smem);
    uint64_t *     empty      = full + kMaxSlots;
    volatile int * abort_flag = reinterpret_cast<volatile int *>(smem + 128);
    float *        rms_scale  = reinterpret_cast<float *>(smem + 192);         // [M_T]
    double *       rms_part   = reinterpret_cast<double *>(smem + 256);        // [kConsumerWarps][M_T]
    uint8_t *      xc         = smem + kHeaderBytes;                           // codes
    float *        xd         = reinterpret_cast<float *>(xc + L.x_codes_bytes);  // scales
    uint8_t *      ring       = smem + L.ring_off;

    const int warp  = threadIdx.x / 32;
    const int lane  = threadIdx.x % 32;
    const int K     = p.K;
    const int NB    = K / kQK;
    const int P     = K / 64;
    const int G     = gridDim.x;
    const int base  = p.N / G;
    const int rem   = p.N % G;
    const int r0    = blockIdx.x * base + min((int) blockIdx.x, rem);
    const int nrows = base + ((int) blockIdx.x < rem ? 1 : 0);
    const int n_tiles = (nrows + L.slot_rows - 1) / L.slot_rows;
    const int S       = L.n_slots;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ---------------- producer: stream this CTA's rows through the ring
        if (lane == 0) {
            const uint64_t pol    = l2_evict_first_policy();
            int            issued = 0;
            for (int t = 0; t < n_tiles; ++t) {
                const int s = t % S;
                if (t >= S && !mbar_wait_bounded(&empty[s], ((t / S) - 1) & 1)) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) {
                    break;
                }
                const int      tr0   = t * L.slot_rows;
                const int      R     = min(L.slot_rows, nrows - tr0);
                const uint32_t bytes = (uint32_t) (R * p.row_bytes);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_copy_g2s(ring + (size_t) s * L.slot_bytes, p.w + (size_t) (r0 + tr0) * p.row_bytes, bytes,
                              &full[s], pol);
                ++issued;
            }
            // Never leave with a copy in flight into this CTA's shared memory.
            for (int t = max(0, issued - S); t < issued; ++t) {
                if (!mbar_wait_bounded(&full[t % S], (t / S) & 1)) {
                    record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
                }
            }
        }
        return;
    }

    // -------------------- consumers: activation prologue (needs the inputs)
    pdl_wait_primary();
    const int M = p.M;
    if (PRO == kProRmsNorm) {
        double ss[M_T];
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
            ss[m] = 0.0;
        }
        for (int i = threadIdx.x; i < K; i += kConsumers) {
#pragma unroll
            for (int m = 0; m < M_T; ++m) {
                if (m < M) {
                    const float v = p.x[(size_t) m * p.x_stride + i];
                    ss[m] += (double) __fmul_rn(v, v);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
            }
            if (lane == 0) {
                rms_part[warp * M_T + m] = ss[m];
            }
        }
        named_barrier_sync(1, kConsumers);
        if (threadIdx.x < M_T) {
            double tot = 0.0;
            for (int w = 0; w < kConsumerWarps; ++w) {
                tot += rms_part[w * M_T + threadIdx.x];
            }
            const float mean          = (float) (tot / (double) K);
            rms_scale[threadIdx.x]    = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, p.eps)));
        }
        named_barrier_sync(1, kConsumers);
    }

    // Warp w quantizes blocks w, w+8, ...; lane j holds value j of a block.
    // Loads are issued kChunk blocks at a time so they overlap in flight.
    constexpr int kChunk = 8;
    const int     NBM    = M * NB;
    for (int base_blk = warp; base_blk < NBM; base_blk += kConsumerWarps * kChunk) {
        float v[kChunk];
#pragma unroll
        for (int c = 0; c < kChunk; ++c) {
            const int blk = base_blk + c * kConsumerWarps;
            v[c]          = 0.0f;
            if (blk < NBM) {
                const int m   = blk / NB;
                const int idx = (blk % NB) * kQK + lane;
                if (PRO == kProPlain) {
                    v[c] = p.x[(size_t) m * p.x_stride + idx];
                } else if (PRO == kProRmsNorm) {
                    v[c] = __fmul_rn(__fmul_rn(p.x[(size_t) m * p.x_stride + idx], rms_scale[m]), p.norm_w[idx]);
                } else if (PRO == kProGqa) {
                    const int head = idx / p.head_dim;
                    v[c] = p.x[(size_t) m * p.x_stride + (head / p.group) * p.head_dim + idx % p.head_dim];
                } else {
                    const float gte = p.x[(size_t) m * p.x_stride + idx];
                    const float up  = p.x2[(size_t) m * p.x_stride + idx];
                    v[c]            = __fmul_rn(silu_f32(gte), up);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < kChunk; ++c) {
            const int blk = base_blk + c * kConsumerWarps;
            if (blk < NBM) {  // warp-uniform
                const int m = blk / NB;
                const int b = blk % NB;
                stage_activation_block<MODE>(v[c], m, b, lane, P, NB, xc, xd);
                if (p.pro_out != nullptr && blockIdx.x == 0) {
                    p.pro_out[(size_t) m * p.pro_out_stride + b * kQK + lane] = v[c];
                }
            }
        }
    }
    named_barrier_sync(1, kConsumers);

    // ------------------------------------------------------ consume tiles
    for (int t = 0; t < n_tiles; ++t) {
        const int s = t % S;
        if (!mbar_wait_bounded(&full[s], (t / S) & 1)) {
            record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
            *abort_flag = 1;
            break;
        }
        const int       tr0  = t * L.slot_rows;
        const int       R    = min(L.slot_rows, nrows - tr0);
        const uint8_t * tile = ring + (size_t) s * L.slot_bytes;
        dot_tile_rows<M_T>(tile, R, p.row_bytes, P, NB, xc, xd, M, warp, lane, kConsumerWarps,
                           [&](int rr, int m, float acc) {
                               const int n                           = r0 + tr0 + rr;
                               p.y[(size_t) m * p.y_stride + n] = acc;
                               if (p.y_res != nullptr) {
                                   p.y_res[(size_t) m * p.res_stride + n] =
                                       __fadd_rn(p.res[(size_t) m * p.res_stride + n], acc);
                               }
                           });
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty[s]);
        }
        if (*abort_flag) {
            break;
        }
    }
}

// ----------------------------------------------------------- generic path

__global__ void __launch_bounds__(256) gemv_generic_kernel(const uint8_t * __restrict__ w, size_t row_bytes,
                                                           int64_t NB, int64_t N, const uint8_t * __restrict__ xq,
                                                           int64_t M, float * __restrict__ y, size_t y_stride) {
    const int     warp = threadIdx.x / 32;
    const int     lane = threadIdx.x % 32;
    const int64_t step = (int64_t) gridDim.x * 8;
    for (int64_t i = (int64_t) blockIdx.x * 8 + warp; i < N * M; i += step) {
        const int64_t n   = i / M;
        const int64_t m   = i % M;
        float         acc = 0.0f;
        for (int64_t b = lane; b < NB; b += 32) {
            const uint8_t * wb = w + n * row_bytes + b * kBlockBytes;
            const uint8_t * xb = xq + (m * NB + b) * kBlockBytes;
            int             s  = 0;
#pragma unroll 8
            for (int j = 0; j < kQK; ++j) {
                s += (int) (int8_t) wb[2 + j] * (int) (int8_t) xb[2 + j];
            }
            const float dw = __half2float(__ushort_as_half((unsigned short) (wb[0] | (wb[1] << 8))));
            const float dx = __half2float(__ushort_as_half((unsigned short) (xb[0] | (xb[1] << 8))));
            acc            = __fmaf_rn((float) s, __fmul_rn(dw, dx), acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            acc += __shfl_xor_sync(0xffffffffu, acc, off);
        }
        if (lane == 0) {
            *reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(y) + m * y_stride + n * 4) = acc;
        }
    }
}

// ----------------------------------------------------------- dispatch

using KernelFn = void (*)(const GemvParams, const Layout);

template <int M_T, int MODE>
KernelFn pick_pro(int pro) {
    switch (pro) {
        case kProRmsNorm: return gemv_q8_0_kernel<M_T, MODE, kProRmsNorm>;
        case kProGqa: return gemv_q8_0_kernel<M_T, MODE, kProGqa>;
        case kProSwiGlu: return gemv_q8_0_kernel<M_T, MODE, kProSwiGlu>;
        default: return gemv_q8_0_kernel<M_T, MODE, kProPlain>;
    }
}

template <int M_T>
KernelFn pick_mode(int mode, int pro) {
    switch (mode) {
        case B200Q8_QUANT_CPU_X86: return pick_pro<M_T, B200Q8_QUANT_CPU_X86>(pro);
        case B200Q8_QUANT_CPU_ARM: return pick_pro<M_T, B200Q8_QUANT_CPU_ARM>(pro);
        default: return pick_pro<M_T, B200Q8_QUANT_REF>(pro);
    }
}

int mt_for(int M) {
    return M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
}

KernelFn pick(int M, int mode, int pro) {
    switch (mt_for(M)) {
        case 1: return pick_mode<1>(mode, pro);
        case 2: return pick_mode<2>(mode, pro);
        case 4: return pick_mode<4>(mode, pro);
        default: return pick_mode<8>(mode, pro);
    }
}

bool layout_for(const GemvParams & p, int sm_count, int & grid, Layout & L) {
    grid                   = std::min(p.N, sm_count);
    const int rows_per_cta = (p.N + grid - 1) / grid;
    return make_layout(p.K, p.row_bytes, rows_per_cta, mt_for(p.M), L);
}

}  // namespace

bool gemv_supported(const GemvParams & p) {
    if (p.M < 1 || p.M > 8 || p.N < 1 || p.K < 256 || p.K % 256 != 0 || p.row_bytes % 16 != 0 ||
        p.row_bytes < (size_t) (p.K / kQK) * kBlockBytes || (reinterpret_cast<uintptr_t>(p.w) % 16) != 0) {
        return false;
    }
    int    grid;
    Layout L;
    return layout_for(p, 148, grid, L);
}

cudaError_t launch_gemv(const GemvParams & p, cudaStream_t stream, int sm_count, bool pdl) {
    int    grid;
    Layout L;
    if (!layout_for(p, sm_count, grid, L)) {
        return cudaErrorInvalidValue;
    }
    KernelFn fn = pick(p.M, p.mode, p.pro);
    // Opt in to > 48 KiB of dynamic shared memory; idempotent and cheap.
    cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (err != cudaSuccess) {
        return err;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) grid);
    cfg.blockDim           = dim3(kGemvThreads);
    cfg.dynamicSmemBytes   = (size_t) L.smem_bytes;
    cfg.stream             = stream;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs                                          = attr;
        cfg.numAttrs                                       = 1;
    }
    return cudaLaunchKernelEx(&cfg, fn, p, L);
}

cudaError_t launch_gemv_generic(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const uint8_t * xq,
                                int64_t M, float * y, size_t y_stride_bytes, cudaStream_t stream) {
    const int64_t warps = N * M;
    int64_t       ctas  = (warps + 7) / 8;
    ctas                = std::min<int64_t>(std::max<int64_t>(ctas, 1), 148 * 16);
    gemv_generic_kernel<<<(unsigned) ctas, 256, 0, stream>>>(w, row_bytes, K / kQK, N, xq, M, y, y_stride_bytes);
    return cudaGetLastError();
}

}  // namespace b200q8
