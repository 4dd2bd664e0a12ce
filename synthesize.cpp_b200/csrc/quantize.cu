// quantize.cu -- F32 -> Q8_0 packing / activation quantization, Q8_0 -> F32
// dequantization and GET_ROWS for sm_100a.
//
// All three are HBM-bound byte work.  The packing kernel reads 1 KiB of fp32
// per warp iteration with two fully coalesced 16-byte loads per lane and
// writes one 272-byte run of eight blocks with 16-byte stores, so each warp
// touches whole 32-byte sectors on both sides.  Rows whose layout does not
// allow that (strided rows, unaligned pointers, a ragged tail) go through a
// warp-per-block kernel with the same arithmetic.
#include "common.cuh"
#include "kernels.h"

namespace b200q8 {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps   = kThreads / 32;

// Fast path: x is a dense run of n_blocks*32 floats (16-byte aligned), dst a
// dense run of n_blocks*34 bytes (16-byte aligned).  One warp per run of
// eight blocks; lane l holds floats [4l, 4l+4) and [128+4l, 128+4l+4), i.e.
// values 4*(l%8).. of blocks l/8 and 4 + l/8.
template <int MODE>
__global__ void __launch_bounds__(kThreads) quantize_dense_kernel(const float4 * __restrict__ x,
                                                                  uint8_t * __restrict__ dst, int64_t n_super) {
    __shared__ __align__(16) uint8_t stage[kWarps][kSuperBytes];
    const int      warp = threadIdx.x / 32;
    const int      lane = threadIdx.x % 32;
    const int      g    = lane % 8;
    uint8_t *      s    = stage[warp];
    const int64_t  step = (int64_t) gridDim.x * kWarps;
    for (int64_t sb = (int64_t) blockIdx.x * kWarps + warp; sb < n_super; sb += step) {
        const float4 a = __ldcs(x + sb * 64 + lane);
        const float4 b = __ldcs(x + sb * 64 + 32 + lane);
        float        va[4] = { a.x, a.y, a.z, a.w };
        float        vb[4] = { b.x, b.y, b.z, b.w };
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float(&v)[4]   = half ? vb : va;
            const float       am = block_amax<8, 4>(v, g);
            const QuantParams p  = quant_params<MODE>(am);
            uint32_t          w  = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                w |= (uint32_t) (quant_code<MODE>(v[e], p.id) & 0xff) << (8 * e);
            }
            const int blk = half * 4 + lane / 8;
            const int off = blk * kBlockBytes + 2 + 4 * g;  // 2-byte aligned
            *reinterpret_cast<uint16_t *>(s + off)     = (uint16_t) (w & 0xffffu);
            *reinterpret_cast<uint16_t *>(s + off + 2) = (uint16_t) (w >> 16);
            if (g == 0) {
                *reinterpret_cast<uint16_t *>(s + blk * kBlockBytes) = p.dbits;
            }
        }
        __syncwarp();
        if (lane < kSuperBytes / 16) {
            const uint4 v = *reinterpret_cast<const uint4 *>(s + 16 * lane);
            __stcs(reinterpret_cast<uint4 *>(dst + sb * kSuperBytes) + lane, v);
        }
        __syncwarp();
    }
}

// General path: one warp per block, lane j holds value j.  Row r of x at
// x + r*x_stride bytes, its block b written at dst + r*dst_stride + 34*b.
template <int MODE>
__global__ void __launch_bounds__(kThreads) quantize_general_kernel(const uint8_t * __restrict__ x, size_t x_stride,
                                                                    uint8_t * __restrict__ dst, size_t dst_stride,
                                                                    int64_t rows, int64_t nb, int64_t first_block) {
    const int     warp  = threadIdx.x / 32;
    const int     lane  = threadIdx.x % 32;
    const int64_t total = rows * nb;
    const int64_t step  = (int64_t) gridDim.x * kWarps;
    for (int64_t i = first_block + (int64_t) blockIdx.x * kWarps + warp; i < total; i += step) {
        const int64_t r     = i / nb;
        const int64_t b     = i % nb;
        const float * xr    = reinterpret_cast<const float *>(x + r * x_stride) + b * kQK;
        float         v[1]  = { xr[lane] };
        const float   am    = block_amax<32, 1>(v, lane);
        const QuantParams p = quant_params<MODE>(am);
        uint8_t *     out   = dst + r * dst_stride + b * kBlockBytes;
        out[2 + lane]       = (uint8_t) (quant_code<MODE>(v[0], p.id) & 0xff);
        if (lane == 0) {
            out[0] = (uint8_t) (p.dbits & 0xffu);
            out[1] = (uint8_t) (p.dbits >> 8);
        }
    }
}

// GET_ROWS / dequantize: one warp per block, lane j writes value j.
__global__ void __launch_bounds__(kThreads) dequant_rows_kernel(const uint8_t * __restrict__ src, size_t src_stride,
                                                                int64_t src_rows, const int32_t * __restrict__ ids,
                                                                int64_t n_out, int64_t nb, float * __restrict__ out,
                                                                size_t out_stride) {
    const int     warp  = threadIdx.x / 32;
    const int     lane  = threadIdx.x % 32;
    const int64_t total = n_out * nb;
    const int64_t step  = (int64_t) gridDim.x * kWarps;
    for (int64_t i = (int64_t) blockIdx.x * kWarps + warp; i < total; i += step) {
        const int64_t o   = i / nb;
        const int64_t b   = i % nb;
        const int64_t r   = ids ? (int64_t) ids[o] : o;
        float *       dst = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(out) + o * out_stride) + b * kQK;
        if (r < 0 || r >= src_rows) {
            dst[lane] = 0.0f;
            if (lane == 0 && b == 0) {
                record_device_error((unsigned) B200Q8_ERR_INVALID_ARG);
            }
            continue;
        }
        const uint8_t * blk = src + r * src_stride + b * kBlockBytes;
        const unsigned short dbits = (unsigned short) (blk[0] | (blk[1] << 8));
        const float          d     = __half2float(__ushort_as_half(dbits));
        dst[lane]                  = __fmul_rn((float) (int8_t) blk[2 + lane], d);
    }
}

// 16-bit sources (F16 / BF16): each value is widened to fp32 exactly, as the
// quantize tool's dequantize_to_f32 does (tools/synthesize-quantize/
// quantize.cpp:67-83), and then quantized exactly like an F32 source.
template <int SRC>
__device__ __forceinline__ float widen16(uint32_t bits) {
    return SRC == kSrcF16 ? __half2float(__ushort_as_half((unsigned short) bits)) : __uint_as_float(bits << 16);
}

// Dense 16-bit rows: the F32 dense kernel's layout, lane l holding values
// [4l, 4l+4) and [128+4l, 128+4l+4) of a 256-value run as two 8-byte loads.
template <int MODE, int SRC>
__global__ void __launch_bounds__(kThreads) quantize_dense16_kernel(const uint2 * __restrict__ x,
                                                                    uint8_t * __restrict__ dst, int64_t n_super) {
    __shared__ __align__(16) uint8_t stage[kWarps][kSuperBytes];
    const int     warp = threadIdx.x / 32;
    const int     lane = threadIdx.x % 32;
    const int     g    = lane % 8;
    uint8_t *     s    = stage[warp];
    const int64_t step = (int64_t) gridDim.x * kWarps;
    for (int64_t sb = (int64_t) blockIdx.x * kWarps + warp; sb < n_super; sb += step) {
        const uint2 a     = __ldcs(x + sb * 64 + lane);
        const uint2 b     = __ldcs(x + sb * 64 + 32 + lane);
        float       va[4] = { widen16<SRC>(a.x & 0xffffu), widen16<SRC>(a.x >> 16), widen16<SRC>(a.y & 0xffffu),
                              widen16<SRC>(a.y >> 16) };
        float       vb[4] = { widen16<SRC>(b.x & 0xffffu), widen16<SRC>(b.x >> 16), widen16<SRC>(b.y & 0xffffu),
                              widen16<SRC>(b.y >> 16) };
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float(&v)[4]   = half ? vb : va;
            const float       am = block_amax<8, 4>(v, g);
            const QuantParams p  = quant_params<MODE>(am);
            uint32_t          w  = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                w |= (uint32_t) (quant_code<MODE>(v[e], p.id) & 0xff) << (8 * e);
            }
            const int blk = half * 4 + lane / 8;
            const int off = blk * kBlockBytes + 2 + 4 * g;
            *reinterpret_cast<uint16_t *>(s + off)     = (uint16_t) (w & 0xffffu);
            *reinterpret_cast<uint16_t *>(s + off + 2) = (uint16_t) (w >> 16);
            if (g == 0) {
                *reinterpret_cast<uint16_t *>(s + blk * kBlockBytes) = p.dbits;
            }
        }
        __syncwarp();
        if (lane < kSuperBytes / 16) {
            const uint4 v = *reinterpret_cast<const uint4 *>(s + 16 * lane);
            __stcs(reinterpret_cast<uint4 *>(dst + sb * kSuperBytes) + lane, v);
        }
        __syncwarp();
    }
}

// General 16-bit path: one warp per block, lane j holds value j.
template <int MODE, int SRC>
__global__ void __launch_bounds__(kThreads) quantize_general16_kernel(const uint8_t * __restrict__ x, size_t x_stride,
                                                                      uint8_t * __restrict__ dst, size_t dst_stride,
                                                                      int64_t rows, int64_t nb, int64_t first_block) {
    const int     warp  = threadIdx.x / 32;
    const int     lane  = threadIdx.x % 32;
    const int64_t total = rows * nb;
    const int64_t step  = (int64_t) gridDim.x * kWarps;
    for (int64_t i = first_block + (int64_t) blockIdx.x * kWarps + warp; i < total; i += step) {
        const int64_t      r    = i / nb;
        const int64_t      b    = i % nb;
        const uint16_t *   xr   = reinterpret_cast<const uint16_t *>(x + r * x_stride) + b * kQK;
        float              v[1] = { widen16<SRC>(xr[lane]) };
        const float        am   = block_amax<32, 1>(v, lane);
        const QuantParams  p    = quant_params<MODE>(am);
        uint8_t *          out  = dst + r * dst_stride + b * kBlockBytes;
        out[2 + lane]           = (uint8_t) (quant_code<MODE>(v[0], p.id) & 0xff);
        if (lane == 0) {
            out[0] = (uint8_t) (p.dbits & 0xffu);
            out[1] = (uint8_t) (p.dbits >> 8);
        }
    }
}

int grid_for(int64_t warps_of_work, int sm_count) {
    const int64_t ctas = (warps_of_work + kWarps - 1) / kWarps;
    const int64_t cap  = (int64_t) sm_count * 8;
    return (int) (ctas < 1 ? 1 : (ctas > cap ? cap : ctas));
}

template <int MODE>
cudaError_t launch_quantize_mode(const float * x, int64_t rows, int64_t K, size_t x_stride, void * dst,
                                 size_t dst_stride, cudaStream_t stream, int sm_count) {
    const int64_t nb       = K / kQK;
    const bool    dense    = x_stride == (size_t) K * 4 && dst_stride == (size_t) nb * kBlockBytes;
    const bool    aligned  = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0);
    int64_t       first_gen = 0;
    if (dense && aligned) {
        const int64_t n_super = rows * nb / kSuperBlocks;
        if (n_super > 0) {
            quantize_dense_kernel<MODE><<<grid_for(n_super, sm_count), kThreads, 0, stream>>>(
                reinterpret_cast<const float4 *>(x), reinterpret_cast<uint8_t *>(dst), n_super);
        }
        first_gen = n_super * kSuperBlocks;  // ragged tail, if any, below
        if (first_gen == rows * nb) {
            return cudaGetLastError();
        }
        // The tail is addressed as one dense row of all blocks.
        quantize_general_kernel<MODE><<<grid_for(rows * nb - first_gen, sm_count), kThreads, 0, stream>>>(
            reinterpret_cast<const uint8_t *>(x), (size_t) rows * nb * kQK * 4, reinterpret_cast<uint8_t *>(dst),
            (size_t) rows * nb * kBlockBytes, 1, rows * nb, first_gen);
        return cudaGetLastError();
    }
    quantize_general_kernel<MODE><<<grid_for(rows * nb, sm_count), kThreads, 0, stream>>>(
        reinterpret_cast<const uint8_t *>(x), x_stride, reinterpret_cast<uint8_t *>(dst), dst_stride, rows, nb, 0);
    return cudaGetLastError();
}

template <int MODE, int SRC>
cudaError_t launch_quantize16_mode(const void * x, int64_t rows, int64_t K, size_t x_stride, void * dst,
                                   size_t dst_stride, cudaStream_t stream, int sm_count) {
    const int64_t nb        = K / kQK;
    const bool    dense     = x_stride == (size_t) K * 2 && dst_stride == (size_t) nb * kBlockBytes;
    const bool    aligned   = (reinterpret_cast<uintptr_t>(x) % 8 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0);
    int64_t       first_gen = 0;
    if (dense && aligned) {
        const int64_t n_super = rows * nb / kSuperBlocks;
        if (n_super > 0) {
            quantize_dense16_kernel<MODE, SRC><<<grid_for(n_super, sm_count), kThreads, 0, stream>>>(
                reinterpret_cast<const uint2 *>(x), reinterpret_cast<uint8_t *>(dst), n_super);
        }
        first_gen = n_super * kSuperBlocks;
        if (first_gen == rows * nb) {
            return cudaGetLastError();
        }
        quantize_general16_kernel<MODE, SRC><<<grid_for(rows * nb - first_gen, sm_count), kThreads, 0, stream>>>(
            reinterpret_cast<const uint8_t *>(x), (size_t) rows * nb * kQK * 2, reinterpret_cast<uint8_t *>(dst),
            (size_t) rows * nb * kBlockBytes, 1, rows * nb, first_gen);
        return cudaGetLastError();
    }
    quantize_general16_kernel<MODE, SRC><<<grid_for(rows * nb, sm_count), kThreads, 0, stream>>>(
        reinterpret_cast<const uint8_t *>(x), x_stride, reinterpret_cast<uint8_t *>(dst), dst_stride, rows, nb, 0);
    return cudaGetLastError();
}

template <int SRC>
cudaError_t launch_quantize16(const void * x, int64_t rows, int64_t K, size_t x_stride, void * dst, size_t dst_stride,
                              int mode, cudaStream_t stream, int sm_count) {
    switch (mode) {
        case B200Q8_QUANT_REF:
            return launch_quantize16_mode<B200Q8_QUANT_REF, SRC>(x, rows, K, x_stride, dst, dst_stride, stream, sm_count);
        case B200Q8_QUANT_CPU_X86:
            return launch_quantize16_mode<B200Q8_QUANT_CPU_X86, SRC>(x, rows, K, x_stride, dst, dst_stride, stream,
                                                                     sm_count);
        default:
            return launch_quantize16_mode<B200Q8_QUANT_CPU_ARM, SRC>(x, rows, K, x_stride, dst, dst_stride, stream,
                                                                     sm_count);
    }
}

}  // namespace

cudaError_t launch_quantize_typed(const void * x, int src_type, int64_t rows, int64_t K, size_t x_stride, void * dst,
                                  size_t dst_stride, int mode, cudaStream_t stream, int sm_count) {
    switch (src_type) {
        case kSrcF32:
            return launch_quantize(static_cast<const float *>(x), rows, K, x_stride, dst, dst_stride, mode, stream,
                                   sm_count);
        case kSrcF16: return launch_quantize16<kSrcF16>(x, rows, K, x_stride, dst, dst_stride, mode, stream, sm_count);
        case kSrcBF16: return launch_quantize16<kSrcBF16>(x, rows, K, x_stride, dst, dst_stride, mode, stream, sm_count);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_quantize(const float * x, int64_t rows, int64_t K, size_t x_stride, void * dst, size_t dst_stride,
                            int mode, cudaStream_t stream, int sm_count) {
    switch (mode) {
        case B200Q8_QUANT_REF:
            return launch_quantize_mode<B200Q8_QUANT_REF>(x, rows, K, x_stride, dst, dst_stride, stream, sm_count);
        case B200Q8_QUANT_CPU_X86:
            return launch_quantize_mode<B200Q8_QUANT_CPU_X86>(x, rows, K, x_stride, dst, dst_stride, stream,
                                                              sm_count);
        default:
            return launch_quantize_mode<B200Q8_QUANT_CPU_ARM>(x, rows, K, x_stride, dst, dst_stride, stream,
                                                              sm_count);
    }
}

cudaError_t launch_dequant_rows(const void * src, size_t src_stride, int64_t src_rows, const int32_t * ids,
                                int64_t n_out, int64_t K, float * out, size_t out_stride, cudaStream_t stream,
                                int sm_count) {
    const int64_t nb = K / kQK;
    if (n_out * nb == 0) {
        return cudaSuccess;
    }
    dequant_rows_kernel<<<grid_for(n_out * nb, sm_count), kThreads, 0, stream>>>(
        reinterpret_cast<const uint8_t *>(src), src_stride, src_rows, ids, n_out, nb, out, out_stride);
    return cudaGetLastError();
}

}  // namespace b200q8
