// gemm_tc.cu -- Q8_0 x F32 MUL_MAT for large M on the 5th-generation tensor
// cores (tcgen05.mma kind::i8, sm_100a).
//
// y[m][n] = sum_b fp32(dw[n,b]) * fp32(dx[m,b]) * sum_{i<32} qw[n,32b+i] * qx[m,32b+i]
//
// Two byte passes lay both operands out as planes: int8 codes [rows][K] and
// fp32 scales [K/32][rows] (the weights' from their Q8_0 rows, the
// activations' from the same quantizer as every other path), and for the
// activations also -1.5 * 2^23 * dx, which is exact in fp32 (dx is an fp16
// value: 3 * dx needs 13 significant bits).  A persistent
// kernel then works on tiles of 128 weight rows x 128 tokens:
//  * one producer thread loads, per stage of four Q8_0 blocks (128 bytes of
//    K), each operand's codes as one 2-D TMA box of 128 bytes x 128 rows with
//    the 128-byte swizzle -- the K-major SWIZZLE_128B layout the MMA reads --
//    and the tile's scales (one box each);
//  * one MMA thread issues, per Q8_0 block (K = 32), one
//    tcgen05.mma.cta_group::1.kind::i8 of M = 128, N = 128 into one of four
//    TMEM accumulators of 128 columns.  An accumulator holds the bit pattern
//    of the float 1.5 * 2^23 (0x4B400000) before each MMA and the MMA adds
//    the block's int32 sums to it, so each word reads as 1.5 * 2^23 + sum
//    exactly (|sum| <= 32 * 128 * 128 < 2^22);
//  * sixteen epilogue warps read each block's accumulator with tcgen05.ld and
//    rescale in fp32 on the CUDA cores, in block order:
//    u = fma(v, dx, -1.5 * 2^23 * dx) is (v - 1.5 * 2^23) * dx = sum * dx with
//    one rounding, then acc = fma(u, dw, acc) -- two packed f32x2
//    instructions per pair of outputs --
//    and write the bias back with tcgen05.st.  Accumulators pass between the
//    MMA thread and the epilogue two blocks at a time (one barrier wait and
//    one hand-back per pair), the pair going back when the next pair starts.
// The scales change every 32 values of K, so every block's sums are rescaled
// on the CUDA cores: the tensor pipe takes over the MMA issue and the operand
// loads, the fp32 rescale stays where the mma.sync path has it.
//
// Every wait is bounded; a timeout records B200Q8_ERR_DEVICE_TIMEOUT, sets
// the CTA's stop flag (every role then skips its remaining waits), waits
// (bounded) for the CTA's own copies and MMAs in flight, frees the TMEM and
// returns.  Copies are never multicast.
#include "common.cuh"
#include "kernels.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

namespace b200q8 {
namespace {

constexpr int kTcRows       = 128;  // weight rows per tile (MMA M, TMEM lanes)
constexpr int kTcToks       = 128;  // tokens per tile (MMA N, TMEM columns per accumulator)
constexpr int kTcKB         = 4;    // Q8_0 blocks per pipeline stage: 128 bytes of K, one swizzle row
constexpr int kTcStages     = 5;
constexpr int kTcBufs       = 4;    // TMEM accumulators, handed over in pairs (two blocks per hand-off)
constexpr int kTcPairs      = kTcBufs / 2;
constexpr int kTcTmemCols   = kTcBufs * kTcToks;  // 512: all of an SM's TMEM
constexpr int kTcEpiWarps   = 16;   // 4 per TMEM lane quarter, 32 accumulator columns each
constexpr int kTcEpiCols    = kTcToks * 4 / kTcEpiWarps;
constexpr int kTcThreads    = (2 + kTcEpiWarps) * 32;
constexpr int kTcCodeBytes  = 128 * kTcKB * 32;                      // 16 KiB per operand per stage
constexpr int kTcScaleBytes = kTcKB * 128 * 4;                       // 2 KiB per operand per stage
constexpr int kTcStageBytes = 2 * kTcCodeBytes + 3 * kTcScaleBytes;  // 38 KiB: codes, dw, dx, -B * dx
constexpr int kTcHeader     = 1024;
constexpr int kTcSmem       = kTcHeader + 1024 + kTcStages * kTcStageBytes;  // + slack to a 1 KiB boundary
constexpr int kTcMaxK       = 65536;
constexpr int kTcMaxM       = 1 << 20;

static_assert(kTcSmem <= 227 * 1024, "shared memory per CTA");
static_assert(kTcStageBytes % 1024 == 0 && kTcCodeBytes % 1024 == 0, "swizzle atoms start on 1 KiB boundaries");
static_assert(kTcEpiCols == 32, "one 32-column accumulator slice per epilogue warp and block");

struct TcArgs {
    int     K, N, M;
    int     n_nt;     // row tiles = ceil(N / 128)
    int     n_tiles;  // n_nt * ceil(M / 128)
    float * y;
    size_t  y_stride;  // floats between tokens
};

// 2-D tiled TMA load of the box at (x, y) (x in elements, x * element size a
// multiple of 16 bytes) into this CTA's shared memory, completing on `bar`;
// the box counts in full, elements outside the tensor read as 0.  Never
// multicast.
__device__ __forceinline__ void tc_tma_2d(void * dst_smem, const CUtensorMap * map, int x, int y, uint64_t * bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst_smem)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Shared-memory matrix descriptor, sm100 version 1, K-major, 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), the
// leading byte offset 16 (unused inside one swizzle row), layout type 2.  The
// start address steps by 32 bytes per Q8_0 block inside the 128-byte row;
// the swizzle atoms start on 1 KiB boundaries, so the base offset is 0.
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t) ((saddr >> 4) & 0x3fffu);
    d |= (uint64_t) (16u >> 4) << 16;
    d |= (uint64_t) (1024u >> 4) << 32;
    d |= (uint64_t) 1u << 46;
    d |= (uint64_t) 2u << 61;
    return d;
}

// Instruction descriptor, kind::i8: s32 accumulator, s8 x s8, both K-major,
// N = kTcToks, M = kTcRows.
__host__ __device__ constexpr uint32_t tc_idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (kTcToks >> 3) << 17) |
           ((uint32_t) (kTcRows >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b) {
    // accumulate onto what the accumulator holds (the bias word); no lanes masked
    const uint32_t z = 0, one = 1;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%4, %4, %4, %4}, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(tc_idesc()), "r"(z), "r"(one)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 16 consecutive accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

// The bias word into 32 consecutive accumulator columns of this warp's lanes.
__device__ __forceinline__ void tc_st32_bias(uint32_t taddr) {
    const uint32_t b = 0x4B400000u;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
        "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
        "r"(b)
        : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Bounded wait on the critical path (no suspend hint, so a completed phase is
// seen at once); gives up when *stop becomes non-zero.
__device__ __forceinline__ bool tc_wait(uint64_t * bar, uint32_t parity, const int * stop) {
    if (mbar_test_wait(bar, parity)) {
        return true;
    }
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*(volatile const int *) stop != 0 || clock64() - start > kWaitLimitCycles) {
            return false;
        }
    }
    return true;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap wc_map,
                   const __grid_constant__ CUtensorMap xc_map, const __grid_constant__ CUtensorMap wd_map,
                   const __grid_constant__ CUtensorMap xd_map, const __grid_constant__ CUtensorMap xn_map) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t * full      = reinterpret_cast<uint64_t *>(smem);  // stage landed (TMA)
    uint64_t * empty     = full + kTcStages;                     // stage read (MMA commit + epilogue warps)
    uint64_t * tfull     = empty + kTcStages;                    // accumulator pair written (MMA commit)
    uint64_t * tempty    = tfull + kTcPairs;                     // accumulator pair re-biased (epilogue warps)
    uint64_t * mma_done  = tempty + kTcPairs;                    // every MMA issued has completed
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    int *      stop      = reinterpret_cast<int *>(tmem_slot + 1);
    // stages start on the first 1 KiB boundary after the header (swizzle atoms)
    const uint32_t pad    = (1024u - ((smem_addr(smem) + (uint32_t) kTcHeader) & 1023u)) & 1023u;
    uint8_t *      stages = smem + kTcHeader + pad;

    const int warp     = threadIdx.x >> 5;
    const int lane     = threadIdx.x & 31;
    const int n_kc     = a.K / (32 * kTcKB);  // stages per tile
    const int G        = gridDim.x;
    const int my_tiles = (int) blockIdx.x < a.n_tiles ? (a.n_tiles - (int) blockIdx.x + G - 1) / G : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + kTcEpiWarps);
        }
        for (int p = 0; p < kTcPairs; ++p) {
            mbar_init(&tfull[p], 1);
            mbar_init(&tempty[p], kTcEpiWarps);
        }
        mbar_init(mma_done, 1);
        *stop = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    auto           fail  = [&]() {
        record_device_error((unsigned) B200Q8_ERR_DEVICE_TIMEOUT);
        *(volatile int *) stop = 1;
    };

    if (warp == 0) {
        if (lane == 0) {
            // producer: stage ci of the CTA's (tile, K range) sequence uses slot ci % S
            const uint64_t pol = l2_evict_last_policy();
            int            ci  = 0;
            for (int it = 0; it < my_tiles && *(volatile int *) stop == 0; ++it) {
                const int t  = (int) blockIdx.x + it * G;
                const int n0 = (t % a.n_nt) * kTcRows;
                const int t0 = (t / a.n_nt) * kTcToks;
                for (int kc = 0; kc < n_kc; ++kc, ++ci) {
                    const int s = ci % kTcStages;
                    const int n = ci / kTcStages;
                    if (n >= 1 && !mbar_wait_bounded_or_flag(&empty[s], (uint32_t) ((n - 1) & 1), stop)) {
                        if (*(volatile int *) stop == 0) fail();
                        break;
                    }
                    uint8_t * st  = stages + (size_t) s * kTcStageBytes;
                    const int kb0 = kc * kTcKB;
                    mbar_arrive_expect_tx(&full[s], (uint32_t) kTcStageBytes);
                    tc_tma_2d(st, &wc_map, kb0 * 32, n0, &full[s], pol);
                    tc_tma_2d(st + kTcCodeBytes, &xc_map, kb0 * 32, t0, &full[s], pol);
                    tc_tma_2d(st + 2 * kTcCodeBytes, &wd_map, n0, kb0, &full[s], pol);
                    tc_tma_2d(st + 2 * kTcCodeBytes + kTcScaleBytes, &xd_map, t0, kb0, &full[s], pol);
                    tc_tma_2d(st + 2 * kTcCodeBytes + 2 * kTcScaleBytes, &xn_map, t0, kb0, &full[s], pol);
                }
            }
            // copies still in flight land before the CTA leaves: the last fill of each slot
            for (int s = 0; s < kTcStages && s < ci; ++s) {
                const int last = (ci - 1 - s) / kTcStages * kTcStages + s;  // last ci' < ci with ci' % S == s
                (void) mbar_wait_bounded(&full[s], (uint32_t) ((last / kTcStages) & 1));
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: one MMA per Q8_0 block into accumulator bi % 4; pair (bi / 2) % 2
            // is waited for before its first block and committed after its second
            int  ci = 0, bi = 0;
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                for (int kc = 0; kc < n_kc && ok; ++kc, ++ci) {
                    const int s = ci % kTcStages;
                    if (!tc_wait(&full[s], (uint32_t) ((ci / kTcStages) & 1), stop)) {
                        if (*(volatile int *) stop == 0) fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(stages + (size_t) s * kTcStageBytes);
#pragma unroll 1
                    for (int j = 0; j < kTcKB; ++j, ++bi) {
                        const int b = bi % kTcBufs;
                        const int p = b >> 1;
                        if ((bi & 1) == 0) {
                            // the MMA thread runs ahead of the epilogue and mostly waits here: a
                            // suspending wait leaves its SMSP's issue slots to the epilogue warps
                            if (!mbar_wait_bounded_or_flag(&tempty[p], (uint32_t) ((bi / kTcBufs) & 1), stop)) {
                                if (*(volatile int *) stop == 0) fail();
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                        tc_mma(tbase + (uint32_t) (b * kTcToks), tc_desc_sw128(sa + 32 * j),
                               tc_desc_sw128(sa + kTcCodeBytes + 32 * j));
                        if (bi & 1) {
                            tc_commit(&tfull[p]);
                        }
                    }
                    if (ok) {
                        tc_commit(&empty[s]);
                    }
                }
            }
            // every MMA issued completes before the TMEM is freed
            tc_commit(mma_done);
            (void) mbar_wait_bounded(mma_done, 0);
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (tile rows) and
        // accumulator columns 32 * ((w - 2) / 4) .. + 31 (tokens)
        const int      q  = warp & 3;
        const int      cg = (warp - 2) >> 2;
        const int      r  = 32 * q + lane;
        const uint32_t tl = tbase + ((uint32_t) (32 * q) << 16) + (uint32_t) (cg * kTcEpiCols);
#pragma unroll 1
        for (int b = 0; b < kTcBufs; ++b) {
            tc_st32_bias(tl + b * kTcToks);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            for (int p = 0; p < kTcPairs; ++p) {
                mbar_arrive(&tempty[p]);
            }
        }
        int          ci = 0, bi = 0;
        int          held = -1;  // accumulator pair re-biased (tcgen05.st issued) but not yet handed back
        bool         ok   = true;
        // hand the held pair back to the MMA thread once its bias stores completed
        auto release = [&]() {
            if (held >= 0) {
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty[held]);
                }
                held = -1;
            }
        };
        for (int it = 0; it < my_tiles; ++it) {
            const int t  = (int) blockIdx.x + it * G;
            const int n0 = (t % a.n_nt) * kTcRows;
            const int t0 = (t / a.n_nt) * kTcToks;
            float2    acc[kTcEpiCols / 2];
#pragma unroll
            for (int i = 0; i < kTcEpiCols / 2; ++i) {
                acc[i] = make_float2(0.0f, 0.0f);
            }
            for (int kc = 0; kc < n_kc; ++kc, ++ci) {
                const int s = ci % kTcStages;
                if (ok && !tc_wait(&full[s], (uint32_t) ((ci / kTcStages) & 1), stop)) {
                    if (*(volatile int *) stop == 0) fail();
                    ok = false;
                }
                ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld / st need the whole warp
                const uint8_t * st = stages + (size_t) s * kTcStageBytes;
                const float *   wd = reinterpret_cast<const float *>(st + 2 * kTcCodeBytes);
                const float *   xd = wd + kTcKB * 128;
                const float *   xn = xd + kTcKB * 128;
#pragma unroll 1
                for (int j = 0; j < kTcKB; j += 2, bi += 2) {
                    const int p = (bi % kTcBufs) >> 1;
                    if (ok && !tc_wait(&tfull[p], (uint32_t) ((bi / kTcBufs) & 1), stop)) {
                        if (*(volatile int *) stop == 0) fail();
                        ok = false;
                    }
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) {
                        continue;
                    }
                    tc_fence_after();
                    release();  // the previous pair
#pragma unroll 1
                    for (int q2 = 0; q2 < 2; ++q2) {
                        const int      jb  = j + q2;
                        const int      b   = 2 * p + q2;
                        const float    dw  = wd[jb * 128 + r];
                        const float2   dw2 = make_float2(dw, dw);
                        const float4 * dx  = reinterpret_cast<const float4 *>(xd + jb * 128 + cg * kTcEpiCols);
                        const float4 * dn  = reinterpret_cast<const float4 *>(xn + jb * 128 + cg * kTcEpiCols);
                        // two halves of 16 columns: the scales first, then the accumulator words
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float4 d[4], e[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                d[i] = dx[4 * h + i];
                                e[i] = dn[4 * h + i];
                            }
                            uint32_t v[16];
                            tc_ld16(tl + b * kTcToks + 16 * h, v);
                            tc_wait_ld();
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float2 u0 = __ffma2_rn(
                                    make_float2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])),
                                    make_float2(d[i].x, d[i].y), make_float2(e[i].x, e[i].y));
                                const float2 u1 = __ffma2_rn(
                                    make_float2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])),
                                    make_float2(d[i].z, d[i].w), make_float2(e[i].z, e[i].w));
                                const int a0 = 8 * h + 2 * i;
                                acc[a0]      = __ffma2_rn(u0, dw2, acc[a0]);
                                acc[a0 + 1]  = __ffma2_rn(u1, dw2, acc[a0 + 1]);
                            }
                        }
                        // back to the bias; the pair is handed back when the next one starts (or below)
                        tc_st32_bias(tl + b * kTcToks);
                    }
                    held = p;
                }
                __syncwarp();
                if (ok && lane == 0) {
                    mbar_arrive(&empty[s]);
                }
            }
            release();
            // tokens t0 + 32 * cg + i of row n0 + r: a warp's 32 rows are one 128-byte run per token
            const int row = n0 + r;
            if (ok && *(volatile int *) stop == 0 && row < a.N) {
                float * yb = a.y + row;
#pragma unroll
                for (int i = 0; i < kTcEpiCols / 2; ++i) {
                    const int tok = t0 + cg * kTcEpiCols + 2 * i;
                    if (tok < a.M) {
                        yb[(size_t) tok * a.y_stride] = acc[i].x;
                    }
                    if (tok + 1 < a.M) {
                        yb[(size_t) (tok + 1) * a.y_stride] = acc[i].y;
                    }
                }
            }
        }
        tc_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTcTmemCols));
    }
}

// Weights: Q8_0 rows -> codes [N][K] and fp32 scales [K/32][pitch].  One
// warp per (row, 256-wide chunk): lanes 0..16 load the chunk's 272 bytes,
// lane l writes codes 8l .. 8l + 7 (block l / 4) as one 8-byte store.
__global__ void __launch_bounds__(256) tc_repack_weights_kernel(const uint8_t * __restrict__ w, size_t row_bytes,
                                                                int K, int N, uint8_t * __restrict__ codes,
                                                                float * __restrict__ scales, int pitch) {
    __shared__ __align__(16) uint8_t stage[8][kSuperBytes];
    const int     warp  = threadIdx.x >> 5;
    const int     lane  = threadIdx.x & 31;
    const int     n_ch  = K / 256;
    const int64_t total = (int64_t) N * n_ch;
    uint8_t *     s     = stage[warp];
    for (int64_t u = (int64_t) blockIdx.x * 8 + warp; u < total; u += (int64_t) gridDim.x * 8) {
        const int64_t n = u / n_ch;
        const int     c = (int) (u - n * n_ch);
        if (lane < kSuperBytes / 16) {
            reinterpret_cast<uint4 *>(s)[lane] =
                __ldcs(reinterpret_cast<const uint4 *>(w + (size_t) n * row_bytes + (size_t) c * kSuperBytes) + lane);
        }
        __syncwarp();
        const int       blk = lane >> 2;
        const uint8_t * src = s + blk * kBlockBytes + 2 + (lane & 3) * 8;  // 2-byte aligned
        uint64_t        v   = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v |= (uint64_t) *reinterpret_cast<const uint16_t *>(src + 2 * i) << (16 * i);
        }
        *reinterpret_cast<uint64_t *>(codes + (size_t) n * K + (size_t) c * 256 + 8 * lane) = v;
        if ((lane & 3) == 0) {
            const __half d = *reinterpret_cast<const __half *>(s + blk * kBlockBytes);
            scales[(size_t) (c * 8 + blk) * pitch + n] = __half2float(d);
        }
        __syncwarp();
    }
}

// Activations: F32 rows (16-byte aligned, stride a multiple of 4 floats) ->
// codes [M][K] and fp32 scales [K/32][pitch], quantized as every other path
// quantizes them (quant_params / quant_code of the call's mode).  One warp
// per (token, 256-wide chunk): lane l holds values 4(l % 8) .. + 3 of blocks
// l / 8 and 4 + l / 8.
template <int MODE>
__global__ void __launch_bounds__(256) tc_stage_acts_kernel(const float * __restrict__ x, size_t x_stride, int K,
                                                            int M, uint8_t * __restrict__ codes,
                                                            float * __restrict__ scales, float * __restrict__ nbscales,
                                                            int pitch) {
    const int     warp  = threadIdx.x >> 5;
    const int     lane  = threadIdx.x & 31;
    const int     g     = lane & 7;
    const int     n_ch  = K / 256;
    const int64_t total = (int64_t) M * n_ch;
    for (int64_t u = (int64_t) blockIdx.x * 8 + warp; u < total; u += (int64_t) gridDim.x * 8) {
        const int64_t  m     = u / n_ch;
        const int      c     = (int) (u - m * n_ch);
        const float4 * xr    = reinterpret_cast<const float4 *>(x + (size_t) m * x_stride + (size_t) c * 256);
        const float4   a0    = __ldcs(xr + lane);
        const float4   a1    = __ldcs(xr + 32 + lane);
        const float    va[4] = { a0.x, a0.y, a0.z, a0.w };
        const float    vb[4] = { a1.x, a1.y, a1.z, a1.w };
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float(&v)[4]   = half ? vb : va;
            const float       am = block_amax<8, 4>(v, g);
            const QuantParams p  = quant_params<MODE>(am);
            uint32_t          wv = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                wv |= (uint32_t) (quant_code<MODE>(v[e], p.id) & 0xff) << (8 * e);
            }
            const int blk = half * 4 + (lane >> 3);
            *reinterpret_cast<uint32_t *>(codes + (size_t) m * K + (size_t) c * 256 + half * 128 + 4 * lane) = wv;
            if (g == 0) {
                scales[(size_t) (c * 8 + blk) * pitch + m]   = p.d;
                nbscales[(size_t) (c * 8 + blk) * pitch + m] = -12582912.0f * p.d;  // exact: see the top
            }
        }
    }
}

struct TcPlanes {
    uint8_t * wc;
    float *   wd;
    uint8_t * xc;
    float *   xd;
    float *   xn;  // -1.5 * 2^23 * xd
    int       pitch_n, pitch_m;
    size_t    bytes;
};

size_t tc_align(size_t v) {
    return (v + 255) / 256 * 256;
}

TcPlanes tc_planes(void * ws, int64_t K, int64_t N, int64_t M) {
    TcPlanes p = {};
    p.pitch_n  = (int) ((N + 3) / 4 * 4);
    p.pitch_m  = (int) ((M + 3) / 4 * 4);
    size_t    off  = 0;
    uint8_t * base = static_cast<uint8_t *>(ws);
    p.wc           = base + off;
    off += tc_align((size_t) N * (size_t) K);
    p.wd = reinterpret_cast<float *>(base + off);
    off += tc_align((size_t) (K / 32) * (size_t) p.pitch_n * 4);
    p.xc = base + off;
    off += tc_align((size_t) M * (size_t) K);
    p.xd = reinterpret_cast<float *>(base + off);
    off += tc_align((size_t) (K / 32) * (size_t) p.pitch_m * 4);
    p.xn = reinterpret_cast<float *>(base + off);
    off += tc_align((size_t) (K / 32) * (size_t) p.pitch_m * 4);
    p.bytes = off;
    return p;
}

// rows x K int8 codes, box 128 bytes x 128 rows, 128-byte swizzle
bool tc_encode_codes(CUtensorMap * map, const uint8_t * codes, int64_t K, int64_t rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) {
        return false;
    }
    const cuuint64_t dims[2]    = { (cuuint64_t) K, (cuuint64_t) rows };
    const cuuint64_t strides[1] = { (cuuint64_t) K };
    const cuuint32_t box[2]     = { (cuuint32_t) (kTcKB * 32), 128 };
    const cuuint32_t estr[2]    = { 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(codes), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K/32 x rows fp32 scales (row pitch `pitch` floats), box 128 rows x kTcKB blocks
bool tc_encode_scales(CUtensorMap * map, const float * scales, int64_t K, int64_t rows, int pitch) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) {
        return false;
    }
    const cuuint64_t dims[2]    = { (cuuint64_t) rows, (cuuint64_t) (K / 32) };
    const cuuint64_t strides[1] = { (cuuint64_t) pitch * 4 };
    const cuuint32_t box[2]     = { 128, kTcKB };
    const cuuint32_t estr[2]    = { 1, 1 };
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(scales), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int byte_pass_grid(int64_t warps, int sm_count) {
    const int64_t ctas = (warps + 7) / 8;
    return (int) std::max<int64_t>(1, std::min<int64_t>(ctas, (int64_t) sm_count * 8));
}

}  // namespace

// Smallest M that b200q8_mul_mat sends to the tcgen05 GEMM.  Off (0) by
// default: the mma.sync GEMM is faster at every M measured.
// B200Q8_TC_MIN_M=<M> turns it on from that M (read once per process).
int64_t gemm_tc_min_m() {
    static const int64_t v = [] {
        const char * e = getenv("B200Q8_TC_MIN_M");
        return e != nullptr && e[0] != '\0' ? (int64_t) strtoll(e, nullptr, 10) : (int64_t) 0;
    }();
    return v;
}

bool gemm_tc_supported(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, int64_t M, const float * x,
                       size_t x_stride) {
    return M >= 1 && M <= kTcMaxM && N >= 1 && N <= (int64_t) 1 << 30 && K >= 256 && K % 256 == 0 && K <= kTcMaxK &&
           row_bytes % 16 == 0 && row_bytes >= (size_t) (K / kQK) * kBlockBytes &&
           reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
           (M == 1 || x_stride % 4 == 0) && (int64_t) N * K < ((int64_t) 1 << 40);
}

size_t gemm_tc_workspace_bytes(int64_t K, int64_t N, int64_t M) {
    return tc_planes(nullptr, K, N, M).bytes;
}

cudaError_t launch_gemm_tc(const uint8_t * w, size_t row_bytes, int64_t K, int64_t N, const float * x,
                           size_t x_stride, int64_t M, float * y, size_t y_stride, int mode, void * workspace,
                           cudaStream_t stream, int sm_count) {
    const TcPlanes p = tc_planes(workspace, K, N, M);
    tc_repack_weights_kernel<<<byte_pass_grid(N * (K / 256), sm_count), 256, 0, stream>>>(
        w, row_bytes, (int) K, (int) N, p.wc, p.wd, p.pitch_n);
    const int ga = byte_pass_grid(M * (K / 256), sm_count);
    switch (mode) {
        case B200Q8_QUANT_REF:
            tc_stage_acts_kernel<B200Q8_QUANT_REF>
                <<<ga, 256, 0, stream>>>(x, x_stride, (int) K, (int) M, p.xc, p.xd, p.xn, p.pitch_m);
            break;
        case B200Q8_QUANT_CPU_X86:
            tc_stage_acts_kernel<B200Q8_QUANT_CPU_X86>
                <<<ga, 256, 0, stream>>>(x, x_stride, (int) K, (int) M, p.xc, p.xd, p.xn, p.pitch_m);
            break;
        default:
            tc_stage_acts_kernel<B200Q8_QUANT_CPU_ARM>
                <<<ga, 256, 0, stream>>>(x, x_stride, (int) K, (int) M, p.xc, p.xd, p.xn, p.pitch_m);
            break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return e;
    }
    CUtensorMap wc_map, xc_map, wd_map, xd_map, xn_map;
    if (!tc_encode_codes(&wc_map, p.wc, K, N) || !tc_encode_codes(&xc_map, p.xc, K, M) ||
        !tc_encode_scales(&wd_map, p.wd, K, N, p.pitch_n) || !tc_encode_scales(&xd_map, p.xd, K, M, p.pitch_m) ||
        !tc_encode_scales(&xn_map, p.xn, K, M, p.pitch_m)) {
        return cudaErrorInvalidValue;
    }
    TcArgs a   = {};
    a.K        = (int) K;
    a.N        = (int) N;
    a.M        = (int) M;
    a.n_nt     = (int) ((N + kTcRows - 1) / kTcRows);
    a.n_tiles  = (int) std::min<int64_t>((int64_t) a.n_nt * ((M + kTcToks - 1) / kTcToks), INT32_MAX);
    a.y        = y;
    a.y_stride = y_stride;
    e          = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) {
        return e;
    }
    const int grid = std::max(1, std::min(a.n_tiles, sm_count));
    gemm_tc_kernel<<<grid, kTcThreads, kTcSmem, stream>>>(a, wc_map, xc_map, wd_map, xd_map, xn_map);
    return cudaGetLastError();
}

}  // namespace b200q8
