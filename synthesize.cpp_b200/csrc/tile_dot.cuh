// tile_dot.cuh -- the inner product of a shared-memory tile of Q8_0 weight
// rows with shared-memory Q8_0 activations (int8 dp4a per block, fp32 scale),
// shared by the standalone GEMV and the persistent decode-step kernel.
//
// Activation layout in shared memory (written by stage_activation_block):
//   codes: for token m, block pair p (64 codes) and 16-byte chunk c (0..3),
//          the chunk lives at ((m*4 + c)*P + p)*16, so lanes reading
//          consecutive pairs touch consecutive 16-byte words (no bank
//          conflicts for 128-bit loads);
//   scales: fp32(fp16(d)) at [m*NB + b].
// Weight rows in the tile are ggml block_q8_0 rows (34-byte blocks); a lane
// reads one 68-byte block pair as 17 4-byte words, stride 17 words between
// lanes, which is conflict-free.
#pragma once

#include "common.cuh"

namespace b200q8 {

// Quantizes value v (lane = position in the block) of block b of token m
// and stores the code and scale in the layout above.  All 32 lanes call it.
template <int MODE>
__device__ __forceinline__ void stage_activation_block(float v, int m, int b, int lane, int P, int NB, uint8_t * xc,
                                                       float * xd) {
    float             vv[1] = { v };
    const float       am    = block_amax<32, 1>(vv, lane);
    const QuantParams qp    = quant_params<MODE>(am);
    const int         q     = quant_code<MODE>(v, qp.id);
    const int         pp    = b >> 1;
    const int         pos   = ((b & 1) << 5) + lane;
    const int         wi    = pos >> 2;
    xc[((size_t) (m * 4 + (wi >> 2)) * P + pp) * 16 + (wi & 3) * 4 + (pos & 3)] = (uint8_t) (q & 0xff);
    if (lane == 0) {
        xd[m * NB + b] = qp.d;
    }
}

// Dot products of the R rows of `tile` (row stride row_bytes, K = 64*P) with
// the M staged tokens.  Warps warp0..warp0+n_warps-1 share the rows; a group
// of GS lanes (GS = P rounded up to a power of two, at most 32) takes one
// row.  store(row, m, value) is called once per (row, token) by one lane.
template <int M_T, typename Store>
__device__ __forceinline__ void dot_tile_rows(const uint8_t * tile, int R, size_t row_bytes, int P, int NB,
                                              const uint8_t * xc, const float * xd, int M, int warp, int lane,
                                              int n_warps, Store && store) {
    // GS = P rounded up to a power of two, at most 32; shifts only (a runtime
    // integer division costs ~100 cycles of latency here)
    const int      lgs    = P <= 1 ? 0 : min(5, 32 - __clz(P - 1));
    const int      GS     = 1 << lgs;
    const int      RPW    = 32 >> lgs;
    const int      sub    = lane >> lgs;
    const int      gl     = lane & (GS - 1);
    const uint32_t xc_s   = smem_addr(xc);
    const uint32_t xd_s   = smem_addr(xd);
    const uint32_t tile_s = smem_addr(tile);
    for (int rb = warp * RPW; rb < R; rb += n_warps * RPW) {
        const int  rr     = rb + sub;
        const bool active = rr < R;
        float      acc[M_T];
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
            acc[m] = 0.0f;
        }
        if (active) {
            const uint32_t wr = tile_s + (uint32_t) ((size_t) rr * row_bytes);
            for (int pp = gl; pp < P; pp += GS) {
                uint32_t w[17];
#pragma unroll
                for (int k = 0; k < 17; ++k) {
                    w[k] = lds_u32(wr + (uint32_t) (68 * pp + 4 * k));
                }
                int qa[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    qa[i] = (int) __byte_perm(w[i], w[i + 1], 0x5432);
                }
                const float dA = __half2float(__ushort_as_half((unsigned short) (w[0] & 0xffffu)));
                const float dB = __half2float(__ushort_as_half((unsigned short) (w[8] >> 16)));
#pragma unroll
                for (int m = 0; m < M_T; ++m) {
                    if (m < M) {
                        const uint32_t xv = xc_s + (uint32_t) (((m * 4) * P + pp) * 16);
                        const uint4    x0 = lds_v4(xv);
                        const uint4    x1 = lds_v4(xv + (uint32_t) (P * 16));
                        const uint4    x2 = lds_v4(xv + (uint32_t) (2 * P * 16));
                        const uint4    x3 = lds_v4(xv + (uint32_t) (3 * P * 16));
                        const float2   dx = lds_f2(xd_s + (uint32_t) ((m * NB + 2 * pp) * 4));
                        int            sA = 0;
                        int            sB = 0;
                        int            tA = 0;
                        int            tB = 0;
                        // two independent chains per block halve the dp4a latency
                        sA = __dp4a(qa[0], (int) x0.x, sA);
                        tA = __dp4a(qa[1], (int) x0.y, tA);
                        sA = __dp4a(qa[2], (int) x0.z, sA);
                        tA = __dp4a(qa[3], (int) x0.w, tA);
                        sA = __dp4a(qa[4], (int) x1.x, sA);
                        tA = __dp4a(qa[5], (int) x1.y, tA);
                        sA = __dp4a(qa[6], (int) x1.z, sA);
                        tA = __dp4a(qa[7], (int) x1.w, tA);
                        sB = __dp4a((int) w[9], (int) x2.x, sB);
                        tB = __dp4a((int) w[10], (int) x2.y, tB);
                        sB = __dp4a((int) w[11], (int) x2.z, sB);
                        tB = __dp4a((int) w[12], (int) x2.w, tB);
                        sB = __dp4a((int) w[13], (int) x3.x, sB);
                        tB = __dp4a((int) w[14], (int) x3.y, tB);
                        sB = __dp4a((int) w[15], (int) x3.z, sB);
                        tB = __dp4a((int) w[16], (int) x3.w, tB);
                        acc[m] = __fmaf_rn((float) (sA + tA), __fmul_rn(dA, dx.x), acc[m]);
                        acc[m] = __fmaf_rn((float) (sB + tB), __fmul_rn(dB, dx.y), acc[m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
            for (int off = GS / 2; off > 0; off >>= 1) {
                acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], off);
            }
        }
        if (active && gl == 0) {
#pragma unroll
            for (int m = 0; m < M_T; ++m) {
                if (m < M) {
                    store(rr, m, acc[m]);
                }
            }
        }
    }
}

// This lane's partial dot product of one weight row (shared-window address
// `row`) with the M staged tokens, over block pairs gl, gl+GS, ... < P.
template <int M_T>
__device__ __forceinline__ void dot_row_partial(uint32_t row, int P, int NB, int gl, int GS, uint32_t xc_s,
                                                uint32_t xd_s, int M, float (&acc)[M_T]) {
    for (int pp = gl; pp < P; pp += GS) {
        uint32_t w[17];
#pragma unroll
        for (int k = 0; k < 17; ++k) {
            w[k] = lds_u32(row + (uint32_t) (68 * pp + 4 * k));
        }
        int qa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qa[i] = (int) __byte_perm(w[i], w[i + 1], 0x5432);
        }
        const float dA = __half2float(__ushort_as_half((unsigned short) (w[0] & 0xffffu)));
        const float dB = __half2float(__ushort_as_half((unsigned short) (w[8] >> 16)));
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
            if (m < M) {
                const uint32_t xv = xc_s + (uint32_t) (((m * 4) * P + pp) * 16);
                const uint4    x0 = lds_v4(xv);
                const uint4    x1 = lds_v4(xv + (uint32_t) (P * 16));
                const uint4    x2 = lds_v4(xv + (uint32_t) (2 * P * 16));
                const uint4    x3 = lds_v4(xv + (uint32_t) (3 * P * 16));
                const float2   dx = lds_f2(xd_s + (uint32_t) ((m * NB + 2 * pp) * 4));
                int            sA = 0, tA = 0, sB = 0, tB = 0;
                sA = __dp4a(qa[0], (int) x0.x, sA);
                tA = __dp4a(qa[1], (int) x0.y, tA);
                sA = __dp4a(qa[2], (int) x0.z, sA);
                tA = __dp4a(qa[3], (int) x0.w, tA);
                sA = __dp4a(qa[4], (int) x1.x, sA);
                tA = __dp4a(qa[5], (int) x1.y, tA);
                sA = __dp4a(qa[6], (int) x1.z, sA);
                tA = __dp4a(qa[7], (int) x1.w, tA);
                sB = __dp4a((int) w[9], (int) x2.x, sB);
                tB = __dp4a((int) w[10], (int) x2.y, tB);
                sB = __dp4a((int) w[11], (int) x2.z, sB);
                tB = __dp4a((int) w[12], (int) x2.w, tB);
                sB = __dp4a((int) w[13], (int) x3.x, sB);
                tB = __dp4a((int) w[14], (int) x3.y, tB);
                sB = __dp4a((int) w[15], (int) x3.z, sB);
                tB = __dp4a((int) w[16], (int) x3.w, tB);
                acc[m] = __fmaf_rn((float) (sA + tA), __fmul_rn(dA, dx.x), acc[m]);
                acc[m] = __fmaf_rn((float) (sB + tB), __fmul_rn(dB, dx.y), acc[m]);
            }
        }
    }
}

// Sum over the GS lanes of a group (every lane of the group gets the sum).
template <int M_T>
__device__ __forceinline__ void group_reduce(float (&acc)[M_T], int GS) {
#pragma unroll
    for (int m = 0; m < M_T; ++m) {
        for (int off = GS >> 1; off > 0; off >>= 1) {
            acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], off);
        }
    }
}

// ---------------------------------------------------------------- superblocks
//
// A superblock is 8 consecutive Q8_0 blocks of a row: 272 bytes, 16-byte
// aligned whenever the row is (K % 256 == 0).  A lane reads one with 17
// 128-bit shared loads.  Activation layout for this path ("chunk-major"):
// token m's codes occupy K bytes at m*K; 16-byte chunk c (0..15) of
// superblock j sits at m*K + ((c*NSB + j)*16 XOR 64*(c >= 8)), so the lanes
// of a row group, which read the same chunk of consecutive superblocks, touch
// consecutive 16-byte words.  The XOR moves the second half-superblock's
// chunks by 16 banks: the lanes on the first and on the second half of the
// same superblocks would otherwise read the same banks (a two-way conflict on
// every activation load at K = 1024).  Bit 6 flips inside a 128-byte segment
// of the second half's region, so the layout stays a permutation.  Scales:
// fp32 at [m*NB + b] as before.

// Byte offset of code `pos` (0..255) of superblock j of token m.
__device__ __forceinline__ int sb_code_offset(int m, int K, int NSB, int j, int pos) {
    return m * K + (((((pos >> 4) * NSB + j) << 4) ^ ((pos >> 7) << 6)) | (pos & 15));
}

// Half-superblock units: a lane takes 4 blocks (136 bytes, 8-byte aligned:
// 17 64-bit shared loads) -- twice the lanes of a whole-superblock split on
// the same row, half the work per lane.  Unit u of a row is half (u & 1) of superblock
// (u >> 1).
template <int M_T>
__device__ __forceinline__ void dot_row_half(uint32_t row, int NSB, int NB, int K, int gl, int GS, uint32_t xc_s,
                                             uint32_t xd_s, int M, float (&acc)[M_T]) {
    for (int u = gl; u < 2 * NSB; u += GS) {
        const int j = u >> 1;
        const int h = u & 1;
        uint32_t  w[34];
#pragma unroll
        for (int k = 0; k < 17; ++k) {
            uint32_t lo, hi;
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                         : "=r"(lo), "=r"(hi)
                         : "r"(row + (uint32_t) (272 * j + 136 * h + 8 * k)));
            w[2 * k]     = lo;
            w[2 * k + 1] = hi;
        }
#pragma unroll
        for (int m = 0; m < M_T; ++m) {
            if (m < M) {
                const uint4 dq    = lds_v4(xd_s + (uint32_t) ((m * NB + 8 * j + 4 * h) * 4));
                const float dx[4] = { __uint_as_float(dq.x), __uint_as_float(dq.y), __uint_as_float(dq.z),
                                      __uint_as_float(dq.w) };
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int      wb = 17 * (b >> 1);
                    const float    dw = __half2float(__ushort_as_half(
                        (unsigned short) ((b & 1) ? (w[wb + 8] >> 16) : (w[wb] & 0xffffu))));
                    const int      bs = 4 * h + b;  // block within the superblock
                    // chunks 2bs and 2bs+1 of superblock j (sb_code_offset's layout)
                    const uint32_t xm = xc_s + (uint32_t) (m * K);
                    const uint4    xa = lds_v4(xm + (uint32_t) (((((2 * bs) * NSB + j) << 4)) ^ (h << 6)));
                    const uint4    xb = lds_v4(xm + (uint32_t) (((((2 * bs + 1) * NSB + j) << 4)) ^ (h << 6)));
                    int            s0 = 0, s1 = 0;
                    if (b & 1) {
                        s0 = __dp4a((int) w[wb + 9], (int) xa.x, s0);
                        s1 = __dp4a((int) w[wb + 10], (int) xa.y, s1);
                        s0 = __dp4a((int) w[wb + 11], (int) xa.z, s0);
                        s1 = __dp4a((int) w[wb + 12], (int) xa.w, s1);
                        s0 = __dp4a((int) w[wb + 13], (int) xb.x, s0);
                        s1 = __dp4a((int) w[wb + 14], (int) xb.y, s1);
                        s0 = __dp4a((int) w[wb + 15], (int) xb.z, s0);
                        s1 = __dp4a((int) w[wb + 16], (int) xb.w, s1);
                    } else {
                        s0 = __dp4a((int) __byte_perm(w[wb + 0], w[wb + 1], 0x5432), (int) xa.x, s0);
                        s1 = __dp4a((int) __byte_perm(w[wb + 1], w[wb + 2], 0x5432), (int) xa.y, s1);
                        s0 = __dp4a((int) __byte_perm(w[wb + 2], w[wb + 3], 0x5432), (int) xa.z, s0);
                        s1 = __dp4a((int) __byte_perm(w[wb + 3], w[wb + 4], 0x5432), (int) xa.w, s1);
                        s0 = __dp4a((int) __byte_perm(w[wb + 4], w[wb + 5], 0x5432), (int) xb.x, s0);
                        s1 = __dp4a((int) __byte_perm(w[wb + 5], w[wb + 6], 0x5432), (int) xb.y, s1);
                        s0 = __dp4a((int) __byte_perm(w[wb + 6], w[wb + 7], 0x5432), (int) xb.z, s0);
                        s1 = __dp4a((int) __byte_perm(w[wb + 7], w[wb + 8], 0x5432), (int) xb.w, s1);
                    }
                    acc[m] = __fmaf_rn((float) (s0 + s1), __fmul_rn(dw, dx[b]), acc[m]);
                }
            }
        }
    }
}

}  // namespace b200q8
