// mma_tile.cuh -- int8 tensor-core (mma.sync m16n8k32) helpers shared by the
// batched GEMM and the persistent decode step: one MMA is exactly one Q8_0
// block (K = 32) of 16 weight rows x 8 tokens.
#pragma once

#include "common.cuh"

namespace b200q8 {

// The MMA accumulates onto this bias (the float 1.5 * 2^23): a block sum S
// (|S| <= 32 * 128 * 128 < 2^22) then reads as the float 1.5 * 2^23 + S, and
// one exact fp32 subtraction yields S -- no int -> float conversion.
constexpr int   kMmaBias  = 0x4B400000;
constexpr float kMmaBiasF = 12582912.0f;

// D = A x B + C on registers only: not volatile, so the compiler may
// interleave MMAs with loads.  C is a separate, loop-invariant operand.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint2 b, const int (&c)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// The 8 code bytes 8*tq .. 8*tq+7 of block j of a staged weight row (34-byte
// blocks, so only 2-byte aligned; the alignment class depends on j alone and
// folds away once j is a constant).  Lanes load 8 consecutive bytes rather
// than the two 4-byte groups of the standard fragment: A and B use the same
// permutation of k, so every MMA still sums exactly the products of matching
// codes.  Plain loads: the compiler may schedule them, but not across the
// mbarrier operations (which clobber memory).
__device__ __forceinline__ void ld_w8(int j, const uint8_t * row, int tq, uint2 & r) {
    const int       cls = (j * kBlockBytes + 2) & 7;
    const uint8_t * p   = row + j * kBlockBytes + 2 + 8 * tq;
    if (cls == 0) {
        r = *reinterpret_cast<const uint2 *>(p);
    } else if (cls == 4) {
        r.x = *reinterpret_cast<const uint32_t *>(p);
        r.y = *reinterpret_cast<const uint32_t *>(p + 4);
    } else if (cls == 2) {
        const uint2    v  = *reinterpret_cast<const uint2 *>(p - 2);
        const uint32_t w2 = *reinterpret_cast<const uint32_t *>(p + 6);
        r.x               = __byte_perm(v.x, v.y, 0x5432);
        r.y               = __byte_perm(v.y, w2, 0x5432);
    } else {  // cls == 6
        const uint32_t w0 = *reinterpret_cast<const uint32_t *>(p - 2);
        const uint2    v  = *reinterpret_cast<const uint2 *>(p + 2);
        r.x               = __byte_perm(w0, v.x, 0x5432);
        r.y               = __byte_perm(v.x, v.y, 0x5432);
    }
}

// ld_w8 for a block index known only at run time (one warp-uniform branch).
__device__ __forceinline__ void ld_w8_rt(int j, const uint8_t * row, int tq, uint2 & r) {
    switch (j & 3) {
        case 0: ld_w8(0, row + (j - 0) * kBlockBytes, tq, r); break;
        case 1: ld_w8(1, row + (j - 1) * kBlockBytes, tq, r); break;
        case 2: ld_w8(2, row + (j - 2) * kBlockBytes, tq, r); break;
        default: ld_w8(3, row + (j - 3) * kBlockBytes, tq, r); break;
    }
}

}  // namespace b200q8
