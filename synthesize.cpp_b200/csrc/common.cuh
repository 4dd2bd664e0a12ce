// common.cuh -- shared device helpers for the B200 Q8_0 kernels (sm_100a).
//
// Q8_0 block (ggml block_q8_0): fp16 scale d, then 32 int8 codes; 34 bytes.
// Rows of K/32 blocks.  Eight blocks (256 weights) make 272 bytes, the
// smallest run of blocks that starts and ends on a 16-byte boundary; the
// streaming kernels work in those units or in block pairs (68 bytes, 4-byte
// aligned).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200q8.h"

namespace b200q8 {

constexpr int kQK          = 32;
constexpr int kBlockBytes  = 34;
constexpr int kPairBytes   = 68;
constexpr int kSuperBlocks = 8;    // blocks per 272-byte, 16-byte-aligned run
constexpr int kSuperBytes  = 272;

// Per-device status word written by kernels (first error wins).  The
// library is one translation unit (libb200q8.cu), so this is its only
// definition.
__device__ unsigned int g_device_status = 0u;

__device__ __forceinline__ void record_device_error(unsigned int code) {
    atomicCAS(&g_device_status, 0u, code);
}

// ------------------------------------------------------------------ quantize
//
// Restates quantize_row_q8_0_ref (ggml-quants.c; gguf-py quants.py:378-394)
// and ggml-cpu's two SIMD from_float forms, for one 32-value block held by a
// group of G consecutive lanes, E = 32/G consecutive values per lane.
//
// amax follows the reference's sequential fold amax = MAX(amax, |x_j|) with
// MAX(a,b) = a > b ? a : b, including its NaN behaviour: a NaN at position p
// is replaced by the first later value, so the result is the max over the
// values after the last NaN, or NaN when the last value is NaN.

template <int G>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    }
    return v;
}

template <int G>
__device__ __forceinline__ int group_max_int(int v) {
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) {
        v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
    }
    return v;
}

// All 32 lanes of the warp must call this (shuffles use the full mask).
// lane_in_group = lane % G; v[e] is element lane_in_group*E + e of the block,
// or with STRIDED element lane_in_group + G*e.
template <int G, int E, bool STRIDED = false>
__device__ __forceinline__ float block_amax(const float (&v)[E], int lane_in_group) {
    auto pos = [&](int e) { return STRIDED ? lane_in_group + G * e : lane_in_group * E + e; };
    bool has_nan = false;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        has_nan |= isnan(v[e]);
    }
    if (!__any_sync(0xffffffffu, has_nan)) {
        float m = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            m = fmaxf(m, fabsf(v[e]));
        }
        return group_max<G>(m);
    }
    int last_nan = -1;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        if (isnan(v[e])) {
            last_nan = max(last_nan, pos(e));
        }
    }
    last_nan = group_max_int<G>(last_nan);
    float m  = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        if (pos(e) > last_nan) {
            m = fmaxf(m, fabsf(v[e]));
        }
    }
    m = group_max<G>(m);
    return last_nan == kQK - 1 ? __int_as_float(0x7fc00000) : m;
}

struct QuantParams {
    float          id;     // multiplier applied to each value
    float          d;      // fp32(fp16(d)): the scale the dot product uses
    unsigned short dbits;  // stored fp16 bits of d
};

// amax / 127 rounded to nearest (IEEE single division), for amax >= 0.
// For finite amax: q = RN(amax * r) with r = RN(1/127), then one FMA
// correction with the exact residual amax - 127*q (the division-by-a-constant
// scheme of P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", 1990).  It was checked against IEEE division
// for all 2^31 non-negative finite floats; it uses only correctly rounded
// multiply and FMA, so it gives the same bits on any IEEE machine.
// Infinity and NaN take the plain division.
__device__ __forceinline__ float div127_rn(float amax) {
    if (!(amax <= 3.40282347e38f)) {
        return __fdiv_rn(amax, 127.0f);
    }
    const float r = 0.00787401574803149606f;  // RN(1/127)
    const float q = __fmul_rn(amax, r);
    const float e = __fmaf_rn(-q, 127.0f, amax);
    return __fmaf_rn(e, r, q);
}

template <int MODE>
__device__ __forceinline__ QuantParams quant_params(float amax) {
    QuantParams p;
    const float d = div127_rn(amax);
    if (MODE == B200Q8_QUANT_CPU_X86) {
        p.id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    } else {
        p.id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;  // IEEE reciprocal == 1.0f/d
    }
    if (isnan(d)) {
        p.dbits = 0x7e00u;
    } else {
        p.dbits = __half_as_ushort(__float2half_rn(d));
    }
    p.d = __half2float(__ushort_as_half(p.dbits));
    return p;
}

// One code: x*id rounded (half away from zero for REF, half to even for the
// SIMD forms), stored as the low byte of its int32 conversion.  ggml's amax
// fold skips every value before a block's last NaN, so x*id can be any float:
// NaN, infinities and values outside [-2^31, 2^31) store 0, which is what the
// reference's float -> int8_t store gives on x86 (cvttss2si's 0x80000000).
template <int MODE>
__device__ __forceinline__ int quant_code(float x, float id) {
    const float x0 = __fmul_rn(x, id);
    const float r  = (MODE == B200Q8_QUANT_REF) ? roundf(x0) : rintf(x0);
    return (r >= -2147483648.0f && r < 2147483648.0f) ? static_cast<int>(r) : 0;
}

// silu as ggml's scalar form writes it: x / (1 + expf(-x)).  expf is CUDA's
// (within 2 ulp of the exact value); libm's may differ by an ulp.
__device__ __forceinline__ float silu_f32(float v) {
    return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
}

// ------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}

// `count` arrivals in one operation (one thread standing in for `count`
// warps that are known, through a barrier, to have arrived).
__device__ __forceinline__ void mbar_arrive_count(uint64_t * bar, uint32_t count) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait: about one second of SM clock at most.  Returns false when
// the limit ran out; the caller records B200Q8_ERR_DEVICE_TIMEOUT.
constexpr long long kWaitLimitCycles = 2000000000LL;

// try_wait with a suspend-time hint (ns): for waiters off the critical path,
// so they do not compete for issue slots while they wait.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded_sleep(uint64_t * bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (clock64() - start > kWaitLimitCycles) {
            return false;
        }
    }
    return true;
}

// Bounded wait that also gives up when *flag becomes non-zero (a stop
// request from the CTA's other threads).  Returns true only if the phase
// completed.
__device__ __forceinline__ bool mbar_wait_bounded_or_flag(uint64_t * bar, uint32_t parity, const int * flag) {
    const long long start = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (*(volatile const int *) flag != 0 || clock64() - start > kWaitLimitCycles) {
            return false;
        }
    }
    return true;
}

// Shared-memory loads by shared-window address (explicit .shared space).
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}

// Non-blocking probe of a phase (no suspension, unlike try_wait).
__device__ __forceinline__ bool mbar_test_wait(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t * bar, uint32_t parity) {
    if (mbar_test_wait(bar, parity)) {
        return true;
    }
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > kWaitLimitCycles) {
            return false;
        }
    }
    return true;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.  Never multicast.
__device__ __forceinline__ void bulk_copy_g2s(void * dst_smem, const void * src_gmem, uint32_t bytes, uint64_t * bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// L2 policy for data read exactly once (streamed weights).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// L2 policy for data that other CTAs read again soon (shared activations).
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ uint64_t lds_u64(uint32_t addr) {
    uint64_t v;
    asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// Programmatic dependent launch: no-ops unless the launch enabled it.
__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace b200q8
