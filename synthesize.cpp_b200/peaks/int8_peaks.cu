// int8_peaks.cu -- measured int8 ceilings of a B200 for the Q8_0 GEMM
// (libb200q8_peaks.so; measurement only, not on the product path).
//
// Three kernels, each timed by the caller with CUDA events over a grid of one
// CTA per SM:
//  * tcgen05_i8_kernel: one elected thread per CTA issues
//    tcgen05.mma.cta_group::1.kind::i8 (M = 128, N = 256, K = 32, s8 x s8 ->
//    s32, operands in shared memory, accumulator in TMEM) back to back into two
//    alternating accumulators -- the 5th-generation tensor pipe's int8 rate;
//  * mma_sync_i8_kernel: eight warps issue independent mma.sync.m16n8k32 s8
//    chains from registers -- the legacy tensor path the GEMM uses today;
//  * rescale_kernel: the per-block fp32 rescale a Q8_0 GEMM needs after every
//    K = 32 block (bias-subtract, dw*dx, fma into the accumulator: one packed
//    f32x2 instruction each per pair of outputs) -- the CUDA-core bound every
//    tensor path shares, since Q8_0 scales change every 32 values of K.
//  * tcgen05_latency_kernel (one CTA): the round trips the tcgen05 Q8_0 GEMM's
//    pipeline is built from -- a 16-column tcgen05.ld plus its wait, a
//    32-column tcgen05.st plus its wait, one M = 128, N = 128, K = 32 MMA from
//    issue to its commit arriving on an mbarrier, and 32 such MMAs back to
//    back -- in SM clock cycles.
// tcgen05_i8_kernel also has a check mode: one MMA on known operands, the
// accumulator read back with tcgen05.ld and compared by the caller with the
// exact int32 products, so a timed rate is only reported for an MMA whose
// descriptors were shown to compute the right thing.
//
// Shared-memory operands use the K-major no-swizzle canonical layout: 8-row x
// 16-byte core matrices (128 contiguous bytes), the two 16-byte K halves of a
// 32-byte row 128 bytes apart (leading byte offset), 8-row groups 256 bytes
// apart (stride byte offset).  Every address either offset can reach lies in
// the tiles allocated here.  Every wait is bounded; a timeout sets the error
// word, waits (bounded) once more, frees the TMEM and returns.
#include "../csrc/common.cuh"

namespace {

constexpr int kM      = 128;
constexpr int kN      = 256;
constexpr int kK      = 32;             // bytes of K per MMA (one Q8_0 block)
constexpr int kABytes = kM * kK;        // 4 KiB
constexpr int kBBytes = kN * kK;        // 8 KiB
constexpr int kTmemCols = 2 * kN;       // two accumulators of N columns

// Byte offset of element (row, k) of an operand tile in the canonical layout.
__host__ __device__ __forceinline__ int tile_offset(int row, int k) {
    return (row >> 3) * 256 + (k >> 4) * 128 + (row & 7) * 16 + (k & 15);
}

// Shared-memory matrix descriptor (sm100 "version 1"): start address, leading
// byte offset 128, stride byte offset 256 (all >> 4), no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t) ((saddr >> 4) & 0x3fffu);
    d |= (uint64_t) ((128u >> 4) & 0x3fffu) << 16;
    d |= (uint64_t) ((256u >> 4) & 0x3fffu) << 32;
    d |= (uint64_t) 1u << 46;  // version 1
    return d;                  // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::i8: s32 accumulator, s8 A and B, both
// K-major, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t idesc_i8() {
    return (2u << 4)                      // c_format: S32
           | (1u << 7)                    // a_format: signed 8-bit
           | (1u << 10)                   // b_format: signed 8-bit
           | ((uint32_t) (kN >> 3) << 17) // n_dim
           | ((uint32_t) (kM >> 4) << 24);// m_dim
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate,
                                       uint32_t idesc = idesc_i8()) {
    const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2),
        "r"(mask3)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     b200q8::smem_addr(bar))
                 : "memory");
}

}  // namespace

namespace {

// check != 0: one CTA, one MMA on operands A[r][k] = (r % 7) - 3,
// B[n][k] = ((n + 2k) % 5) - 2, accumulator rows 0..127 x columns 0..N-1
// written to out (int32 [128][N]).  check == 0: each CTA issues `iters` MMAs
// (all of one CTA's operands are zero; the rate does not depend on values).
// err receives a nonzero word when a wait timed out.
__global__ void __launch_bounds__(128, 1) tcgen05_i8_kernel(int iters, int check, int * out, unsigned * err) {
    __shared__ __align__(1024) uint8_t tiles[kABytes + kBBytes];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kABytes + kBBytes; i += blockDim.x) {
        tiles[i] = 0;
    }
    __syncthreads();
    if (check) {
        for (int i = threadIdx.x; i < kM * kK; i += blockDim.x) {
            const int r = i / kK, k = i % kK;
            tiles[tile_offset(r, k)] = (uint8_t) (int8_t) ((r % 7) - 3);
        }
        for (int i = threadIdx.x; i < kN * kK; i += blockDim.x) {
            const int n = i / kK, k = i % kK;
            tiles[kABytes + tile_offset(n, k)] = (uint8_t) (int8_t) (((n + 2 * k) % 5) - 2);
        }
    }
    if (threadIdx.x == 0) {
        b200q8::mbar_init(&bar, 1);
        b200q8::fence_mbar_init();
    }
    // the operands, written by ordinary stores, are read by the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         b200q8::smem_addr(&tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tbase = tmem_base;
    bool           ok    = true;
    if (threadIdx.x == 0) {
        const uint64_t a = smem_desc(b200q8::smem_addr(tiles));
        const uint64_t b = smem_desc(b200q8::smem_addr(tiles + kABytes));
        const int      n = check ? 1 : iters;
        for (int i = 0; i < n; ++i) {
            // two accumulators (columns 0 and N) taken in turn; each starts fresh on its first MMA
            mma_i8(tbase + (uint32_t) ((i & 1) * kN), a, b, i >= 2 ? 1u : 0u);
        }
        mma_commit(&bar);
        if (!b200q8::mbar_wait_bounded(&bar, 0)) {
            atomicExch(err, 1u);
            ok = b200q8::mbar_wait_bounded(&bar, 0);  // once more before the TMEM is freed
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (check && ok) {
        // warp w reads TMEM lanes 32w..32w+31 (accumulator rows), 8 columns per load
        for (int c = 0; c < kN; c += 8) {
            uint32_t v[8];
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                         : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                           "=r"(v[7])
                         : "r"(tbase + ((uint32_t) (32 * warp) << 16) + (uint32_t) c));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            for (int j = 0; j < 8; ++j) {
                out[(32 * warp + lane) * kN + c + j] = (int) v[j];
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols));
    }
}

}  // namespace

namespace {

// Eight warps per CTA, each `iters` rounds of 8 independent
// mma.sync.m16n8k32 s8 chains on register operands (16 x 8 x 32 MACs each).
__global__ void __launch_bounds__(256, 1) mma_sync_i8_kernel(int iters, int seed, int * sink) {
    const uint32_t a[4] = { 0x01020304u ^ (uint32_t) seed, 0x05060708u, 0x090a0b0cu, 0x0d0e0f10u };
    const uint2    b    = make_uint2(0x11121314u ^ (uint32_t) threadIdx.x, 0x15161718u);
    int            d[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        d[c][0] = d[c][1] = d[c][2] = d[c][3] = c;
    }
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                         "{%0,%1,%2,%3};"
                         : "+r"(d[c][0]), "+r"(d[c][1]), "+r"(d[c][2]), "+r"(d[c][3])
                         : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
        }
    }
    int s = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        s += d[c][0] + d[c][1] + d[c][2] + d[c][3];
    }
    if (s == 0x7fffffff) {
        sink[0] = s;  // keeps the chains live
    }
}

// The Q8_0 per-block rescale as the GEMM's epilogue of every block does it:
// for each pair of outputs, subtract the MMA bias (the block sum reads as the
// float 1.5 * 2^23 + S), form dw * dx and fma into the accumulator -- three
// packed f32x2 instructions per two block-outputs.  Eight independent
// accumulator pairs per thread, eight warps per CTA.
__global__ void __launch_bounds__(256, 1) rescale_kernel(int iters, float seed, float * sink) {
    float2       acc[8];
    float2       s[8];
    const float2 nbias = make_float2(-12582912.0f, -12582912.0f);
    float2       dw[8];  // one weight-row scale pair per chain, as each output pair has its own
    float2       dx = make_float2(0.25f, 0.125f + threadIdx.x * 1e-6f);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        acc[c] = make_float2(0.0f, 0.0f);
        s[c]   = make_float2(12582912.0f + c, 12582912.0f - c);
        dw[c]  = make_float2(seed + c, seed * 0.5f - c);
    }
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float2 v = __fadd2_rn(s[c], nbias);
            acc[c]         = __ffma2_rn(v, __fmul2_rn(dw[c], dx), acc[c]);
        }
        dx.x += 1e-7f;  // a new scale product each block, as in the GEMM
    }
    float t = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        t += acc[c].x + acc[c].y;
    }
    if (t == 1234.5f) {
        sink[0] = t;
    }
}

// One CTA of 128 threads: out[0..1] = best / mean cycles of a 16-column
// tcgen05.ld + wait (16 tries), out[2..3] the same for a 32-column
// tcgen05.st + wait, out[4] one 128 x 128 x 32 MMA from issue to its commit
// arriving, out[5] 32 such MMAs back to back (issue to the last commit).
// Operands are the zeroed tiles of tcgen05_i8_kernel's layout; every TMEM
// address stays inside the 512 columns allocated.
__global__ void __launch_bounds__(128, 1) tcgen05_latency_kernel(long long * out, unsigned * err) {
    __shared__ __align__(1024) uint8_t tiles[kABytes + kBBytes];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kABytes + kBBytes; i += blockDim.x) {
        tiles[i] = 0;
    }
    if (threadIdx.x == 0) {
        b200q8::mbar_init(&bar, 1);
        b200q8::fence_mbar_init();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         b200q8::smem_addr(&tmem_base)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tb = tmem_base;
    const uint32_t tl = tb + ((uint32_t) (32 * warp) << 16);
    long long      best = 1LL << 60, sum = 0;
    for (int r = 0; r < 16; ++r) {
        uint32_t        v[16];
        const long long t0 = clock64();
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(tl + 16u * (uint32_t) (r & 7)));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        uint32_t x = 0;
        for (int i = 0; i < 16; ++i) {
            x ^= v[i];
        }
        const long long t1 = clock64();
        if (x == 0xdeadbeefu) {
            out[7] = x;  // keeps the loads live
        }
        best = min(best, t1 - t0);
        sum += t1 - t0;
    }
    if (threadIdx.x == 0) {
        out[0] = best;
        out[1] = sum / 16;
    }
    best = 1LL << 60;
    sum  = 0;
    for (int r = 0; r < 16; ++r) {
        const uint32_t  b  = 0u;
        const long long t0 = clock64();
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
            "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(tl + 32u * (uint32_t) (r & 7)),
            "r"(b)
            : "memory");
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        const long long t1 = clock64();
        best               = min(best, t1 - t0);
        sum += t1 - t0;
    }
    if (threadIdx.x == 0) {
        out[2] = best;
        out[3] = sum / 16;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x == 0) {
        constexpr uint32_t idesc128 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (128 >> 3) << 17) |
                                      ((uint32_t) (kM >> 4) << 24);
        const uint64_t a  = smem_desc(b200q8::smem_addr(tiles));
        const uint64_t bd = smem_desc(b200q8::smem_addr(tiles + kABytes));
        uint32_t       ph = 0;
        const int      ns[2] = { 1, 32 };
        for (int q = 0; q < 2; ++q) {
            const long long t0 = clock64();
            for (int i = 0; i < ns[q]; ++i) {
                mma_i8(tb + 128u * (uint32_t) (i & 3), a, bd, 0u, idesc128);
            }
            mma_commit(&bar);
            bool ok = b200q8::mbar_wait_bounded(&bar, ph);
            if (!ok) {
                atomicExch(err, 1u);
                ok = b200q8::mbar_wait_bounded(&bar, ph);  // once more before the TMEM is freed
            }
            ph ^= 1u;
            out[4 + q] = ok ? clock64() - t0 : -1;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(512));
    }
}

}  // namespace

extern "C" {

// tcgen05_latency_kernel's six figures (cycles) into out_host.  Returns 0, a
// CUDA error code, or -1 when a wait timed out.
int b200q8p_tcgen05_latency(long long * out_host) {
    long long * out = nullptr;
    unsigned *  err = nullptr;
    cudaError_t e   = cudaMalloc(&out, sizeof(long long) * 8);
    if (e == cudaSuccess) e = cudaMalloc(&err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(out, 0, sizeof(long long) * 8);
    for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {  // the second run is reported
        tcgen05_latency_kernel<<<1, 128>>>(out, err);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    unsigned herr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(out_host, out, sizeof(long long) * 6, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&herr, err, sizeof(unsigned), cudaMemcpyDeviceToHost);
    cudaFree(out);
    cudaFree(err);
    return e != cudaSuccess ? (int) e : herr != 0 ? -1 : 0;
}

// One tcgen05 MMA on known operands; out (host, int32 [128][256]) receives
// the accumulator.  Returns 0, or a CUDA error code, or -1 when a wait timed
// out.
int b200q8p_tcgen05_check(int * out_host) {
    int *      out = nullptr;
    unsigned * err = nullptr;
    cudaError_t e  = cudaMalloc(&out, sizeof(int) * kM * kN);
    if (e == cudaSuccess) e = cudaMalloc(&err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(out, 0xff, sizeof(int) * kM * kN);
    if (e == cudaSuccess) {
        tcgen05_i8_kernel<<<1, 128>>>(1, 1, out, err);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    unsigned herr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(out_host, out, sizeof(int) * kM * kN, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&herr, err, sizeof(unsigned), cudaMemcpyDeviceToHost);
    cudaFree(out);
    cudaFree(err);
    return e != cudaSuccess ? (int) e : herr != 0 ? -1 : 0;
}

// kind 0: tcgen05 i8 (iters MMAs of 128 x 256 x 32 per CTA); 1: mma.sync i8
// (iters x 8 MMAs of 16 x 8 x 32 per warp, 8 warps); 2: the rescale (iters x
// 16 block-outputs per thread, 256 threads).  grid CTAs, `reps` launches timed
// together with CUDA events; *ms receives the time per launch.  Returns 0, a
// CUDA error code, or -1 when a wait timed out.
int b200q8p_run(int kind, int grid, int iters, int reps, float * ms) {
    void *     sink = nullptr;
    unsigned * err  = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e  = cudaMalloc(&sink, 64);
    if (e == cudaSuccess) e = cudaMalloc(&err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    // the tcgen05 CTAs ask for shared memory no two of them fit in, so each
    // has an SM (and its TMEM) to itself
    constexpr int kOneCtaSmem = 160 * 1024;
    if (e == cudaSuccess && kind == 0) {
        e = cudaFuncSetAttribute(tcgen05_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kOneCtaSmem);
    }
    auto launch = [&]() {
        if (kind == 0) {
            tcgen05_i8_kernel<<<grid, 128, kOneCtaSmem>>>(iters, 0, nullptr, err);
        } else if (kind == 1) {
            mma_sync_i8_kernel<<<grid, 256>>>(iters, 1, static_cast<int *>(sink));
        } else {
            rescale_kernel<<<grid, 256>>>(iters, 0.75f, static_cast<float *>(sink));
        }
        return cudaGetLastError();
    };
    if (e == cudaSuccess) e = launch();  // warm-up
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaEventRecord(e0);
    for (int r = 0; r < reps && e == cudaSuccess; ++r) {
        e = launch();
    }
    if (e == cudaSuccess) e = cudaEventRecord(e1);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float t = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
    unsigned herr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&herr, err, sizeof(unsigned), cudaMemcpyDeviceToHost);
    *ms = t / (float) (reps > 0 ? reps : 1);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(sink);
    cudaFree(err);
    return e != cudaSuccess ? (int) e : herr != 0 ? -1 : 0;
}

}  // extern "C"
