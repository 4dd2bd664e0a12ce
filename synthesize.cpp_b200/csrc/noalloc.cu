// noalloc.cu -- b200q8_mul_mat_noalloc: the Q8_0 MUL_MAT for callers that
// cannot allocate device memory.
//
// b200q8_mul_mat needs caller scratch (the quantized activations) for shapes
// outside its streaming fast path, and the caller gets it from
// b200q8_mul_mat_workspace_size + its own allocator.  Some callers have no
// allocator to turn to at the point of the call: a ggml backend computes a
// graph whose buffers were all placed by ggml-alloc beforehand and cannot
// grow them mid-graph; a real-time audio/streaming callback must not block on
// cudaMalloc's device-wide synchronisation.  This entry point takes the
// scratch from a fixed array in the library's own device memory instead.
//
// The array, its limits and its sharing rules:
//  * kNoAllocScratchBytes (1 MiB) per device, a file-scope __device__ array
//    that every GPU which loads this library holds until the process exits;
//  * a call is accepted when M * (K/32) * 34 bytes (its activations in Q8_0)
//    fit in the array, and rejected with B200Q8_ERR_INVALID_ARG otherwise;
//  * it runs the path b200q8_mul_mat would run with a workspace of the
//    array's size: the tensor-core GEMM when the shape suits it and its
//    staged activation records fit in the array; else the streaming GEMV,
//    which needs no scratch at all; else the general kernel on activations
//    quantized into the array;
//  * all calls on a device share the one array and it keeps whatever the last
//    call left in it.  Nothing in it has to start at zero: every byte a
//    kernel reads from it is written first by the same call.  Two calls whose
//    kernels overlap on the GPU (different streams, no ordering between them)
//    race on the array and may corrupt each other's results; order them on
//    one stream or with events;
//  * the array's name is only a host-side stand-in in host code, so its
//    device address is looked up with cudaGetSymbolAddress, with the device
//    current.  The first call made on a device does that lookup; make it
//    before any stream capture begins.  Later calls on a stream that is not
//    capturing look the address up again, so a device reset (which reloads
//    the module and may move the array) is picked up by the next such call;
//    calls during a capture use the address found last.
#include "common.cuh"
#include "kernels.h"

#include <mutex>

namespace b200q8 {
b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...);
b200q8_status_t cuda_error(cudaError_t e, const char * what);
int             current_sm_count();

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
constexpr int    kNoAllocMaxDevices   = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

void *     g_noalloc_ptr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on the current device.  refresh: look
// it up again even when one is cached (the stream is not capturing).
b200q8_status_t noalloc_scratch(void ** out, bool refresh) {
    int         dev = -1;
    cudaError_t e   = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        return cuda_error(e, "mul_mat_noalloc: cudaGetDevice");
    }
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        return set_error(B200Q8_ERR_UNSUPPORTED, "mul_mat_noalloc: device %d is beyond the %d supported", dev,
                         kNoAllocMaxDevices);
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr || refresh) {
        void * p = nullptr;
        e        = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                              "mul_mat_noalloc: cudaGetSymbolAddress of the static scratch");
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return B200Q8_OK;
}

// True when `s` is known not to be capturing.  A query that fails (the legacy
// stream while another stream captures in global mode answers with an error)
// counts as capturing, so the cached address is used.
bool stream_not_capturing(cudaStream_t s) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
        (void) cudaGetLastError();
        return false;
    }
    return cs == cudaStreamCaptureStatusNone;
}

}  // namespace
}  // namespace b200q8

using namespace b200q8;

extern "C" b200q8_status_t b200q8_mul_mat_noalloc(const void * w, int64_t K, int64_t N, size_t w_row_bytes,
                                                  const float * x, int64_t M, size_t x_col_stride, float * y,
                                                  size_t y_col_stride, int32_t mode, b200q8_stream_t stream) {
    if (K <= 0 || K % kQK != 0 || N < 0 || M < 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat_noalloc: K (%lld) must be a positive multiple of 32",
                         (long long) K);
    }
    if (mode != B200Q8_QUANT_REF && mode != B200Q8_QUANT_CPU_X86 && mode != B200Q8_QUANT_CPU_ARM) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat_noalloc: unknown mode %d", mode);
    }
    if (N == 0 || M == 0) {
        return B200Q8_OK;
    }
    const size_t row = (size_t) (K / kQK) * kBlockBytes;
    if ((size_t) M > kNoAllocScratchBytes / row) {
        return set_error(B200Q8_ERR_INVALID_ARG,
                         "mul_mat_noalloc: M*(K/32)*34 = %lld bytes of scratch exceeds the static maximum of %zu "
                         "bytes; use b200q8_mul_mat with a workspace",
                         (long long) M * (long long) row, kNoAllocScratchBytes);
    }
    if (w == nullptr || x == nullptr || y == nullptr || w_row_bytes < row ||
        (reinterpret_cast<uintptr_t>(x) % 4) != 0 || (reinterpret_cast<uintptr_t>(y) % 4) != 0 ||
        x_col_stride % 4 != 0 || y_col_stride % 4 != 0 ||
        (M > 1 && (x_col_stride < (size_t) K * 4 || y_col_stride < (size_t) N * 4))) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat_noalloc: bad pointer, alignment, row size or stride");
    }
    cudaStream_t    s       = reinterpret_cast<cudaStream_t>(stream);
    void *          scratch = nullptr;
    b200q8_status_t st      = noalloc_scratch(&scratch, stream_not_capturing(s));
    if (st != B200Q8_OK) {
        return st;
    }
    const int    sms = current_sm_count();
    const size_t xs  = M > 1 ? x_col_stride / 4 : (size_t) K;
    const size_t ys  = M > 1 ? y_col_stride / 4 : (size_t) N;
    const auto * wb  = static_cast<const uint8_t *>(w);
    // 1. the int8 tensor-core GEMM, its staged records in the array
    if (N <= INT32_MAX && K <= INT32_MAX && gemm_supported(wb, w_row_bytes, K, N, M) &&
        gemm_workspace_bytes(K, M) <= kNoAllocScratchBytes) {
        cudaError_t e = launch_gemm(wb, w_row_bytes, K, N, x, xs, M, y, ys, mode, scratch, s, sms);
        return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "mul_mat_noalloc: tensor-core GEMM launch");
    }
    // 2. the streaming GEMV, 8 tokens per launch, no scratch
    GemvParams p = {};
    p.w          = wb;
    p.row_bytes  = w_row_bytes;
    p.K          = (int) K;
    p.N          = (int) N;
    p.M          = (int) std::min<int64_t>(M, 8);
    p.pro        = kProPlain;
    p.x          = x;
    p.x_stride   = xs;
    p.y          = y;
    p.y_stride   = ys;
    p.mode       = mode;
    if (N <= INT32_MAX && K <= INT32_MAX && gemv_supported(p)) {
        for (int64_t m0 = 0; m0 < M; m0 += 8) {
            p.M           = (int) std::min<int64_t>(M - m0, 8);
            p.x           = x + m0 * xs;
            p.y           = y + m0 * ys;
            cudaError_t e = launch_gemv(p, s, sms, false);
            if (e != cudaSuccess) {
                return cuda_error(e, "mul_mat_noalloc: gemv launch");
            }
        }
        return B200Q8_OK;
    }
    // 3. general shapes: activations quantized into the array, then the plain kernel
    cudaError_t e = launch_quantize(x, M, K, xs * 4, scratch, row, mode, s, sms);
    if (e == cudaSuccess) {
        e = launch_gemv_generic(wb, w_row_bytes, K, N, static_cast<const uint8_t *>(scratch), M, y, ys * 4, s);
    }
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "mul_mat_noalloc launch");
}
