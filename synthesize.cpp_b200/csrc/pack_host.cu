// pack_host.cu -- ggml_quantize_chunk(GGML_TYPE_Q8_0, ...) on HOST buffers.
//
// tools/synthesize-quantize/quantize.cpp:297-301 dequantizes each source tensor
// to an F32 host vector and calls ggml_quantize_chunk into the output GGUF's
// host buffer.  This entry point takes exactly those buffers.  Rows move in
// chunks through a two-deep pipeline per device:
//
//   host threads copy chunk k of src into pinned staging k%2
//     -> H2D copy -> quantize_dense_kernel -> D2H copy into pinned staging
//   while the GPU works on chunk k, the host copies chunk k-1's codes out to
//   dst and chunk k+1's floats in.
//
// The pinned and device staging (two input and two output buffers, 32 MiB of
// F32 each by default) is allocated on a device's first call and kept for the
// next ones: a quantize run makes hundreds of calls, and page-locking the
// caller's buffers or allocating per call cost more than the copies.
// b200q8_quantize_chunk_host_release() frees it.  Calls on one device are
// serialised by a mutex.  A tool call, not a hot-path one.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace b200q8 {
b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...);
b200q8_status_t cuda_error(cudaError_t e, const char * what);
int             current_sm_count();
}  // namespace b200q8

using namespace b200q8;

namespace {

constexpr int    kMaxDevices     = 64;
constexpr size_t kChunkInBytes   = (size_t) 32 << 20;  // F32 per staging buffer
constexpr int    kMaxCopyThreads = 16;

struct Staging {
    size_t       cap_in  = 0;  // bytes per input buffer
    size_t       cap_out = 0;  // bytes per output buffer
    float *      pin_in[2]  = { nullptr, nullptr };
    uint8_t *    pin_out[2] = { nullptr, nullptr };
    float *      dev_in[2]  = { nullptr, nullptr };
    uint8_t *    dev_out[2] = { nullptr, nullptr };
    cudaStream_t st[2]      = { nullptr, nullptr };
    cudaEvent_t  done[2]    = { nullptr, nullptr };
};

std::mutex g_mu[kMaxDevices];
Staging    g_staging[kMaxDevices];

void free_staging(Staging & s) {
    for (int i = 0; i < 2; ++i) {
        if (s.st[i]) {
            cudaStreamSynchronize(s.st[i]);
            cudaStreamDestroy(s.st[i]);
        }
        if (s.done[i]) cudaEventDestroy(s.done[i]);
        if (s.pin_in[i]) cudaFreeHost(s.pin_in[i]);
        if (s.pin_out[i]) cudaFreeHost(s.pin_out[i]);
        if (s.dev_in[i]) cudaFree(s.dev_in[i]);
        if (s.dev_out[i]) cudaFree(s.dev_out[i]);
    }
    s = Staging();
}

// Staging that holds at least one row of this width (the current device).
// Q8_0 output is 34/64 of a 16-bit input (34/128 of an F32 one) for every K,
// so one output size serves every shape and source type.
cudaError_t ensure_staging(Staging & s, size_t row_in) {
    if (s.cap_in >= row_in) {
        return cudaSuccess;
    }
    free_staging(s);
    const size_t cap_in  = std::max(kChunkInBytes, row_in);
    const size_t cap_out = (cap_in * kBlockBytes + 2 * kQK - 1) / (2 * kQK);
    cudaError_t  e       = cudaSuccess;
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
        e = cudaHostAlloc(reinterpret_cast<void **>(&s.pin_in[i]), cap_in, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void **>(&s.pin_out[i]), cap_out, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaMalloc(&s.dev_in[i], cap_in);
        if (e == cudaSuccess) e = cudaMalloc(&s.dev_out[i], cap_out);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.st[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.done[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) {
        free_staging(s);
        return e;
    }
    s.cap_in  = cap_in;
    s.cap_out = cap_out;
    return cudaSuccess;
}

// memcpy split over host threads (large copies run at several threads' bandwidth).
void parallel_copy(void * dst, const void * src, size_t bytes) {
    static const int hw = (int) std::max(1u, std::thread::hardware_concurrency());
    const int        t  = (int) std::min<size_t>(std::min(hw, kMaxCopyThreads), std::max<size_t>(1, bytes >> 22));
    if (t <= 1) {
        memcpy(dst, src, bytes);
        return;
    }
    const size_t             part = (bytes / t + 63) & ~(size_t) 63;
    std::vector<std::thread> pool;
    pool.reserve(t - 1);
    for (int i = 1; i < t; ++i) {
        const size_t off = std::min(bytes, (size_t) i * part);
        const size_t n   = std::min(bytes - off, part);
        pool.emplace_back([=] { memcpy(static_cast<uint8_t *>(dst) + off, static_cast<const uint8_t *>(src) + off, n); });
    }
    memcpy(dst, src, std::min(bytes, part));
    for (auto & th : pool) {
        th.join();
    }
}

b200q8_status_t pack_host(const void * src, int src_type, size_t es, void * dst, int64_t start, int64_t nrows,
                          int64_t n_per_row, size_t * written, int32_t device) {
    if (n_per_row <= 0 || n_per_row % kQK != 0 || start < 0 || nrows < 0 || start % n_per_row != 0 ||
        (nrows > 0 && (src == nullptr || dst == nullptr))) {
        return set_error(B200Q8_ERR_INVALID_ARG,
                         "quantize_chunk_host: n_per_row must be a positive multiple of 32 and start a multiple of it");
    }
    if (device < 0 || device >= kMaxDevices) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_chunk_host: device %d out of range", device);
    }
    const size_t  row_in    = (size_t) n_per_row * es;
    const size_t  row_out   = (size_t) (n_per_row / kQK) * kBlockBytes;
    const int64_t start_row = start / n_per_row;
    if (written != nullptr) {
        *written = (size_t) nrows * row_out;
    }
    if (nrows == 0) {
        return B200Q8_OK;
    }
    std::lock_guard<std::mutex> lock(g_mu[device]);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        return cuda_error(e, "quantize_chunk_host: cudaSetDevice");
    }
    Staging & s = g_staging[device];
    e           = ensure_staging(s, row_in);
    if (e != cudaSuccess) {
        cudaSetDevice(prev);
        return cuda_error(e, "quantize_chunk_host: staging allocation");
    }
    const uint8_t * s_rows    = static_cast<const uint8_t *>(src) + (size_t) start * es;
    uint8_t *      d_rows     = static_cast<uint8_t *>(dst) + (size_t) start_row * row_out;
    const int64_t  chunk_rows = (int64_t) (s.cap_in / row_in);
    const int64_t  n_chunks   = (nrows + chunk_rows - 1) / chunk_rows;
    const int      sms        = current_sm_count();
    auto           rows_of    = [&](int64_t k) { return std::min(chunk_rows, nrows - k * chunk_rows); };
    // copy chunk k's codes from pinned staging to dst once its D2H finished
    auto drain = [&](int64_t k) -> cudaError_t {
        const int         i  = (int) (k & 1);
        const cudaError_t e2 = cudaEventSynchronize(s.done[i]);
        if (e2 == cudaSuccess) {
            parallel_copy(d_rows + (size_t) (k * chunk_rows) * row_out, s.pin_out[i], (size_t) rows_of(k) * row_out);
        }
        return e2;
    };
    for (int64_t k = 0; k < n_chunks && e == cudaSuccess; ++k) {
        const int     i    = (int) (k & 1);
        const int64_t rows = rows_of(k);
        if (k >= 2) {
            e = drain(k - 2);  // frees staging i
            if (e != cudaSuccess) {
                break;
            }
        }
        parallel_copy(s.pin_in[i], s_rows + (size_t) (k * chunk_rows) * row_in, (size_t) rows * row_in);
        e = cudaMemcpyAsync(s.dev_in[i], s.pin_in[i], (size_t) rows * row_in, cudaMemcpyHostToDevice, s.st[i]);
        if (e == cudaSuccess) {
            e = launch_quantize_typed(s.dev_in[i], src_type, rows, n_per_row, row_in, s.dev_out[i], row_out,
                                      B200Q8_QUANT_REF, s.st[i], sms);
        }
        if (e == cudaSuccess) {
            e = cudaMemcpyAsync(s.pin_out[i], s.dev_out[i], (size_t) rows * row_out, cudaMemcpyDeviceToHost, s.st[i]);
        }
        if (e == cudaSuccess) {
            e = cudaEventRecord(s.done[i], s.st[i]);
        }
    }
    for (int64_t k = std::max<int64_t>(0, n_chunks - 2); k < n_chunks && e == cudaSuccess; ++k) {
        e = drain(k);
    }
    if (e != cudaSuccess) {
        // leave nothing in flight on the staging before reporting
        cudaStreamSynchronize(s.st[0]);
        cudaStreamSynchronize(s.st[1]);
    }
    cudaSetDevice(prev);
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "quantize_chunk_host");
}

}  // namespace

extern "C" b200q8_status_t b200q8_quantize_chunk_host(const float * src, void * dst, int64_t start, int64_t nrows,
                                                      int64_t n_per_row, size_t * written, int32_t device) {
    return pack_host(src, kSrcF32, 4, dst, start, nrows, n_per_row, written, device);
}

extern "C" b200q8_status_t b200q8_quantize_chunk_host_typed(const void * src, int32_t src_type, void * dst,
                                                            int64_t start, int64_t nrows, int64_t n_per_row,
                                                            size_t * written, int32_t device) {
    const size_t es = src_type == B200Q8_SRC_F32 ? 4 : (src_type == B200Q8_SRC_F16 || src_type == B200Q8_SRC_BF16) ? 2 : 0;
    if (es == 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_chunk_host_typed: unknown source type %d", src_type);
    }
    return pack_host(src, src_type, es, dst, start, nrows, n_per_row, written, device);
}

extern "C" void b200q8_quantize_chunk_host_release(void) {
    int prev = 0;
    cudaGetDevice(&prev);
    for (int d = 0; d < kMaxDevices; ++d) {
        std::lock_guard<std::mutex> lock(g_mu[d]);
        if (g_staging[d].cap_in != 0 && cudaSetDevice(d) == cudaSuccess) {
            free_staging(g_staging[d]);
        }
    }
    cudaSetDevice(prev);
}
