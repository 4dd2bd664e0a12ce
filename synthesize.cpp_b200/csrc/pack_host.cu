// pack_host.cu -- ggml_quantize_chunk(GGML_TYPE_Q8_0, ...) on HOST buffers.
//
// tools/synthesize-quantize/quantize.cpp:297-301 dequantizes each source tensor
// to an F32 host vector and calls ggml_quantize_chunk into the output GGUF's
// host buffer.  This entry point takes exactly those buffers: rows stream
// host -> device -> host in chunks through two CUDA streams (copy in, pack,
// copy out overlap across chunks), packed by the same bit-exact kernel as
// b200q8_quantize_rows.  The user buffers are page-locked for the duration
// of the call when the driver allows it, so the copies run as DMA.  It is a
// tool call, not a hot-path one: it allocates its device staging buffers and
// frees them before returning.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace b200q8 {
b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...);
b200q8_status_t cuda_error(cudaError_t e, const char * what);
int             current_sm_count();
}  // namespace b200q8

using namespace b200q8;

extern "C" b200q8_status_t b200q8_quantize_chunk_host(const float * src, void * dst, int64_t start, int64_t nrows,
                                                      int64_t n_per_row, size_t * written, int32_t device) {
    if (n_per_row <= 0 || n_per_row % kQK != 0 || start < 0 || nrows < 0 || start % n_per_row != 0 ||
        (nrows > 0 && (src == nullptr || dst == nullptr))) {
        return set_error(B200Q8_ERR_INVALID_ARG,
                         "quantize_chunk_host: n_per_row must be a positive multiple of 32 and start a multiple of it");
    }
    const size_t  row_in    = (size_t) n_per_row * sizeof(float);
    const size_t  row_out   = (size_t) (n_per_row / kQK) * kBlockBytes;
    const int64_t start_row = start / n_per_row;
    if (written != nullptr) {
        *written = (size_t) nrows * row_out;
    }
    if (nrows == 0) {
        return B200Q8_OK;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        return cuda_error(e, "quantize_chunk_host: cudaSetDevice");
    }
    const float * s_rows = src + start;
    uint8_t *     d_rows = static_cast<uint8_t *>(dst) + (size_t) start_row * row_out;
    // page-lock the caller's buffers when possible (plain copies otherwise)
    const bool pin_src = cudaHostRegister(const_cast<float *>(s_rows), (size_t) nrows * row_in,
                                          cudaHostRegisterReadOnly) == cudaSuccess;
    if (!pin_src) {
        cudaGetLastError();
    }
    const bool pin_dst = cudaHostRegister(d_rows, (size_t) nrows * row_out, cudaHostRegisterDefault) == cudaSuccess;
    if (!pin_dst) {
        cudaGetLastError();
    }
    const int64_t chunk_rows = std::max<int64_t>(1, (int64_t) ((size_t) 128 << 20) / (int64_t) row_in);
    float *       dsrc[2]    = { nullptr, nullptr };
    uint8_t *     ddst[2]    = { nullptr, nullptr };
    cudaStream_t  st[2]      = { nullptr, nullptr };
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
        e = cudaMalloc(&dsrc[i], (size_t) chunk_rows * row_in);
        if (e == cudaSuccess) e = cudaMalloc(&ddst[i], (size_t) chunk_rows * row_out);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking);
    }
    const int sms = current_sm_count();
    for (int64_t r0 = 0, k = 0; r0 < nrows && e == cudaSuccess; r0 += chunk_rows, ++k) {
        const int     i    = (int) (k & 1);
        const int64_t rows = std::min(chunk_rows, nrows - r0);
        e = cudaMemcpyAsync(dsrc[i], s_rows + r0 * n_per_row, (size_t) rows * row_in, cudaMemcpyHostToDevice, st[i]);
        if (e == cudaSuccess) {
            e = launch_quantize(dsrc[i], rows, n_per_row, row_in, ddst[i], row_out, B200Q8_QUANT_REF, st[i], sms);
        }
        if (e == cudaSuccess) {
            e = cudaMemcpyAsync(d_rows + (size_t) r0 * row_out, ddst[i], (size_t) rows * row_out,
                                cudaMemcpyDeviceToHost, st[i]);
        }
    }
    for (int i = 0; i < 2; ++i) {
        if (st[i]) {
            const cudaError_t e2 = cudaStreamSynchronize(st[i]);
            if (e == cudaSuccess) e = e2;
            cudaStreamDestroy(st[i]);
        }
        cudaFree(dsrc[i]);
        cudaFree(ddst[i]);
    }
    if (pin_src) cudaHostUnregister(const_cast<float *>(s_rows));
    if (pin_dst) cudaHostUnregister(d_rows);
    cudaSetDevice(prev);
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "quantize_chunk_host");
}
