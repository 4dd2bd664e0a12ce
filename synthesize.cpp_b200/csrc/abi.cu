// abi.cu -- the extern "C" entry points of libb200q8.so (include/b200q8.h).
//
// Validation, error reporting and kernel dispatch only.  Mirrors the
// reference's ABI discipline (include/synthesize.h:34-55, catch-all at
// src/synthesize.cpp:673-681): every failure is a status code plus a
// per-thread message, nothing throws or aborts across the boundary.
#include "common.cuh"
#include "kernels.h"

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

namespace b200q8 {

namespace {

thread_local std::string     t_err_msg;
thread_local b200q8_status_t t_err_code = B200Q8_OK;

}  // namespace

b200q8_status_t set_error(b200q8_status_t code, const char * fmt, ...) {
    char    buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_err_msg  = buf;
    t_err_code = code;
    return code;
}

b200q8_status_t cuda_error(cudaError_t e, const char * what) {
    return set_error(e == cudaErrorMemoryAllocation ? B200Q8_ERR_OOM : B200Q8_ERR_BACKEND, "%s: %s (%s)", what,
                     cudaGetErrorName(e), cudaGetErrorString(e));
}

int current_sm_count() {
    static int      cached[64] = {};
    int             dev        = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
        return 148;
    }
    if (dev < 64 && cached[dev] > 0) {
        return cached[dev];
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        n = 148;
    }
    if (dev < 64) {
        cached[dev] = n;
    }
    return n;
}

}  // namespace b200q8

using namespace b200q8;

namespace {

bool aligned(const void * p, size_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

size_t align_up(size_t v, size_t a) {
    return (v + a - 1) / a * a;
}

bool valid_mode(int32_t mode) {
    return mode == B200Q8_QUANT_REF || mode == B200Q8_QUANT_CPU_X86 || mode == B200Q8_QUANT_CPU_ARM;
}

}  // namespace

extern "C" {

int32_t b200q8_version(void) {
    return 100;  // 0.1.0
}

b200q8_status_t b200q8_last_error(char * buf, size_t len) {
    if (buf != nullptr && len > 0) {
        const size_t n = std::min(len - 1, t_err_msg.size());
        memcpy(buf, t_err_msg.data(), n);
        buf[n] = '\0';
    }
    return t_err_code;
}

b200q8_status_t b200q8_device_status(int32_t device, int32_t clear) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) {
        return set_error(B200Q8_ERR_BACKEND, "b200q8_device_status: no CUDA device");
    }
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        return cuda_error(e, "b200q8_device_status: cudaSetDevice");
    }
    unsigned int word = 0;
    e                 = cudaDeviceSynchronize();
    if (e == cudaSuccess) {
        e = cudaMemcpyFromSymbol(&word, g_device_status, sizeof(word));
    }
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e                       = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        return cuda_error(e, "b200q8_device_status");
    }
    if (word != 0) {
        return set_error((b200q8_status_t) word, "a kernel on device %d recorded status %u", device, word);
    }
    return B200Q8_OK;
}

b200q8_status_t b200q8_quantize_rows(const float * x, int64_t rows, int64_t K, size_t x_row_stride, void * dst,
                                     size_t dst_row_stride, int32_t mode, b200q8_stream_t stream) {
    if (rows < 0 || K < 0 || K % kQK != 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows: K (%lld) must be a non-negative multiple of 32",
                         (long long) K);
    }
    if (!valid_mode(mode)) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows: unknown mode %d", mode);
    }
    if (rows == 0 || K == 0) {
        return B200Q8_OK;
    }
    const size_t nb = (size_t) K / kQK;
    if (x == nullptr || dst == nullptr || !aligned(x, 4) || x_row_stride % 4 != 0 ||
        (rows > 1 && (x_row_stride < (size_t) K * 4 || dst_row_stride < nb * kBlockBytes))) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows: bad pointer, alignment or stride");
    }
    cudaError_t e = launch_quantize(x, rows, K, rows > 1 ? x_row_stride : (size_t) K * 4, dst,
                                    rows > 1 ? dst_row_stride : nb * kBlockBytes, mode,
                                    reinterpret_cast<cudaStream_t>(stream), current_sm_count());
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "quantize_rows launch");
}

b200q8_status_t b200q8_quantize_rows_typed(const void * x, int32_t src_type, int64_t rows, int64_t K,
                                           size_t x_row_stride, void * dst, size_t dst_row_stride, int32_t mode,
                                           b200q8_stream_t stream) {
    const size_t es = src_type == B200Q8_SRC_F32 ? 4 : (src_type == B200Q8_SRC_F16 || src_type == B200Q8_SRC_BF16) ? 2 : 0;
    if (es == 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows_typed: unknown source type %d", src_type);
    }
    if (rows < 0 || K < 0 || K % kQK != 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows_typed: K (%lld) must be a non-negative multiple of 32",
                         (long long) K);
    }
    if (!valid_mode(mode)) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows_typed: unknown mode %d", mode);
    }
    if (rows == 0 || K == 0) {
        return B200Q8_OK;
    }
    const size_t nb = (size_t) K / kQK;
    if (x == nullptr || dst == nullptr || !aligned(x, es) || x_row_stride % es != 0 ||
        (rows > 1 && (x_row_stride < (size_t) K * es || dst_row_stride < nb * kBlockBytes))) {
        return set_error(B200Q8_ERR_INVALID_ARG, "quantize_rows_typed: bad pointer, alignment or stride");
    }
    cudaError_t e = launch_quantize_typed(x, src_type, rows, K, rows > 1 ? x_row_stride : (size_t) K * es, dst,
                                          rows > 1 ? dst_row_stride : nb * kBlockBytes, mode,
                                          reinterpret_cast<cudaStream_t>(stream), current_sm_count());
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "quantize_rows_typed launch");
}

b200q8_status_t b200q8_quantize_chunk(const float * src, void * dst, int64_t start, int64_t nrows,
                                      int64_t n_per_row, size_t * written, b200q8_stream_t stream) {
    if (n_per_row <= 0 || n_per_row % kQK != 0 || start < 0 || nrows < 0 || start % n_per_row != 0) {
        return set_error(B200Q8_ERR_INVALID_ARG,
                         "quantize_chunk: n_per_row must be a positive multiple of 32 and start a multiple of it");
    }
    const size_t  row_size  = (size_t) (n_per_row / kQK) * kBlockBytes;
    const int64_t start_row = start / n_per_row;
    if (written != nullptr) {
        *written = (size_t) nrows * row_size;
    }
    return b200q8_quantize_rows(src + start, nrows, n_per_row, (size_t) n_per_row * 4,
                                static_cast<uint8_t *>(dst) + (size_t) start_row * row_size, row_size,
                                B200Q8_QUANT_REF, stream);
}

b200q8_status_t b200q8_dequantize_rows(const void * src, int64_t rows, int64_t K, size_t src_row_stride, float * dst,
                                       size_t dst_row_stride, b200q8_stream_t stream) {
    if (rows < 0 || K < 0 || K % kQK != 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "dequantize_rows: K must be a non-negative multiple of 32");
    }
    if (rows == 0 || K == 0) {
        return B200Q8_OK;
    }
    if (src == nullptr || dst == nullptr || !aligned(dst, 4) || dst_row_stride % 4 != 0 ||
        (rows > 1 && (src_row_stride < (size_t) K / kQK * kBlockBytes || dst_row_stride < (size_t) K * 4))) {
        return set_error(B200Q8_ERR_INVALID_ARG, "dequantize_rows: bad pointer, alignment or stride");
    }
    cudaError_t e = launch_dequant_rows(src, src_row_stride, rows, nullptr, rows, K, dst, dst_row_stride,
                                        reinterpret_cast<cudaStream_t>(stream), current_sm_count());
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "dequantize_rows launch");
}

b200q8_status_t b200q8_get_rows(const void * table, int64_t K, int64_t rows, size_t table_row_stride,
                                const int32_t * ids, int64_t n_ids, float * out, size_t out_row_stride,
                                b200q8_stream_t stream) {
    if (K < 0 || K % kQK != 0 || rows < 0 || n_ids < 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "get_rows: K must be a non-negative multiple of 32");
    }
    if (n_ids == 0 || K == 0) {
        return B200Q8_OK;
    }
    if (table == nullptr || ids == nullptr || out == nullptr || !aligned(out, 4) || !aligned(ids, 4) ||
        out_row_stride % 4 != 0 || table_row_stride < (size_t) K / kQK * kBlockBytes ||
        (n_ids > 1 && out_row_stride < (size_t) K * 4)) {
        return set_error(B200Q8_ERR_INVALID_ARG, "get_rows: bad pointer, alignment or stride");
    }
    cudaError_t e = launch_dequant_rows(table, table_row_stride, rows, ids, n_ids, K, out, out_row_stride,
                                        reinterpret_cast<cudaStream_t>(stream), current_sm_count());
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "get_rows launch");
}

// M <= 8 products with at least this many weight bytes (default: all of
// them) run on the tensor-core GEMM too: one MMA per 16 rows x block, so the
// weight stream is HBM-bound (a 142 MB M = 1 product streams at 4.8 TB/s,
// against 2.5 TB/s for the dp4a GEMV, whose per-block instruction count caps
// it).  Calls without a large enough workspace keep the GEMV.
// B200Q8_GEMV_VIA_GEMM_MIN_BYTES overrides (bytes, read once).
static size_t gemv_via_gemm_min_bytes() {
    static const size_t v = [] {
        const char * e = getenv("B200Q8_GEMV_VIA_GEMM_MIN_BYTES");
        return e != nullptr && e[0] != '\0' ? (size_t) strtoull(e, nullptr, 10) : (size_t) 0;
    }();
    return v;
}

static bool small_m_via_gemm(int64_t K, int64_t N, int64_t M) {
    return M >= 1 && M <= 8 && (size_t) N * (size_t) (K / kQK) * kBlockBytes >= gemv_via_gemm_min_bytes();
}

// Workspace every path but the tcgen05 GEMM can run in: the larger of the
// general path's quantized activations (M rows of K/32 blocks) and the
// mma.sync GEMM's staged activation records.
static size_t base_workspace_size(int64_t K, int64_t N, int64_t M) {
    const size_t general = align_up((size_t) M * (size_t) (K / kQK) * kBlockBytes, 256);
    const size_t staged  = K % 256 == 0 ? align_up(gemm_workspace_bytes(K, M), 256) : 0;
    return M > 8 || small_m_via_gemm(K, N, M) ? std::max(general, staged) : general;
}

// Shapes the tcgen05 GEMM takes (given aligned pointers), when it is on.
static bool tc_shape(int64_t K, int64_t N, int64_t M) {
    const int64_t min_m = gemm_tc_min_m();
    return min_m > 0 && M >= min_m && M > 8 && K % 256 == 0 && N >= 1;
}

size_t b200q8_mul_mat_workspace_size(int64_t K, int64_t N, int64_t M) {
    if (K <= 0 || M <= 0 || K % kQK != 0) {
        return 0;
    }
    const size_t base = base_workspace_size(K, N, M);
    return tc_shape(K, N, M) ? std::max(base, align_up(gemm_tc_workspace_bytes(K, N, M), 256)) : base;
}

b200q8_status_t b200q8_mul_mat(const void * w, int64_t K, int64_t N, size_t w_row_bytes, const float * x, int64_t M,
                               size_t x_col_stride, float * y, size_t y_col_stride, int32_t mode, void * workspace,
                               size_t workspace_bytes, b200q8_stream_t stream) {
    if (K <= 0 || K % kQK != 0 || N < 0 || M < 0) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat: K (%lld) must be a positive multiple of 32",
                         (long long) K);
    }
    if (!valid_mode(mode)) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat: unknown mode %d", mode);
    }
    if (N == 0 || M == 0) {
        return B200Q8_OK;
    }
    if (N > INT32_MAX || K > INT32_MAX) {
        return set_error(B200Q8_ERR_UNSUPPORTED, "mul_mat: N and K must fit in 32 bits");
    }
    const size_t min_row = (size_t) (K / kQK) * kBlockBytes;
    if (w == nullptr || x == nullptr || y == nullptr || w_row_bytes < min_row || !aligned(x, 4) || !aligned(y, 4) ||
        x_col_stride % 4 != 0 || y_col_stride % 4 != 0 ||
        (M > 1 && (x_col_stride < (size_t) K * 4 || y_col_stride < (size_t) N * 4))) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat: bad pointer, alignment, row size or stride");
    }
    cudaStream_t st  = reinterpret_cast<cudaStream_t>(stream);
    const int    sms = current_sm_count();
    const size_t xs  = M > 1 ? x_col_stride / 4 : (size_t) K;
    const size_t ys  = M > 1 ? y_col_stride / 4 : (size_t) N;

    GemvParams p = {};
    p.w          = static_cast<const uint8_t *>(w);
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
    // large M, when switched on: the tcgen05 GEMM if the workspace holds its
    // planes (the workspace size query then asks for them); else the mma.sync
    // GEMM below
    if (tc_shape(K, N, M) && gemm_tc_supported(p.w, w_row_bytes, K, N, M, x, xs) && workspace != nullptr &&
        aligned(workspace, 16) && workspace_bytes >= gemm_tc_workspace_bytes(K, N, M)) {
        cudaError_t e = launch_gemm_tc(p.w, w_row_bytes, K, N, x, xs, M, y, ys, mode, workspace, st, sms);
        return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "mul_mat: tcgen05 GEMM launch");
    }
    if (M > 8 && gemm_supported(p.w, w_row_bytes, K, N, M)) {
        const size_t need = base_workspace_size(K, N, M);
        if (workspace == nullptr || workspace_bytes < need) {
            return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat: M > 8 needs %zu bytes of workspace (got %zu)", need,
                             workspace_bytes);
        }
        cudaError_t e = launch_gemm(p.w, w_row_bytes, K, N, x, xs, M, y, ys, mode, workspace, st, sms);
        return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "mul_mat: tensor-core GEMM launch");
    }
    if (small_m_via_gemm(K, N, M) && gemm_supported(p.w, w_row_bytes, K, N, M) && workspace != nullptr &&
        workspace_bytes >= gemm_workspace_bytes(K, M)) {
        cudaError_t e = launch_gemm(p.w, w_row_bytes, K, N, x, xs, M, y, ys, mode, workspace, st, sms);
        return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "mul_mat: tensor-core GEMM launch");
    }
    if (gemv_supported(p)) {
        for (int64_t m0 = 0; m0 < M; m0 += 8) {
            p.M           = (int) std::min<int64_t>(M - m0, 8);
            p.x           = x + m0 * xs;
            p.y           = y + m0 * ys;
            cudaError_t e = launch_gemv(p, st, sms, false);
            if (e != cudaSuccess) {
                return cuda_error(e, "mul_mat: gemv launch");
            }
        }
        return B200Q8_OK;
    }
    // General shapes: quantize x into the workspace, then a plain kernel.
    const size_t need = base_workspace_size(K, N, M);
    if (workspace == nullptr || workspace_bytes < need) {
        return set_error(B200Q8_ERR_INVALID_ARG, "mul_mat: this shape needs %zu bytes of workspace (got %zu)", need,
                         workspace_bytes);
    }
    const size_t xq_row = min_row;
    cudaError_t  e      = launch_quantize(x, M, K, xs * 4, workspace, xq_row, mode, st, sms);
    if (e == cudaSuccess) {
        e = launch_gemv_generic(static_cast<const uint8_t *>(w), w_row_bytes, K, N,
                                static_cast<const uint8_t *>(workspace), M, y, ys * 4, st);
    }
    return e == cudaSuccess ? B200Q8_OK : cuda_error(e, "mul_mat: general path launch");
}

}  // extern "C"
