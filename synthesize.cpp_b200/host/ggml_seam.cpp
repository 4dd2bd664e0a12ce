// ggml_seam.cpp -- ggml-backend supports_op / graph_compute for the Q8_0
// MUL_MAT and GET_ROWS nodes, over the C ABI of libb200q8.so.
//
// The reference's CPU path computes these nodes in ggml-cpu (reached from
// src/arch/qwen3-tts/operations.cpp:39-41,90-92,142, talker.cpp:44,86, through
// GraphRun::run, model.cpp:101-126).  A backend module claims a node with
// supports_op and computes it here: 2-D slices go straight to
// b200q8_mul_mat / b200q8_get_rows; dims 2 and 3 loop over slices with ggml's
// broadcast rule.
#include "b200q8_ggml.h"

#include <algorithm>
#include <cstdint>

namespace {

bool is_contiguous_rows(const b200q8_ggml_tensor * t, size_t elem) {
    return t->nb[0] == elem;
}

bool mul_mat_ok(const b200q8_ggml_tensor * n) {
    const b200q8_ggml_tensor * w = n->src[0];
    const b200q8_ggml_tensor * x = n->src[1];
    if (w == nullptr || x == nullptr || w->type != B200Q8_GGML_TYPE_Q8_0 || x->type != B200Q8_GGML_TYPE_F32 ||
        n->type != B200Q8_GGML_TYPE_F32) {
        return false;
    }
    const int64_t K = w->ne[0];
    if (K <= 0 || K % B200Q8_QK8_0 != 0 || x->ne[0] != K || n->ne[0] != w->ne[1] || n->ne[1] != x->ne[1] ||
        n->ne[2] != x->ne[2] || n->ne[3] != x->ne[3]) {
        return false;
    }
    if (w->ne[2] <= 0 || w->ne[3] <= 0 || x->ne[2] % w->ne[2] != 0 || x->ne[3] % w->ne[3] != 0) {
        return false;
    }
    // Q8_0 rows are whole blocks; activations and result need unit element stride
    return w->nb[0] == B200Q8_BLOCK_BYTES && w->nb[1] >= (size_t) (K / B200Q8_QK8_0) * B200Q8_BLOCK_BYTES &&
           is_contiguous_rows(x, sizeof(float)) && is_contiguous_rows(n, sizeof(float));
}

bool get_rows_ok(const b200q8_ggml_tensor * n) {
    const b200q8_ggml_tensor * t   = n->src[0];
    const b200q8_ggml_tensor * ids = n->src[1];
    if (t == nullptr || ids == nullptr || t->type != B200Q8_GGML_TYPE_Q8_0 || ids->type != B200Q8_GGML_TYPE_I32 ||
        n->type != B200Q8_GGML_TYPE_F32) {
        return false;
    }
    const int64_t K = t->ne[0];
    // ggml_get_rows: result [K, ids->ne[0], ids->ne[1], ids->ne[2]]; table dims 2,3 follow ids dims 1,2
    return K > 0 && K % B200Q8_QK8_0 == 0 && n->ne[0] == K && n->ne[1] == ids->ne[0] && n->ne[2] == ids->ne[1] &&
           n->ne[3] == ids->ne[2] && ids->nb[0] == sizeof(int32_t) && is_contiguous_rows(n, sizeof(float)) &&
           t->nb[0] == B200Q8_BLOCK_BYTES && ids->ne[1] == t->ne[2] && ids->ne[2] == t->ne[3];
}

}  // namespace

extern "C" {

int32_t b200q8_ggml_supports_op(const b200q8_ggml_tensor * node) {
    if (node == nullptr) {
        return 0;
    }
    switch (node->op) {
        case B200Q8_GGML_OP_MUL_MAT: return mul_mat_ok(node) ? 1 : 0;
        case B200Q8_GGML_OP_GET_ROWS: return get_rows_ok(node) ? 1 : 0;
        default: return 0;
    }
}

size_t b200q8_ggml_workspace_size(const b200q8_ggml_tensor * node) {
    if (node == nullptr || node->op != B200Q8_GGML_OP_MUL_MAT || !mul_mat_ok(node)) {
        return 0;
    }
    // slices run one after another on one stream and share the workspace
    return b200q8_mul_mat_workspace_size(node->src[0]->ne[0], node->src[0]->ne[1], node->src[1]->ne[1]);
}

b200q8_status_t b200q8_ggml_compute_node(const b200q8_ggml_tensor * node, void * workspace, size_t workspace_bytes,
                                         int32_t mode, b200q8_stream_t stream) {
    if (!b200q8_ggml_supports_op(node)) {
        return B200Q8_ERR_UNSUPPORTED;
    }
    if (node->op == B200Q8_GGML_OP_MUL_MAT) {
        const b200q8_ggml_tensor * w  = node->src[0];
        const b200q8_ggml_tensor * x  = node->src[1];
        const int64_t              r2 = x->ne[2] / w->ne[2];
        const int64_t              r3 = x->ne[3] / w->ne[3];
        for (int64_t i13 = 0; i13 < x->ne[3]; ++i13) {
            for (int64_t i12 = 0; i12 < x->ne[2]; ++i12) {
                const uint8_t * wp = static_cast<const uint8_t *>(w->data) + (i12 / r2) * w->nb[2] + (i13 / r3) * w->nb[3];
                const uint8_t * xp = static_cast<const uint8_t *>(x->data) + i12 * x->nb[2] + i13 * x->nb[3];
                uint8_t *       yp = static_cast<uint8_t *>(node->data) + i12 * node->nb[2] + i13 * node->nb[3];
                const b200q8_status_t st = b200q8_mul_mat(wp, w->ne[0], w->ne[1], w->nb[1],
                                                          reinterpret_cast<const float *>(xp), x->ne[1], x->nb[1],
                                                          reinterpret_cast<float *>(yp), node->nb[1], mode, workspace,
                                                          workspace_bytes, stream);
                if (st != B200Q8_OK) {
                    return st;
                }
            }
        }
        return B200Q8_OK;
    }
    const b200q8_ggml_tensor * t   = node->src[0];
    const b200q8_ggml_tensor * ids = node->src[1];
    for (int64_t i2 = 0; i2 < ids->ne[2]; ++i2) {
        for (int64_t i1 = 0; i1 < ids->ne[1]; ++i1) {
            const uint8_t * tp = static_cast<const uint8_t *>(t->data) + i1 * t->nb[2] + i2 * t->nb[3];
            const uint8_t * ip = static_cast<const uint8_t *>(ids->data) + i1 * ids->nb[1] + i2 * ids->nb[2];
            uint8_t *       op = static_cast<uint8_t *>(node->data) + i1 * node->nb[2] + i2 * node->nb[3];
            const b200q8_status_t st =
                b200q8_get_rows(tp, t->ne[0], t->ne[1], t->nb[1], reinterpret_cast<const int32_t *>(ip), ids->ne[0],
                                reinterpret_cast<float *>(op), node->nb[1], stream);
            if (st != B200Q8_OK) {
                return st;
            }
        }
    }
    return B200Q8_OK;
}

b200q8_status_t b200q8_ggml_graph_compute(const b200q8_ggml_tensor * const * nodes, int32_t n_nodes, void * workspace,
                                          size_t workspace_bytes, int32_t mode, b200q8_stream_t stream) {
    if (n_nodes < 0 || (n_nodes > 0 && nodes == nullptr)) {
        return B200Q8_ERR_INVALID_ARG;
    }
    for (int32_t i = 0; i < n_nodes; ++i) {
        const b200q8_status_t st = b200q8_ggml_compute_node(nodes[i], workspace, workspace_bytes, mode, stream);
        if (st != B200Q8_OK) {
            return st;
        }
    }
    return B200Q8_OK;
}

}  // extern "C"
