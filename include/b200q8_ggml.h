// b200q8_ggml.h -- the ggml-backend face of the B200 Q8_0 path (host C++).
//
// A ggml backend decides per graph node whether it can run it
// (`supports_op`, reached from BackendPlan::assign_to_primary,
// src/backend-plan.cpp:149-156) and then computes the nodes it claimed
// (`graph_compute`).  This header mirrors the part of `struct ggml_tensor`
// that MUL_MAT and GET_ROWS nodes carry -- type, op, ne[4], nb[4], data,
// src[0..1] -- with ggml's type ids, so a backend module can fill it
// field-for-field from a real ggml_tensor and hand it over.  The broadcast
// rules are ggml's: src0 dims 2 and 3 are repeated over src1's
// (i02 = i12 / (ne12/ne02), i03 = i13 / (ne13/ne03)).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "b200q8.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type values (ggml.h; gguf-py GGMLQuantizationType) for the types this path uses. */
#define B200Q8_GGML_TYPE_F32  0
#define B200Q8_GGML_TYPE_F16  1
#define B200Q8_GGML_TYPE_Q8_0 8
#define B200Q8_GGML_TYPE_I32  26

/* The two ops of the path. */
#define B200Q8_GGML_OP_MUL_MAT  1
#define B200Q8_GGML_OP_GET_ROWS 2

typedef struct b200q8_ggml_tensor {
    int32_t                            type;
    int32_t                            op; /* B200Q8_GGML_OP_* for nodes, 0 for leaves */
    int64_t                            ne[4];
    size_t                             nb[4];
    void *                             data; /* device memory */
    const struct b200q8_ggml_tensor *  src[2];
} b200q8_ggml_tensor;

/* ggml_backend supports_op: 1 when this path computes `node` exactly as
 * ggml-cpu does (MUL_MAT of a Q8_0 src0 by an F32 src1 into F32; GET_ROWS of
 * a Q8_0 table by I32 ids into F32), with contiguous rows. */
int32_t b200q8_ggml_supports_op(const b200q8_ggml_tensor * node);

/* Device scratch the node needs (0 for GET_ROWS). */
size_t b200q8_ggml_workspace_size(const b200q8_ggml_tensor * node);

/* Computes one claimed node on `stream`.  workspace: at least
 * b200q8_ggml_workspace_size(node) bytes of device memory. */
b200q8_status_t b200q8_ggml_compute_node(const b200q8_ggml_tensor * node, void * workspace, size_t workspace_bytes,
                                         int32_t mode, b200q8_stream_t stream);

/* ggml_backend graph_compute over the claimed nodes, in order. */
b200q8_status_t b200q8_ggml_graph_compute(const b200q8_ggml_tensor * const * nodes, int32_t n_nodes, void * workspace,
                                          size_t workspace_bytes, int32_t mode, b200q8_stream_t stream);

#ifdef __cplusplus
}
#endif
