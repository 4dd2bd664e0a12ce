/* b200q8_gguf.h -- GGUF packages on the B200 Q8_0 path.
 *
 * Reads a package's metadata and tensor table (the format the reference loads
 * through src/gguf-metadata.cpp:12-46) and builds the talker decode step of a
 * Qwen3-TTS package from it: hyperparameters under
 * "synthesize.qwen3-tts.talker.*" (src/arch/qwen3-tts/weights.cpp:128-138),
 * tensors named as the reference's catalog resolves them
 * (src/arch/qwen3-tts/catalog.cpp:239-281).  The file is memory-mapped; tensor
 * data pointers are host pointers into the mapping, valid until close.
 * Exported by libb200q8.so.  Every call returns a b200q8_status_t; the
 * message is in b200q8_last_error(). */
#ifndef B200Q8_GGUF_H
#define B200Q8_GGUF_H

#include "b200q8.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200q8_gguf b200q8_gguf;

typedef struct {
    const char * name;    /* NUL-terminated copy, owned by the handle */
    int32_t      type;    /* ggml type id (B200Q8_GGML_TYPE_* values: F32 0, F16 1, Q8_0 8, BF16 30, ...) */
    int32_t      n_dims;
    int64_t      ne[4];   /* ggml order: ne[0] contiguous; unused dims are 1 */
    uint64_t     offset;  /* bytes from the start of the data section */
    uint64_t     nbytes;  /* 0 for a type this library does not size */
    const void * data;    /* host pointer into the mapped file */
} b200q8_gguf_tensor_info;

/* Opens and validates a GGUF file (versions 2 and 3): every string, count,
 * tensor extent and offset is checked against the file size; anything
 * malformed is B200Q8_ERR_INVALID_ARG. */
b200q8_status_t b200q8_gguf_open(const char * path, b200q8_gguf ** out);
void            b200q8_gguf_close(b200q8_gguf * g);

int64_t         b200q8_gguf_tensor_count(const b200q8_gguf * g);
/* Index of the tensor with this name, or -1. */
int64_t         b200q8_gguf_find_tensor(const b200q8_gguf * g, const char * name);
b200q8_status_t b200q8_gguf_tensor(const b200q8_gguf * g, int64_t index, b200q8_gguf_tensor_info * out);

/* Scalar metadata; a missing key or another value type is B200Q8_ERR_INVALID_ARG. */
b200q8_status_t b200q8_gguf_get_u32(const b200q8_gguf * g, const char * key, uint32_t * out);
b200q8_status_t b200q8_gguf_get_f32(const b200q8_gguf * g, const char * key, float * out);
/* String metadata, NUL-terminated into buf (truncated to buf_size - 1). */
b200q8_status_t b200q8_gguf_get_str(const b200q8_gguf * g, const char * key, char * buf, size_t buf_size);

/* The talker decode step of a Qwen3-TTS package, on `device`: uploads the
 * layers' Q8_0 projections, their F32 RMS-norm weights and the Q8_0
 * codec_embedding table into one device buffer the chain owns, then
 * b200q8_chain_create with these hyperparameters.  A projection or the
 * table in another type (a non-Q8_MIXED package) is B200Q8_ERR_UNSUPPORTED. */
b200q8_status_t b200q8_gguf_talker_chain(const b200q8_gguf * g, int32_t device, int64_t max_m, int32_t mode,
                                         b200q8_chain ** out);

/* Everything one decode frame needs, from a package, on `device`:
 *   *talker     the talker step with the reference's attention (per-layer
 *               self_attn.q_norm / k_norm, talker.rope_theta; n_ctx cached
 *               positions for each of n_slots streams) and output stage
 *               (talker.model.norm, talker.codec_head);
 *   *predictor  the code predictor (talker.code_predictor.model.layers.*,
 *               its norm and lm_head.{g}; cache of code_group_count
 *               positions; max_m = max(8, 2 * max_m)) with its codec tables;
 *   *frame      (optional: frame may be NULL) b200q8_frame_create over both,
 *               with sampling.repetition_penalty (1 when the key is absent)
 *               and, when the package holds talker.model.text_embedding,
 *               the talker's text projection (its Q8_0 embedding and
 *               text_projection.linear_fc1 / linear_fc2 with F32 biases,
 *               talker.text_hidden_size / text_vocab_size), so that frames
 *               run from text token ids.
 * Hyperparameters follow weights.cpp:128-212 (the predictor's
 * intermediate_size falls back to the talker's; eps and rope_theta are the
 * talker's, model.cpp:315-322).  A predictor of another width than the
 * talker gets its small_to_mtp_projection (Q8_0 weight, F32 bias) uploaded
 * and handed to the frame.  A tensor not in Q8_0 / F32 as the step needs is
 * B200Q8_ERR_UNSUPPORTED.  Each chain owns its weights; destroy the frame
 * before the chains. */
b200q8_status_t b200q8_gguf_decoder(const b200q8_gguf * g, int32_t device, int64_t max_m, int32_t mode,
                                    int64_t n_ctx, int64_t n_slots, b200q8_chain ** talker,
                                    b200q8_chain ** predictor, b200q8_frame ** frame);

#ifdef __cplusplus
}
#endif

#endif /* B200Q8_GGUF_H */
