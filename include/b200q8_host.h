/* b200q8_host.h -- the C++ host side of Qwen3-TTS decoding on the B200 Q8_0
 * path: a package loaded onto one GPU and the per-frame decode loop, driven
 * from host code the way the reference drives its ggml graphs.
 *
 * Exported by libb200q8_host.so (C++17 over the C ABI of libb200q8.so and
 * the CUDA runtime).  It replaces, for the talker + code predictor, the two
 * halves of the reference's synthesis path that reach the Q8_0 hot path:
 *   b200q8h_decoder_load  -- synth_model_load's package load
 *                            (src/synthesize.cpp:575-682, weights placed by
 *                            src/arch/qwen3-tts/model.cpp:573-698), here
 *                            b200q8_gguf_open + b200q8_gguf_decoder on the
 *                            device instead of ggml-cpu buffers;
 *   b200q8h_decoder_run   -- the frame loop of run_synthesis
 *                            (src/arch/qwen3-tts/model.cpp:1310-1489): each
 *                            frame's text token, the talker step, the
 *                            semantic code, the code predictor's calls, the
 *                            frame's codes read back to the host before the
 *                            next frame is formed, and the stop on the codec
 *                            end-of-speech code.
 * Greedy selection (request.sample == false) or replayed codes; sampling with
 * a temperature stays on the host in the reference and is not offered here.
 * Every call returns a b200q8_status_t; the message of the calling thread's
 * last failure is in b200q8h_last_error(). */
#ifndef B200Q8_HOST_H
#define B200Q8_HOST_H

#include "b200q8.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200q8h_decoder b200q8h_decoder;

typedef struct b200q8h_decoder_params {
    int32_t device;       /* CUDA device index                                     */
    int64_t max_streams;  /* streams decoded together (M of every frame), >= 1      */
    int64_t n_ctx;        /* talker positions cached per stream                    */
    int32_t mode;         /* activation quantizer, B200Q8_QUANT_*                  */
} b200q8h_decoder_params;

typedef struct b200q8h_decoder_info {
    int64_t hidden;       /* talker hidden width                                   */
    int32_t groups;       /* codes per frame (code_group_count)                    */
    int64_t talker_vocab; /* codec vocabulary of code 0                            */
    int64_t text_hidden;  /* 0 when the package has no text projection           */
    int64_t text_vocab;
} b200q8h_decoder_info;

/* Loads a Q8_MIXED Qwen3-TTS package (GGUF) onto params->device: the talker
 * with attention, codec head and text projection, the code predictor, and the
 * decode frame over them.  A package whose tensors are not in the types the
 * path takes (Q8_0 projections and tables, F32 norms and biases) is
 * B200Q8_ERR_UNSUPPORTED; a malformed one B200Q8_ERR_INVALID_ARG. */
b200q8_status_t b200q8h_decoder_load(const char * package_path, const b200q8h_decoder_params * params,
                                     b200q8h_decoder ** out);
b200q8_status_t b200q8h_decoder_info_get(const b200q8h_decoder * dec, b200q8h_decoder_info * out);

typedef struct b200q8h_run_params {
    int64_t         M;          /* streams, 1 .. max_streams                                      */
    int64_t         n_frames;   /* frames to run at most                                          */
    /* each frame's text input, host memory: text_ids [n_frames][M] (needs the
     * package's text projection) or text_rows [n_frames][M][hidden]; one of
     * the two */
    const int32_t * text_ids;
    const float *   text_rows;
    const int32_t * first_prev; /* [M][groups] codes before frame 0 (host); NULL: all zero         */
    int32_t         start_pos;  /* talker position of frame 0 (the prompt's length)               */
    const int32_t * replay;     /* [n_frames][M][groups] codes to take instead of choosing; NULL   */
    int32_t         stop_code;  /* a stream ends at the frame whose code 0 is this; < 0: none      */
} b200q8h_run_params;

/* Runs up to n_frames frames for M streams (slot m = stream m; each stream's
 * chosen-code history is cleared first).  codes [n_frames][M][groups] (host)
 * receives every frame's codes; frames_out [M] (host) the frames each stream
 * ran before its stop code (the stop frame itself excluded, as the reference
 * does not emit it).  The loop ends when every stream has stopped or after
 * n_frames.  Frames of streams that already stopped still run (the batch
 * stays fixed) and their codes are left as computed. */
b200q8_status_t b200q8h_decoder_run(b200q8h_decoder * dec, const b200q8h_run_params * params, int32_t * codes,
                                    int64_t * frames_out);

void b200q8h_decoder_free(b200q8h_decoder * dec);

/* The status and message of the calling thread's last failed b200q8h_ call
 * (a failure inside libb200q8.so carries that library's message). */
b200q8_status_t b200q8h_last_error(char * buf, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* B200Q8_HOST_H */
