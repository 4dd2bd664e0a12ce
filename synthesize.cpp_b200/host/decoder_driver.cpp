// decoder_driver.cpp -- b200q8h_decoder_*: a Qwen3-TTS package loaded onto one
// GPU and its per-frame decode loop, in host C++ over the C ABI of
// libb200q8.so and the CUDA runtime.
//
// The reference loads a package in synth_model_load (src/synthesize.cpp:
// 575-682; the talker and predictor weights go to CPU ggml buffers at
// src/arch/qwen3-tts/model.cpp:573-698) and decodes it in run_synthesis's
// frame loop (model.cpp:1310-1489): every frame it sets the frame's text
// token and position, computes the talker graph, reads the logits back and
// chooses code 0, stops on the codec end-of-speech code, then runs the code
// predictor's calls and reads each of their codes.  Here the whole frame
// (text projection, talker step, selection, predictor) is one device graph
// (b200q8_frame_run); the host keeps what the reference's host keeps: the
// loop, each frame's inputs, the frame's codes read back before the next frame
// is formed, and the stop decision.
#include "b200q8_gguf.h"
#include "b200q8_host.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

namespace {

thread_local b200q8_status_t t_status = B200Q8_OK;
thread_local std::string     t_message;

b200q8_status_t fail(b200q8_status_t code, const char * fmt, ...) {
    char    buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_status  = code;
    t_message = buf;
    return code;
}

// A failure inside libb200q8.so: keep its message.
b200q8_status_t fail_lib(b200q8_status_t code, const char * what) {
    char buf[512] = {};
    b200q8_last_error(buf, sizeof(buf));
    return fail(code, "%s: %s", what, buf);
}

b200q8_status_t fail_cuda(cudaError_t e, const char * what) {
    return fail(e == cudaErrorMemoryAllocation ? B200Q8_ERR_OOM : B200Q8_ERR_BACKEND, "%s: %s", what,
                cudaGetErrorString(e));
}

// Restores the caller's current device on scope exit.
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        cudaGetDevice(&prev);
        cudaSetDevice(dev);
    }
    ~DeviceScope() {
        if (prev >= 0) {
            cudaSetDevice(prev);
        }
    }
};

}  // namespace

struct b200q8h_decoder {
    b200q8_chain *       talker    = nullptr;
    b200q8_chain *       predictor = nullptr;
    b200q8_frame *       frame     = nullptr;
    int32_t              device    = 0;
    int64_t              max_m     = 0;
    b200q8h_decoder_info info      = {};
    cudaStream_t         stream    = nullptr;
    // device buffers
    int32_t * d_ids    = nullptr;  // [max_m] this frame's text token ids
    float *   d_text   = nullptr;  // [max_m][hidden] this frame's text rows
    int32_t * d_codes[2] = {};     // [max_m][G] codes, ping-pong: the previous frame's are the next prev
    int32_t * d_pos    = nullptr;  // [max_m]
    int32_t * d_replay = nullptr;  // [max_m][G]
    // pinned host staging
    int32_t * h_ids    = nullptr;
    float *   h_text   = nullptr;
    int32_t * h_codes  = nullptr;
    int32_t * h_pos    = nullptr;
    int32_t * h_replay = nullptr;
};

namespace {

void release(b200q8h_decoder * d) {
    if (d == nullptr) {
        return;
    }
    DeviceScope scope(d->device);
    if (d->stream != nullptr) {
        cudaStreamSynchronize(d->stream);
    }
    b200q8_frame_destroy(d->frame);
    b200q8_chain_destroy(d->talker);
    b200q8_chain_destroy(d->predictor);
    for (void * p : { (void *) d->d_ids, (void *) d->d_text, (void *) d->d_codes[0], (void *) d->d_codes[1],
                      (void *) d->d_pos, (void *) d->d_replay }) {
        if (p != nullptr) {
            cudaFree(p);
        }
    }
    for (void * p : { (void *) d->h_ids, (void *) d->h_text, (void *) d->h_codes, (void *) d->h_pos,
                      (void *) d->h_replay }) {
        if (p != nullptr) {
            cudaFreeHost(p);
        }
    }
    if (d->stream != nullptr) {
        cudaStreamDestroy(d->stream);
    }
    delete d;
}

b200q8_status_t read_info(const b200q8_gguf * g, b200q8h_decoder_info & info) {
    const std::string tp = "synthesize.qwen3-tts.talker.";
    uint32_t          hidden = 0, groups = 0, vocab = 0, th = 0, tv = 0;
    if (b200q8_gguf_get_u32(g, (tp + "hidden_size").c_str(), &hidden) != B200Q8_OK ||
        b200q8_gguf_get_u32(g, (tp + "code_group_count").c_str(), &groups) != B200Q8_OK ||
        b200q8_gguf_get_u32(g, (tp + "codec_vocab_size").c_str(), &vocab) != B200Q8_OK) {
        return fail_lib(B200Q8_ERR_INVALID_ARG, "decoder_load");
    }
    info.hidden       = hidden;
    info.groups       = (int32_t) groups;
    info.talker_vocab = vocab;
    if (b200q8_gguf_find_tensor(g, "talker.model.text_embedding.weight") >= 0 &&
        b200q8_gguf_get_u32(g, (tp + "text_hidden_size").c_str(), &th) == B200Q8_OK &&
        b200q8_gguf_get_u32(g, (tp + "text_vocab_size").c_str(), &tv) == B200Q8_OK) {
        info.text_hidden = th;
        info.text_vocab  = tv;
    }
    return B200Q8_OK;
}

}  // namespace

extern "C" {

b200q8_status_t b200q8h_last_error(char * buf, size_t len) {
    if (buf != nullptr && len > 0) {
        const size_t n = std::min(len - 1, t_message.size());
        std::memcpy(buf, t_message.data(), n);
        buf[n] = '\0';
    }
    return t_status;
}

b200q8_status_t b200q8h_decoder_load(const char * package_path, const b200q8h_decoder_params * params,
                                     b200q8h_decoder ** out) {
    if (package_path == nullptr || params == nullptr || out == nullptr || params->max_streams < 1 ||
        params->n_ctx < 1) {
        return fail(B200Q8_ERR_INVALID_ARG, "decoder_load: null argument or non-positive size");
    }
    *out             = nullptr;
    b200q8_gguf * g  = nullptr;
    b200q8_status_t st = b200q8_gguf_open(package_path, &g);
    if (st != B200Q8_OK) {
        return fail_lib(st, "decoder_load");
    }
    auto * d   = new (std::nothrow) b200q8h_decoder();
    if (d == nullptr) {
        b200q8_gguf_close(g);
        return fail(B200Q8_ERR_OOM, "decoder_load: out of host memory");
    }
    d->device = params->device;
    d->max_m  = params->max_streams;
    st        = read_info(g, d->info);
    if (st == B200Q8_OK) {
        st = b200q8_gguf_decoder(g, params->device, params->max_streams, params->mode, params->n_ctx,
                                 params->max_streams, &d->talker, &d->predictor, &d->frame);
        if (st != B200Q8_OK) {
            fail_lib(st, "decoder_load");
        }
    }
    b200q8_gguf_close(g);  // the chains hold device copies of everything they use
    if (st != B200Q8_OK) {
        release(d);
        return st;
    }
    DeviceScope  scope(d->device);
    const size_t M = (size_t) d->max_m, H = (size_t) d->info.hidden, G = (size_t) d->info.groups;
    cudaError_t  e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
    auto dev = [&](void ** p, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc(p, std::max<size_t>(bytes, 16));
        if (e == cudaSuccess) e = cudaMemset(*p, 0, std::max<size_t>(bytes, 16));
    };
    auto pin = [&](void ** p, size_t bytes) {
        if (e == cudaSuccess) e = cudaMallocHost(p, std::max<size_t>(bytes, 16));
    };
    dev((void **) &d->d_ids, M * 4);
    dev((void **) &d->d_text, M * H * 4);
    dev((void **) &d->d_codes[0], M * G * 4);
    dev((void **) &d->d_codes[1], M * G * 4);
    dev((void **) &d->d_pos, M * 4);
    dev((void **) &d->d_replay, M * G * 4);
    pin((void **) &d->h_ids, M * 4);
    pin((void **) &d->h_text, M * H * 4);
    pin((void **) &d->h_codes, M * G * 4);
    pin((void **) &d->h_pos, M * 4);
    pin((void **) &d->h_replay, M * G * 4);
    if (e != cudaSuccess) {
        st = fail_cuda(e, "decoder_load: device buffers");
        release(d);
        return st;
    }
    *out = d;
    return B200Q8_OK;
}

b200q8_status_t b200q8h_decoder_info_get(const b200q8h_decoder * dec, b200q8h_decoder_info * out) {
    if (dec == nullptr || out == nullptr) {
        return fail(B200Q8_ERR_INVALID_ARG, "decoder_info_get: null argument");
    }
    *out = dec->info;
    return B200Q8_OK;
}

b200q8_status_t b200q8h_decoder_run(b200q8h_decoder * d, const b200q8h_run_params * p, int32_t * codes,
                                    int64_t * frames_out) {
    if (d == nullptr || p == nullptr || codes == nullptr || frames_out == nullptr) {
        return fail(B200Q8_ERR_INVALID_ARG, "decoder_run: null argument");
    }
    if (p->M < 1 || p->M > d->max_m || p->n_frames < 0 || (p->text_ids == nullptr) == (p->text_rows == nullptr)) {
        return fail(B200Q8_ERR_INVALID_ARG, "decoder_run: M must be in [1, %lld], n_frames >= 0, and exactly one of "
                                            "text_ids / text_rows given", (long long) d->max_m);
    }
    if (p->text_ids != nullptr && d->info.text_hidden == 0) {
        return fail(B200Q8_ERR_INVALID_ARG, "decoder_run: text_ids need a package with a text projection");
    }
    if (p->text_ids != nullptr) {
        for (int64_t i = 0; i < p->n_frames * p->M; ++i) {
            if (p->text_ids[i] < 0 || p->text_ids[i] >= d->info.text_vocab) {
                return fail(B200Q8_ERR_INVALID_ARG, "decoder_run: text id %d at %lld is outside the vocabulary",
                            p->text_ids[i], (long long) i);
            }
        }
    }
    DeviceScope   scope(d->device);
    const int64_t M = p->M, G = d->info.groups, H = d->info.hidden;
    cudaStream_t  s = d->stream;
    // a new utterance per stream: empty chosen-code history, the given first prev codes
    b200q8_status_t st = b200q8_frame_reset_history(d->frame, -1, s);
    if (st != B200Q8_OK) {
        return fail_lib(st, "decoder_run");
    }
    cudaError_t e = p->first_prev != nullptr
                        ? cudaMemcpyAsync(d->d_codes[0], p->first_prev, (size_t) (M * G) * 4, cudaMemcpyHostToDevice, s)
                        : cudaMemsetAsync(d->d_codes[0], 0, (size_t) (M * G) * 4, s);
    std::vector<int> stopped((size_t) M, 0);
    for (int64_t m = 0; m < M; ++m) {
        frames_out[m] = 0;
    }
    int64_t live = M;
    for (int64_t f = 0; f < p->n_frames && live > 0 && e == cudaSuccess; ++f) {
        // this frame's inputs, staged through pinned memory
        for (int64_t m = 0; m < M; ++m) {
            d->h_pos[m] = p->start_pos + (int32_t) f;
        }
        e = cudaMemcpyAsync(d->d_pos, d->h_pos, (size_t) M * 4, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess && p->text_ids != nullptr) {
            std::memcpy(d->h_ids, p->text_ids + f * M, (size_t) M * 4);
            e = cudaMemcpyAsync(d->d_ids, d->h_ids, (size_t) M * 4, cudaMemcpyHostToDevice, s);
        } else if (e == cudaSuccess) {
            std::memcpy(d->h_text, p->text_rows + f * M * H, (size_t) (M * H) * 4);
            e = cudaMemcpyAsync(d->d_text, d->h_text, (size_t) (M * H) * 4, cudaMemcpyHostToDevice, s);
        }
        if (e == cudaSuccess && p->replay != nullptr) {
            std::memcpy(d->h_replay, p->replay + f * M * G, (size_t) (M * G) * 4);
            e = cudaMemcpyAsync(d->d_replay, d->h_replay, (size_t) (M * G) * 4, cudaMemcpyHostToDevice, s);
        }
        if (e != cudaSuccess) {
            break;
        }
        int32_t *         out = d->d_codes[(f + 1) & 1];
        b200q8_frame_args a   = {};
        a.M                   = M;
        a.text                = p->text_ids != nullptr ? nullptr : d->d_text;
        a.text_ids            = p->text_ids != nullptr ? d->d_ids : nullptr;
        a.prev                = d->d_codes[f & 1];
        a.pos                 = d->d_pos;
        a.replay              = p->replay != nullptr ? d->d_replay : nullptr;
        a.codes               = out;
        st                    = b200q8_frame_run(d->frame, &a, s);
        if (st != B200Q8_OK) {
            return fail_lib(st, "decoder_run");
        }
        // the frame's codes come back before the next frame is formed
        e = cudaMemcpyAsync(d->h_codes, out, (size_t) (M * G) * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) {
            e = cudaStreamSynchronize(s);
        }
        if (e != cudaSuccess) {
            break;
        }
        std::memcpy(codes + f * M * G, d->h_codes, (size_t) (M * G) * 4);
        for (int64_t m = 0; m < M; ++m) {
            if (stopped[(size_t) m]) {
                continue;
            }
            if (p->stop_code >= 0 && d->h_codes[m * G] == p->stop_code) {
                stopped[(size_t) m] = 1;
                --live;
            } else {
                ++frames_out[m];
            }
        }
    }
    if (e != cudaSuccess) {
        return fail_cuda(e, "decoder_run");
    }
    const uint32_t dev_status = b200q8_device_status(d->device, 1);
    if (dev_status != 0) {
        return fail((b200q8_status_t) dev_status, "decoder_run: the device recorded status %u", dev_status);
    }
    return B200Q8_OK;
}

void b200q8h_decoder_free(b200q8h_decoder * dec) {
    release(dec);
}

}  // extern "C"
