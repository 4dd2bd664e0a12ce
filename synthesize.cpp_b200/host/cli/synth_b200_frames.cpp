// synth_b200_frames -- decodes frames of a Qwen3-TTS Q8_MIXED package on one
// B200 from the command line: the package is loaded with b200q8h_decoder_load
// and the frame loop runs through b200q8h_decoder_run (include/b200q8_host.h),
// the device counterparts of the reference's synth_model_load and
// run_synthesis frame loop (src/synthesize.cpp:575-682,
// src/arch/qwen3-tts/model.cpp:1310-1489).
//
//   synth_b200_frames PACKAGE --streams M --frames F --out CODES
//                     (--text-ids FILE | --text-rows FILE)
//                     [--prev FILE] [--replay FILE] [--start-pos P]
//                     [--stop-code C] [--device D] [--n-ctx N]
//
// Input files are raw little-endian arrays: text ids int32 [F][M], text rows
// float32 [F][M][hidden], prev int32 [M][groups], replay int32 [F][M][groups].
// CODES receives int32 [F][M][groups].  One JSON line on stdout reports the
// frames each stream ran and the wall-clock rate of the loop.
#include "b200q8_host.h"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace {

template <typename T>
bool read_file(const std::string & path, std::vector<T> & out, size_t count) {
    FILE * f = std::fopen(path.c_str(), "rb");
    if (f == nullptr) {
        std::fprintf(stderr, "cannot open %s\n", path.c_str());
        return false;
    }
    out.resize(count);
    const size_t got = std::fread(out.data(), sizeof(T), count, f);
    std::fclose(f);
    if (got != count) {
        std::fprintf(stderr, "%s: expected %zu values, read %zu\n", path.c_str(), count, got);
        return false;
    }
    return true;
}

int usage() {
    std::fprintf(stderr,
                 "usage: synth_b200_frames PACKAGE --streams M --frames F --out CODES "
                 "(--text-ids FILE | --text-rows FILE) [--prev FILE] [--replay FILE] [--start-pos P] "
                 "[--stop-code C] [--device D] [--n-ctx N]\n");
    return 2;
}

}  // namespace

int main(int argc, char ** argv) {
    if (argc < 2) {
        return usage();
    }
    std::string package = argv[1], out_path, ids_path, rows_path, prev_path, replay_path;
    long long   M = 0, F = 0, start_pos = 0, stop_code = -1, device = 0, n_ctx = 0;
    for (int i = 2; i < argc; ++i) {
        const std::string a = argv[i];
        if (i + 1 >= argc) {
            return usage();
        }
        const char * v = argv[++i];
        if (a == "--streams") M = std::atoll(v);
        else if (a == "--frames") F = std::atoll(v);
        else if (a == "--out") out_path = v;
        else if (a == "--text-ids") ids_path = v;
        else if (a == "--text-rows") rows_path = v;
        else if (a == "--prev") prev_path = v;
        else if (a == "--replay") replay_path = v;
        else if (a == "--start-pos") start_pos = std::atoll(v);
        else if (a == "--stop-code") stop_code = std::atoll(v);
        else if (a == "--device") device = std::atoll(v);
        else if (a == "--n-ctx") n_ctx = std::atoll(v);
        else return usage();
    }
    if (M < 1 || F < 1 || out_path.empty() || ids_path.empty() == rows_path.empty()) {
        return usage();
    }
    char                   msg[512];
    b200q8h_decoder_params prm = {};
    prm.device                 = (int32_t) device;
    prm.max_streams            = M;
    prm.n_ctx                  = n_ctx > 0 ? n_ctx : start_pos + F;
    prm.mode                   = B200Q8_QUANT_REF;
    b200q8h_decoder * dec      = nullptr;
    if (b200q8h_decoder_load(package.c_str(), &prm, &dec) != B200Q8_OK) {
        b200q8h_last_error(msg, sizeof(msg));
        std::fprintf(stderr, "load failed: %s\n", msg);
        return 1;
    }
    b200q8h_decoder_info info = {};
    b200q8h_decoder_info_get(dec, &info);
    const size_t         G = (size_t) info.groups;
    std::vector<int32_t> ids, prev, replay;
    std::vector<float>   rows;
    bool                 ok = true;
    if (!ids_path.empty()) ok = read_file(ids_path, ids, (size_t) (F * M));
    if (ok && !rows_path.empty()) ok = read_file(rows_path, rows, (size_t) (F * M) * (size_t) info.hidden);
    if (ok && !prev_path.empty()) ok = read_file(prev_path, prev, (size_t) M * G);
    if (ok && !replay_path.empty()) ok = read_file(replay_path, replay, (size_t) (F * M) * G);
    if (!ok) {
        b200q8h_decoder_free(dec);
        return 1;
    }
    b200q8h_run_params run = {};
    run.M                  = M;
    run.n_frames           = F;
    run.text_ids           = ids.empty() ? nullptr : ids.data();
    run.text_rows          = rows.empty() ? nullptr : rows.data();
    run.first_prev         = prev.empty() ? nullptr : prev.data();
    run.start_pos          = (int32_t) start_pos;
    run.replay             = replay.empty() ? nullptr : replay.data();
    run.stop_code          = (int32_t) stop_code;
    std::vector<int32_t> codes((size_t) (F * M) * G, -1);
    std::vector<int64_t> frames((size_t) M, 0);
    const auto           t0 = std::chrono::steady_clock::now();
    const b200q8_status_t st = b200q8h_decoder_run(dec, &run, codes.data(), frames.data());
    const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (st != B200Q8_OK) {
        b200q8h_last_error(msg, sizeof(msg));
        std::fprintf(stderr, "run failed: %s\n", msg);
        b200q8h_decoder_free(dec);
        return 1;
    }
    FILE * f = std::fopen(out_path.c_str(), "wb");
    if (f == nullptr || std::fwrite(codes.data(), sizeof(int32_t), codes.size(), f) != codes.size()) {
        std::fprintf(stderr, "cannot write %s\n", out_path.c_str());
        if (f != nullptr) std::fclose(f);
        b200q8h_decoder_free(dec);
        return 1;
    }
    std::fclose(f);
    long long total = 0;
    std::printf("{\"streams\": %lld, \"groups\": %zu, \"frames\": [", M, G);
    for (long long m = 0; m < M; ++m) {
        total += frames[(size_t) m];
        std::printf("%s%lld", m ? ", " : "", (long long) frames[(size_t) m]);
    }
    std::printf("], \"seconds\": %.6f, \"stream_frames_per_s\": %.3f}\n", secs, secs > 0 ? total / secs : 0.0);
    b200q8h_decoder_free(dec);
    return 0;
}
