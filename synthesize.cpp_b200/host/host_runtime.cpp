// host_runtime.cpp -- host-side helpers of the B200 Q8_0 path (C++17, no CUDA).
//
//  * the seeded N(0,1) stream used for every synthetic input: the algorithm
//    of synth::NormalRandomStream (src/random-stream.cpp:10-48 in the
//    reference): a splitmix64 state advanced by 0x9e3779b97f4a7c15 per draw,
//    the Marsaglia polar method in double precision, the spare value kept for
//    the next call;
//  * a multi-tensor fill that runs independent seeded streams on host
//    threads (each tensor is one stream, so threading does not change values);
//  * the reference's default CPU thread rule, min(n/2, n-1)
//    (src/cpu-parallelism.cpp:93-99), for reporting the CPU baseline.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

class SeededNormal {
  public:
    explicit SeededNormal(uint64_t seed) : state_(seed) {}

    float next() {
        if (have_spare_) {
            have_spare_ = false;
            return spare_;
        }
        double a = 0.0, b = 0.0, r = 0.0;
        do {
            a = 2.0 * uniform() - 1.0;
            b = 2.0 * uniform() - 1.0;
            r = a * a + b * b;
        } while (r >= 1.0 || r == 0.0);
        const double f = std::sqrt(-2.0 * std::log(r) / r);
        spare_         = static_cast<float>(b * f);
        have_spare_    = true;
        return static_cast<float>(a * f);
    }

  private:
    uint64_t bits() {
        state_ += UINT64_C(0x9e3779b97f4a7c15);
        uint64_t z = state_;
        z          = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
        z          = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
        return z ^ (z >> 31);
    }

    double uniform() { return (static_cast<double>(bits() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

    uint64_t state_;
    float    spare_      = 0.0f;
    bool     have_spare_ = false;
};

}  // namespace

extern "C" {

// out[i] = scale * normal_i (scale == 1 gives the plain stream).
void b200q8h_normal_fill(uint64_t seed, float scale, float * out, size_t n) {
    SeededNormal s(seed);
    if (scale == 1.0f) {
        for (size_t i = 0; i < n; ++i) {
            out[i] = s.next();
        }
    } else {
        for (size_t i = 0; i < n; ++i) {
            out[i] = scale * s.next();
        }
    }
}

// Fills `count` tensors, tensor j from its own stream seeds[j], on up to
// `threads` host threads (<= 0: hardware concurrency).
void b200q8h_normal_fill_many(int count, const uint64_t * seeds, const float * scales, float * const * outs,
                              const size_t * ns, int threads) {
    if (count <= 0) {
        return;
    }
    int t = threads > 0 ? threads : static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
    t     = std::min(t, count);
    std::atomic<int>         next{ 0 };
    std::vector<std::thread> pool;
    auto                     work = [&]() {
        for (int j = next.fetch_add(1); j < count; j = next.fetch_add(1)) {
            b200q8h_normal_fill(seeds[j], scales[j], outs[j], ns[j]);
        }
    };
    for (int i = 1; i < t; ++i) {
        pool.emplace_back(work);
    }
    work();
    for (auto & th : pool) {
        th.join();
    }
}

int b200q8h_default_threads(int available) {
    if (available <= 2) {
        return 1;
    }
    return std::min(available / 2, available - 1);
}

}  // extern "C"
