// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI face over the two self-contained reference sources that the
// harness uses, compiled from where they lie in the reference tree
// (src/random-stream.cpp, src/cpu-parallelism.cpp) by oracle/Makefile's
// `ref` target into oracle/_ref/.  It pins the oracle's restatements of the
// seeded normal stream (src/random-stream.cpp:10-48) and of the default CPU
// thread policy (src/cpu-parallelism.cpp:93-99) against the reference itself.
#include "cpu-parallelism.h"
#include "random-stream.h"

#include <cstddef>
#include <cstdint>

extern "C" {

void ref_normal_fill(uint64_t seed, float * out, size_t count) {
    synth::NormalRandomStream stream(seed);
    stream.fill(out, count);
}

void ref_uniform_fill(uint64_t seed, float * out, size_t count) {
    synth::NormalRandomStream stream(seed);
    stream.fill_uniform(out, count);
}

int ref_default_synthesis_threads(void) {
    return synth::default_synthesis_threads();
}

int ref_available_cpu_parallelism(void) {
    return synth::available_cpu_parallelism();
}
}
