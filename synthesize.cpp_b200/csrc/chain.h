// chain.h -- step-chain internals shared with the frame runner (internal).
#pragma once

#include "../../include/b200q8.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200q8 {

// One step's arguments: b200q8_step_args with its defaults resolved (table,
// h_out and the output buffers point at the chain's own storage where the
// caller passed NULL; hidden_out == nullptr means no output stage).
struct StepIO {
    int64_t         M          = 0;
    const int32_t * ids        = nullptr;
    const uint8_t * table      = nullptr;
    int64_t         table_rows = 0;
    const float *   x_in       = nullptr;
    const int32_t * pos        = nullptr;
    const int32_t * slots      = nullptr;
    float *         h_out      = nullptr;
    float *         hidden_out = nullptr;
    float *         logits     = nullptr;
    int             head       = 0;
};

inline bool same_io(const StepIO & a, const StepIO & b) {
    return a.M == b.M && a.ids == b.ids && a.table == b.table && a.table_rows == b.table_rows && a.x_in == b.x_in &&
           a.pos == b.pos && a.slots == b.slots && a.h_out == b.h_out && a.hidden_out == b.hidden_out &&
           a.logits == b.logits && a.head == b.head;
}

struct ChainInfo {
    int             device;
    int             sms;
    int64_t         hidden;
    int64_t         max_m;
    bool            attn;
    int64_t         n_ctx;
    int64_t         n_slots;
    int             n_heads;  // 0: no output desc
    int64_t         vocab;
    const uint8_t * table;
    int64_t         table_rows;
};

ChainInfo chain_info(const b200q8_chain * c);

// The chain's activation quantizer (B200Q8_QUANT_*).
int chain_mode(const b200q8_chain * c);

// Checks a against the chain and fills io (sets the error message on failure).
b200q8_status_t chain_resolve(b200q8_chain * c, const b200q8_step_args & a, StepIO & io);

// Enqueues the step's kernels on st (which may be capturing).
cudaError_t chain_enqueue(b200q8_chain * c, cudaStream_t st, const StepIO & io);

// Whether the chain puts its persistent single-launch step into captured
// graphs; disable = true turns that off (the per-op form is captured then).
bool chain_persistent_in_graph(b200q8_chain * c, bool disable);

}  // namespace b200q8
