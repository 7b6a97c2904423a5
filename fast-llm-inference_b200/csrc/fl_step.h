// One speculative step (or one stack pass) as a single persistent kernel:
// a list of phases executed in order by every CTA, separated by grid-wide
// barriers, with a producer warp streaming the weights of all GEMV phases
// through one TMA ring that never drains between phases.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fl_kernels.h"
#include "fl_state.h"

namespace fl {

enum PhaseKind : int {
    PH_GEMV = 0,          // INT8 GEMV over this CTA's rows (epilogue in `epi`)
    PH_ATTN = 1,          // split-K decode attention (units over CTAs)
    PH_DRAFT_PICK = 2,    // CTA 0: greedy draft token j = arg (launch_draft_pick)
    PH_VERIFY_PREP = 3,   // CTA 0: verify rows (launch_verify_prep)
    PH_ACCEPT = 4,        // CTA 0: acceptance (launch_accept)
    PH_CATCHUP_PREP = 5,  // CTA 0: next draft catch-up rows (launch_catchup_prep)
};

struct Phase {
    int kind;
    int epi;   // PH_GEMV: Epilogue
    int arg;   // PH_DRAFT_PICK: j
    GemvParams g;
    AttnParams a;
};

struct StepParams {
    const Phase* phases;
    int nphases;
    StepBuffers sb;        // control phases
    int K;                 // drafted tokens per step
    unsigned* bar;         // grid barrier: [0] arrivals, [1] generation
    const int* done;       // skip everything when set at kernel start
    int region_bytes;      // activation / attention scratch region
    int slot_bytes;        // ring slot size
    int S;                 // ring slots
};

// Shared-memory plan for a phase list (host): fills region / slot / S and
// returns false if some GEMV phase cannot be served.
bool step_plan(const Phase* host_phases, int n, StepParams& sp, size_t* smem_bytes);

cudaError_t launch_step(const StepParams& p, size_t smem_bytes, cudaStream_t s);

int step_grid();

}  // namespace fl
