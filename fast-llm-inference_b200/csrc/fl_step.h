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
    unsigned* bar;         // [0..1] 64-bit barrier counter (zero at launch), [2] error word
    const int* done;       // skip everything when set at kernel start
    int region_bytes;      // activation / attention scratch region
    int slot_bytes;        // ring slot size
    int S;                 // ring slots
    // Optional phase trace (nullptr = off), 6 words per phase, %globaltimer ns:
    // [6i] CTA 0 start of phase i, [6i+1] CTA 0 end of its work in phase i,
    // [6i+2] latest end over all CTAs (atomicMax; timestamps only grow, so
    // after a decode every word holds the last launch's value); GEMV phases,
    // CTA 0: [6i+3] activation prologue done, [6i+4] ns warp 0 waited for
    // full ring stages, [6i+5] first stage ready.
    unsigned long long* trace;
    // Stage trace of phase `trace_phase` (-1 = off), CTA 0, after the phase
    // words: 64 stages x 8 words = warp 0 stage ready, warp 0 stage done,
    // warp 7 stage ready, warp 7 stage done, producer starts waiting for the
    // slot, producer issues the stage, 2 unused.
    int trace_phase;
};

// Shared-memory plan for a phase list (host): fills region / slot / S and
// returns false if some GEMV phase cannot be served.
bool step_plan(const Phase* host_phases, int n, StepParams& sp, size_t* smem_bytes);

// Raises the kernel's dynamic shared-memory limit (call outside capture).
cudaError_t step_set_smem(size_t smem_bytes);

// Cooperative launch, grid = step_grid() CTAs of one per SM.
cudaError_t launch_step(const StepParams& p, size_t smem_bytes, cudaStream_t s);

int step_grid();

}  // namespace fl
