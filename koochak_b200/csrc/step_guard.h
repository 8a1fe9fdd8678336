// Device-side skip of an optimizer step.
//
// The optimizer kernels (AdamW, the Muon prologue / epilogue / update-gather,
// the NorMuon second moments, the sharded Adam step, the hyperball
// projection) read an optional device flag before touching any persistent
// state and return at once when it is non-zero. The flag is the gradient
// gate's found-inf / non-finite value, so a step the gate rejects (GradScaler
// overflow, non-finite gradients under clipping) is skipped on the device
// without the host first reading the gate's result: the host enqueues the
// step, and checks the outcome afterwards (the optimizer then rolls back its
// host-side step counters). The Python layer sets the flag for the duration
// of one optimizer step.
#pragma once

namespace kb {

// The flag of the step being enqueued (null: no device-side skip).
const float* step_skip_ptr();
void set_step_skip_ptr(const float* p);

__device__ __forceinline__ bool step_skipped(const float* skip) { return skip != nullptr && *skip != 0.f; }

}  // namespace kb
