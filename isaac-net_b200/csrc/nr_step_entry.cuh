#pragma once
// Host-side pieces of the step entry points shared by nr_step.cu (inb_nr_step) and nr_step_noalloc.cu
// (inb_nr_step_noalloc).
#include "nr_common.cuh"

namespace inb {
// Argument checks of a step call (0 or the negative status of the entry points); *gain_need = float32 elements of
// the step's gain rows: (UL rows + 1) S E R with one cell, UL rows x C S E R with C > 1 cells.
int check_args(const InbStepArgs& a, long long* gain_need);
// The launches of a checked call on stream `s` (radio, fading, MAC, finish, as a.phases selects); 0 or -100 - error.
// mac_wait: an event (or NULL) the MAC launches wait for, after the fading launch.
int launch_all(const InbStepArgs& a, cudaStream_t s, cudaEvent_t mac_wait);
// Whether a call with these phases launches the fading or the MAC kernel, the two that use the gain rows.
inline bool uses_gain_rows(int phases) { return phases == 0 || (phases & 6) != 0; }
}  // namespace inb
