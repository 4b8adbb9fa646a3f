// Instantiation of the fused step kernel for groups of 16 lanes with the SR / BSR grant pipeline (its own translation
// unit, compiled in parallel with the others).
#include "nr_step_launch.cuh"
namespace inb {
cudaError_t launch_step_g16_bsr(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  return launch_gw<16, true>(a, stream, rg);
}
}  // namespace inb
