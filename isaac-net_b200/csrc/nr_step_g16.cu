// Instantiation of the fused step kernel for groups of 16 lanes (one translation unit per width, compiled in
// parallel).
#include "nr_step_launch.cuh"
namespace inb {
cudaError_t launch_step_g16(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  return launch_gw<16, false>(a, stream, rg);
}
}  // namespace inb
