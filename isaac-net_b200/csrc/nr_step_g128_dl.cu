// Instantiation of the fused step kernel's downlink instances for groups of 128 lanes (its own translation unit,
// compiled in parallel with the others).
#include "nr_step_launch.cuh"
namespace inb {
cudaError_t launch_step_g128_dl(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  return launch_gw_dl<128>(a, stream, rg);
}
}  // namespace inb
