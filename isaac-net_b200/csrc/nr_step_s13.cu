// Instantiation of the fused step kernel for up to 13 RBGs (one translation unit per RBG bound, so the
// variants compile in parallel).
#include "nr_step_launch.cuh"
namespace inb {
cudaError_t launch_step_s13(const InbStepArgs& a, cudaStream_t stream) { return launch_sm<13>(a, stream); }
}  // namespace inb
