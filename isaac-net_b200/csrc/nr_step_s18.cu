// Instantiation of the fused step kernel for up to 18 RBGs (one translation unit per RBG bound, so the
// variants compile in parallel).
#include "nr_step_launch.cuh"
namespace inb {
cudaError_t launch_step_s18(const InbStepArgs& a, cudaStream_t stream) { return launch_sm<18>(a, stream); }
}  // namespace inb
