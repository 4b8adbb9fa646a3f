// Instantiation of the fused step kernel for up to 32 RBGs (one translation unit per RBG bound, so the
// variants compile in parallel).
#include "nr_step_launch.cuh"
namespace inb {
cudaError_t launch_step_s32(const InbStepArgs& a, cudaStream_t stream) { return launch_sm<32>(a, stream); }
}  // namespace inb
