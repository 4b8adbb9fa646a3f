#pragma once
#include "nr_step.cuh"
namespace inb {
template <int GW, int SM>
static cudaError_t launch_gw(const InbStepArgs& a, cudaStream_t stream) {
  const int gpb = GW > 32 ? 1 : 128 / GW;
  dim3 grid((a.p.E + gpb - 1) / gpb), block(GW > 32 ? GW : 128);
  nr_step_kernel<GW, SM><<<grid, block, 0, stream>>>(a);
  return cudaGetLastError();
}

template <int SM>
static cudaError_t launch_sm(const InbStepArgs& a, cudaStream_t stream) {
  const int R = a.p.R;
  if (R <= 16) return launch_gw<16, SM>(a, stream);
  if (R <= 32) return launch_gw<32, SM>(a, stream);
  if (R <= 64) return launch_gw<64, SM>(a, stream);
  return launch_gw<128, SM>(a, stream);
}

}  // namespace inb
