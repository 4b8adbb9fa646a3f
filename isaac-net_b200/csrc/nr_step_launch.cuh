#pragma once
// Launch of the fused step kernel for one group width GW (robots per env rounded up to a power of two).
#include "nr_step.cuh"
namespace inb {
template <int GW, int NCT, int SV>
cudaError_t launch_gw_mc(const InbStepArgs& a, cudaStream_t stream) {
  constexpr int NT = GW > 32 ? GW : 128;
  const int gpb = GW > 32 ? 1 : 128 / GW;
  const int vecs = a.ul_ref_in != nullptr ? 3 : 2;
  const size_t smem = (size_t)vecs * a.p.S * (NT + 1) * sizeof(float);
  static size_t configured = 0;   // dynamic shared memory above 48 KB needs an opt-in, once per size
  if (smem > 48 * 1024 && smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(nr_step_kernel<GW, NCT, SV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  dim3 grid((a.p.E + gpb - 1) / gpb), block(NT);
  nr_step_kernel<GW, NCT, SV><<<grid, block, smem, stream>>>(a);
  return cudaGetLastError();
}

template <int GW, int SV>
cudaError_t launch_gw_sv(const InbStepArgs& a, cudaStream_t stream) {
  if (a.p.C == 2) return launch_gw_mc<GW, 2, SV>(a, stream);
  if (a.p.C == 3) return launch_gw_mc<GW, 3, SV>(a, stream);
  return launch_gw_mc<GW, 1, SV>(a, stream);
}

template <int GW>
cudaError_t launch_gw(const InbStepArgs& a, cudaStream_t stream) {
  if (a.p.sched == 2) return launch_gw_sv<GW, 1>(a, stream);   // round robin
  if (a.p.pf_rbg) return launch_gw_sv<GW, 2>(a, stream);       // PF with the per-RBG metric
  return launch_gw_sv<GW, 0>(a, stream);
}
}  // namespace inb
