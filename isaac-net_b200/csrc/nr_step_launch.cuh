#pragma once
#include <atomic>
// Launch of the fused step kernel for one group width GW (robots per env rounded up to a power of two).
#include "nr_step.cuh"
namespace inb {
template <int GW, int NCT, int SV, bool BSR, bool DL = false>
cudaError_t launch_gw_mc(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  constexpr int NT = GW > 32 ? GW : 128;
  const int gpb = GW > 32 ? 1 : 128 / GW;
  const int vecs = a.ul_ref_in != nullptr ? 3 : 2;
  const size_t smem = (size_t)vecs * a.p.S * (NT + 1) * sizeof(float);
  // dynamic shared memory above 48 KB needs an opt-in, which holds per device: remembered per device and size
  static std::atomic<size_t> configured[64];
  if (smem > 48 * 1024) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || smem > configured[dev].load(std::memory_order_acquire)) {
      e = cudaFuncSetAttribute(nr_step_kernel<GW, NCT, SV, BSR, DL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) {   // raise the remembered size (several threads may race here; the max wins)
        size_t cur = configured[dev].load(std::memory_order_relaxed);
        while (smem > cur && !configured[dev].compare_exchange_weak(cur, smem, std::memory_order_acq_rel)) {
        }
      }
    }
  }
  const int n = rg.e1 - rg.e0;
  if (n <= 0) return cudaSuccess;
  dim3 grid((n + gpb - 1) / gpb), block(NT);
  nr_step_kernel<GW, NCT, SV, BSR, DL><<<grid, block, smem, stream>>>(a, rg.e0, rg.e1);
  return cudaGetLastError();
}

template <int GW, int SV, bool BSR>
cudaError_t launch_gw_sv(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  if (a.p.C == 2) return launch_gw_mc<GW, 2, SV, BSR>(a, stream, rg);
  if (a.p.C == 3) return launch_gw_mc<GW, 3, SV, BSR>(a, stream, rg);
  return launch_gw_mc<GW, 1, SV, BSR>(a, stream, rg);
}

// the instances of one group width, with (BSR = true) or without the SR / BSR grant pipeline
template <int GW, bool BSR>
cudaError_t launch_gw(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  if (a.p.sched == 2) return launch_gw_sv<GW, 1, BSR>(a, stream, rg);   // round robin
  if (a.p.pf_rbg) return launch_gw_sv<GW, 2, BSR>(a, stream, rg);       // PF with the per-RBG metric
  return launch_gw_sv<GW, 0, BSR>(a, stream, rg);
}

// the downlink instances of one group width (one cell, no BSR pipeline)
template <int GW>
cudaError_t launch_gw_dl(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  if (a.p.sched == 2) return launch_gw_mc<GW, 1, 1, false, true>(a, stream, rg);
  if (a.p.pf_rbg) return launch_gw_mc<GW, 1, 2, false, true>(a, stream, rg);
  return launch_gw_mc<GW, 1, 0, false, true>(a, stream, rg);
}
}  // namespace inb
