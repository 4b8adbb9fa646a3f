// C entry point of the fused NR uplink step: argument checks and dispatch to the kernel variant of the group width
// (nr_step_g16.cu ... nr_step_g128.cu; the kernel itself is in nr_step.cuh).
#include "nr_common.cuh"
namespace inb {
cudaError_t launch_step_g16(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_step_g32(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_step_g64(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_step_g128(const InbStepArgs& a, cudaStream_t stream);
}  // namespace inb

extern "C" int inb_nr_step(const InbStepArgs* args, void* cuda_stream) {
  if (args == nullptr) return -1;
  const InbStepArgs& a = *args;
  const InbParams& p = a.p;
  if (p.E <= 0) return 0;
  if (p.R < 1 || p.R > 128 || p.S < 1 || p.S > INB_MAX_S || p.P < 1 || p.P > INB_MAX_P || p.F < 1 ||
      p.F > INB_MAX_F || p.M < 0 || p.M > INB_MAX_M || p.MCS < 1 || p.MCS > INB_MAX_MCS || p.K_rows < 0 ||
      p.K_rows > INB_MAX_ROWS || p.max_tx < 1 || p.mcs_max < 0 || p.mcs_max >= p.MCS)
    return -2;
  if (p.C_axis < 2 || p.G_axis < 2 || p.N < 1) return -3;
  if (a.pos == nullptr && a.pathgain_in == nullptr) return -4;
  if (a.pos != nullptr && a.pathgain_in == nullptr && (a.t.fk == nullptr || a.t.fphi == nullptr || a.t.gnb == nullptr))
    return -5;
  cudaStream_t s = (cudaStream_t)cuda_stream;
  cudaError_t err;
  if (p.R <= 16)
    err = inb::launch_step_g16(a, s);
  else if (p.R <= 32)
    err = inb::launch_step_g32(a, s);
  else if (p.R <= 64)
    err = inb::launch_step_g64(a, s);
  else
    err = inb::launch_step_g128(a, s);
  return err == cudaSuccess ? 0 : -100 - (int)err;
}

extern "C" int inb_abi_version(void) { return INB_ABI_VERSION; }
