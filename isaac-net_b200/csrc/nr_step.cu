// C entry point of the NR uplink step: argument checks, then three launches on the caller's stream: the fading
// (nr_fading.cu), the MAC kernel variant of the group width (nr_step_g16.cu ... nr_step_g128.cu; the kernel is in
// nr_step.cuh) and the end-of-step finish (nr_finish.cu).
#include "nr_common.cuh"
namespace inb {
cudaError_t launch_step_g16(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_step_g32(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_step_g64(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_step_g128(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_fading(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_finish(const InbStepArgs& a, cudaStream_t stream);
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
  int n_ul = 0;
  for (int k = 0; k < p.K_rows; ++k) n_ul += p.rows[k][1] > 0 ? 1 : 0;
  if (a.gain == nullptr || a.gain_cap < (long long)(n_ul + 1) * p.S * p.E * p.R) return -6;
  cudaStream_t s = (cudaStream_t)cuda_stream;
  cudaError_t err = inb::launch_fading(a, s);
  if (err != cudaSuccess) return -100 - (int)err;
  if (p.R <= 16)
    err = inb::launch_step_g16(a, s);
  else if (p.R <= 32)
    err = inb::launch_step_g32(a, s);
  else if (p.R <= 64)
    err = inb::launch_step_g64(a, s);
  else
    err = inb::launch_step_g128(a, s);
  if (err == cudaSuccess) err = inb::launch_finish(a, s);
  return err == cudaSuccess ? 0 : -100 - (int)err;
}

extern "C" int inb_abi_version(void) { return INB_ABI_VERSION; }
