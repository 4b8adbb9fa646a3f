// C entry points of the NR uplink step: argument checks, then the launches on the caller's stream: the radio (radio
// map / blockage, nr_radio.cu; only with InbStepArgs.rm.on), the fading (nr_fading.cu), the MAC kernel variant of the
// group width (nr_step_g16.cu ... nr_step_g128.cu; the kernel is in nr_step.cuh) and the end-of-step finish
// (nr_finish.cu).
#include "nr_step_entry.cuh"
namespace inb {
cudaError_t launch_step_g16(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g32(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g64(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g128(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g16_bsr(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g32_bsr(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g64_bsr(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g128_bsr(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g16_dl(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g32_dl(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g64_dl(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_step_g128_dl(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_fading(const InbStepArgs& a, cudaStream_t stream, const Range& rg);
cudaError_t launch_radio(const InbStepArgs& a, cudaStream_t stream);
cudaError_t launch_finish(const InbStepArgs& a, cudaStream_t stream, const Range& rg);

int check_args(const InbStepArgs& a, long long* gain_need) {
  const InbParams& p = a.p;
  if (p.R < 1 || p.R > 128 || p.S < 1 || p.S > INB_MAX_S || p.P < 1 || p.P > INB_MAX_P || p.F < 1 ||
      p.F > INB_MAX_F || p.M < 0 || p.M > INB_MAX_M || p.MCS < 1 || p.MCS > INB_MAX_MCS || p.K_rows < 0 ||
      p.K_rows > INB_MAX_ROWS || p.max_tx < 1 || p.mcs_max < 0 || p.mcs_max >= p.MCS)
    return -2;
  if (p.C_axis < 2 || p.G_axis < 2 || p.N < 1 || p.Kf < 0 || p.Kf > INB_MAX_KF) return -3;
  if (p.C > 1 && (p.C > INB_MAX_C || a.s.serv == nullptr || a.s.a3_cand == nullptr || a.s.a3_cnt == nullptr ||
                  a.s.ho_end == nullptr || a.s.n_ho == nullptr || a.s.pending == nullptr || a.s.ni_ul == nullptr ||
                  a.o.serving_cell == nullptr))
    return -7;
  if (p.bsr_on && (a.s.bsr_est == nullptr || a.s.bsr_rep_v == nullptr || a.s.bsr_rep_g == nullptr ||
                   a.s.bsr_hid == nullptr || a.s.bsr_hid_until == nullptr || a.s.bsr_enq_seen == nullptr ||
                   a.s.bsr_boot == nullptr || a.s.bsr_armed == nullptr || p.sr_boot_slots < 0 || p.bsr_delay < 0 ||
                   p.rlc_tail_slots < 1))
    return -12;   // the BSR pipeline's state (InbState.bsr_*) or its timing is missing
  if (a.pos == nullptr && a.pathgain_in == nullptr) return -4;
  const InbRadio& rm = a.rm;
  const bool radio = rm.on && a.pathgain_in == nullptr;   // the radio launch runs (poses through the radio)
  const bool formula = !(radio && rm.map_on);
  if (a.pathgain_in == nullptr && formula && (a.t.fk == nullptr || a.t.fphi == nullptr || a.t.gnb == nullptr))
    return -5;
  if (radio) {
    if (rm.pg == nullptr || (rm.map_on && (rm.map == nullptr || rm.H < 2 || rm.W < 2)) || a.t.gnb == nullptr)
      return -11;
    if (rm.blockage && (rm.blk == nullptr || rm.t == nullptr || rm.table == nullptr || rm.bk == nullptr ||
                        rm.bphi == nullptr || rm.xk == nullptr || rm.yk == nullptr || rm.vel == nullptr ||
                        rm.Kb < 1 || rm.Kb > INB_MAX_KF || rm.n_table < INB_CDF_STRIDE ||
                        rm.n_table % INB_CDF_STRIDE != 0 || rm.n_table > 1024 * INB_CDF_STRIDE))
      return -11;
  }
  if (a.o.blocked != nullptr && !(radio && rm.blockage)) return -11;   // blocked bits exist only after the launch
  int n_ul = 0;
  for (int k = 0; k < p.K_rows; ++k) n_ul += p.rows[k][1] > 0 ? 1 : 0;
  if (p.dl_on) {   // the downlink: one cell, its own args (state, outputs, arrivals, counters), DL gain rows
    const InbStepArgs* d = a.dl;
    if (p.C > 1 || d == nullptr || p.n_ul_rows != n_ul || p.n_dl_rows < 0 || d->p.E != p.E || d->p.R != p.R ||
        d->p.S != p.S || d->p.P < 1 || d->p.P > INB_MAX_P || d->p.F < 1 || d->p.F > INB_MAX_F || d->p.M < 0 ||
        d->p.M > INB_MAX_M || d->p.K_rows != p.K_rows || d->p.mcs_max < 0 || d->p.mcs_max >= d->p.MCS ||
        d->p.bsr_on || d->p.tdma || d->p.amc_prev || d->p.phr_cap)
      return -13;
    for (int k = 0; k < p.K_rows; ++k)
      if (p.rows_dl[k][3] >= p.n_dl_rows || d->p.rows_dl[k][3] != p.rows_dl[k][3]) return -13;
  }
  *gain_need = p.C > 1 ? (long long)n_ul * p.C * p.S * p.E * p.R
                       : (long long)(n_ul + 1 + (p.dl_on ? p.n_dl_rows : 0)) * p.S * p.E * p.R;
  return 0;
}

namespace {
// The DL and UL MAC launches and the finish launches of the envs of rg
int launch_mac(const InbStepArgs& a, cudaStream_t s, const Range& rg) {
  const InbParams& p = a.p;
  cudaError_t err = cudaSuccess;
  if (p.dl_on) {   // the downlink MAC and finish first: the uplink MAC advances the step's RNG counter
    InbStepArgs d = *a.dl;
    d.gain = a.gain;
    d.gain_cap = a.gain_cap;
    d.pathgain_in = a.pathgain_in != nullptr ? a.pathgain_in : d.pathgain_in;
    d.dl = nullptr;
    if (p.R <= 16)
      err = launch_step_g16_dl(d, s, rg);
    else if (p.R <= 32)
      err = launch_step_g32_dl(d, s, rg);
    else if (p.R <= 64)
      err = launch_step_g64_dl(d, s, rg);
    else
      err = launch_step_g128_dl(d, s, rg);
    if (err == cudaSuccess) err = launch_finish(d, s, rg);
    if (err != cudaSuccess) return -100 - (int)err;
  }
  const bool b = p.bsr_on != 0;
  if (p.R <= 16)
    err = b ? launch_step_g16_bsr(a, s, rg) : launch_step_g16(a, s, rg);
  else if (p.R <= 32)
    err = b ? launch_step_g32_bsr(a, s, rg) : launch_step_g32(a, s, rg);
  else if (p.R <= 64)
    err = b ? launch_step_g64_bsr(a, s, rg) : launch_step_g64(a, s, rg);
  else
    err = b ? launch_step_g128_bsr(a, s, rg) : launch_step_g128(a, s, rg);
  if (err == cudaSuccess) err = launch_finish(a, s, rg);
  return err == cudaSuccess ? 0 : -100 - (int)err;
}
}  // namespace

int launch_all(const InbStepArgs& args, cudaStream_t s, cudaEvent_t mac_wait) {
  InbStepArgs a = args;
  const InbParams& p = a.p;
  cudaError_t err = cudaSuccess;
  const bool all = a.phases == 0;
  const bool radio = all || (a.phases & 1), fading = all || (a.phases & 2), mac = all || (a.phases & 4);
  if (a.rm.on && a.pathgain_in == nullptr) {   // path gains of this step's poses: the MAC reads them
    if (radio) {
      err = launch_radio(a, s);
      if (err != cudaSuccess) return -100 - (int)err;
    }
    a.pathgain_in = a.rm.pg;
  }
  Range whole;
  whole.e1 = p.E;
  if (fading) {
    err = launch_fading(a, s, whole);
    if (err != cudaSuccess) return -100 - (int)err;
  }
  if (!mac) return 0;
  if (mac_wait != nullptr && cudaStreamWaitEvent(s, mac_wait, 0) != cudaSuccess) return -100 - (int)cudaGetLastError();
  return launch_mac(a, s, whole);
}

}  // namespace inb

extern "C" int inb_nr_step(const InbStepArgs* args, void* cuda_stream) {
  if (args == nullptr) return -1;
  const InbStepArgs& a = *args;
  if (a.p.E <= 0) return 0;
  long long need = 0;
  const int rc = inb::check_args(a, &need);
  if (rc != 0) return rc;
  if (a.gain == nullptr || a.gain_cap < need) return -6;
  return inb::launch_all(a, (cudaStream_t)cuda_stream, nullptr);
}

extern "C" int inb_nr_step_after(const InbStepArgs* args, void* cuda_stream, void* mac_wait_event) {
  if (args == nullptr) return -1;
  const InbStepArgs& a = *args;
  if (a.p.E <= 0) return 0;
  long long need = 0;
  const int rc = inb::check_args(a, &need);
  if (rc != 0) return rc;
  if (a.gain == nullptr || a.gain_cap < need) return -6;
  return inb::launch_all(a, (cudaStream_t)cuda_stream, (cudaEvent_t)mac_wait_event);
}

namespace inb {
__global__ void store2_kernel(int64_t* dst, int64_t v0, int64_t v1) {
  dst[0] = v0;
  dst[1] = v1;
}
}  // namespace inb

extern "C" int inb_store2(int64_t* dst, int64_t v0, int64_t v1, void* cuda_stream) {
  if (dst == nullptr) return -1;
  inb::store2_kernel<<<1, 1, 0, (cudaStream_t)cuda_stream>>>(dst, v0, v1);
  return cudaGetLastError() == cudaSuccess ? 0 : -100;
}

extern "C" int inb_abi_version(void) { return INB_ABI_VERSION; }
