// Network observation packing of one control step (the Isaac-side consumer of the step dict), in one launch.
//
// isaac_net/isaac/net_module.py:340-374 (NetModule.step's post-processing on the engine's own radio) and
// isaac_net/isaac/obs.py:48-87 (NetObs.update): the freshness state last_cap = max(last_cap, newest), the age of
// information, delays in seconds, RSRP, the defaults of blocked / los, tag_delivered, the delay history (the delay of
// the robot's newest delivered message shifted in front) and the selected features, normalised, into x [E,R,dim].
//
// Mapping: FW lanes per robot (FW = 16 or 32), a lane per frame slot (two with F > 32), so the [E,R,F] step-dict
// arrays are read and delay_s / the per-frame feature columns written coalesced; the newest delivered message is a
// segmented (capture step, slot) arg-max over the lanes, ties to the lowest slot as torch.argmax; lane 0 writes the
// per-robot scalars and shifts the history.  Float arithmetic follows torch's CUDA rules op by op: a float tensor
// times a python scalar is a float32 multiply by the scalar rounded to float32, a division by a python scalar is a
// multiply by its float32 reciprocal (inv_* below, computed by the caller), int64 -> float32 rounds to nearest,
// clamp propagates NaN.
#include <cfloat>
#include <cmath>
#include <cstdint>

#include "isaac_net_b200.h"

namespace inb {

__device__ __forceinline__ float obs_fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float obs_clamp01(float x) { return isnan(x) ? x : fminf(fmaxf(x, 0.0f), 1.0f); }
// torch.nan_to_num(x, nan=0.0): NaN -> 0, +-inf -> the largest finite float32 of that sign
__device__ __forceinline__ float obs_nan0(float x) {
  if (isnan(x)) return 0.0f;
  if (isinf(x)) return x > 0.0f ? FLT_MAX : -FLT_MAX;
  return x;
}

template <int FW>
__global__ void __launch_bounds__(256) net_obs_kernel(const InbObsArgs A) {
  const long long gt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long rb = gt / FW;                // robot e R + r
  const int l = (int)(gt % FW);
  const long long NER = (long long)A.E * A.R;
  const bool live = rb < NER;                  // ghost robots still take part in the shuffles
  const int F = A.F;
  const long long rbs = live ? rb : 0;
  const long long e = rbs / A.R;
  const long long fb = rbs * F;
  const int lane = threadIdx.x & 31;
  const unsigned seg = FW >= 32 ? 0xFFFFFFFFu : (((1u << FW) - 1u) << (lane / FW * FW));
  // ---- frames of this lane: delay_s, the arg-max key, the per-frame feature values
  long long best = LLONG_MIN;   // (capture step or -2^62, ~slot) packed as a 128-bit compare below
  int best_f = 0x7FFFFFFF;
  bool any = false;
  float dd[2] = {0.0f, 0.0f};
  bool dl[2] = {false, false};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int f = l + j * FW;
    if (!live || f >= F) continue;
    const bool d = A.delivered[fb + f] != 0;
    const float ds = obs_fm(A.delay[fb + f], A.step_dt);
    if (A.delay_s) A.delay_s[fb + f] = ds;
    dd[j] = obs_nan0(ds);
    dl[j] = d;
    any = any || d;
    const long long key = d ? A.cap[fb + f] : -(1LL << 62);
    if (key > best || (key == best && f < best_f)) {
      best = key;
      best_f = f;
    }
  }
  // segmented arg-max over the robot's lanes: largest key, lowest slot on ties
#pragma unroll
  for (int o = FW / 2; o > 0; o >>= 1) {
    const long long ob = __shfl_xor_sync(0xFFFFFFFFu, best, o, FW);
    const int of = __shfl_xor_sync(0xFFFFFFFFu, best_f, o, FW);
    if (ob > best || (ob == best && of < best_f)) {
      best = ob;
      best_f = of;
    }
  }
  any = (__ballot_sync(0xFFFFFFFFu, any) & seg) != 0u;
  // the delay of the winning slot, from the lane that holds it
  const int owner = best_f % FW, jw = best_f / FW;
  const float mine = jw == 0 ? dd[0] : dd[1];
  const float dwin = __shfl_sync(0xFFFFFFFFu, mine, owner, FW);
  if (!live) return;

  float* const x = A.x + rbs * A.dim;
  // per-frame feature columns
  if (A.off_mask >= 0 || A.off_delay >= 0) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int f = l + j * FW;
      if (f >= F) continue;
      if (A.off_mask >= 0) x[A.off_mask + f] = dl[j] ? 1.0f : 0.0f;
      if (A.off_delay >= 0) x[A.off_delay + f] = dl[j] ? obs_clamp01(obs_fm(dd[j], A.inv_ts)) : 0.0f;
    }
  }
  // one-hot serving cell
  if (A.off_serv >= 0) {
    long long sv = A.serving[rbs];
    sv = sv < 0 ? 0 : (sv > A.G - 1 ? A.G - 1 : sv);
    for (int g = l; g < A.G; g += FW) x[A.off_serv + g] = g == sv ? 1.0f : 0.0f;
  }
  if (l != 0) return;
  // ---- per-robot scalars (lane 0)
  const long long newest = A.newest[rbs];
  long long lc = A.last_cap[rbs];
  lc = newest > lc ? newest : lc;
  A.last_cap[rbs] = lc;
  if (A.last_cap_out) A.last_cap_out[rbs] = lc;
  const float aoi = obs_fm(__ll2float_rn(A.t[e] + 1 - lc), A.step_dt);
  if (A.aoi_s) A.aoi_s[rbs] = aoi;
  const float sinr = A.sinr_db[rbs];
  const float rsrp = __fadd_rn(sinr, A.noise_db);
  if (A.rsrp_dbm) A.rsrp_dbm[rbs] = rsrp;
  const bool blk = A.blocked != nullptr ? A.blocked[rbs] != 0 : false;
  const bool los = A.los != nullptr ? A.los[rbs] != 0 : !blk;
  if (A.blocked_out) A.blocked_out[rbs] = blk ? 1 : 0;
  if (A.los_out) A.los_out[rbs] = los ? 1 : 0;
  if (A.delivered_any) A.delivered_any[rbs] = newest >= 0 ? 1 : 0;
  if (A.tag_delivered != nullptr && A.cur_tag != nullptr && rbs % A.R == 0)
    A.tag_delivered[e] = (A.det_env[e] != 0 && A.cur_tag[e] >= 0) ? 1 : 0;
  // delay history: the newest delivered message's delay shifted in front when the robot had a delivery
  if (A.K > 0 && A.hist != nullptr) {
    float* const h = A.hist + rbs * A.K;
    if (any) {
      for (int k = A.K - 1; k > 0; --k) h[k] = h[k - 1];
      h[0] = obs_clamp01(obs_fm(dwin, A.inv_ts));
    }
    if (A.off_hist >= 0)
      for (int k = 0; k < A.K; ++k) x[A.off_hist + k] = h[k];
  }
  if (A.off_aoi >= 0) x[A.off_aoi] = obs_clamp01(obs_fm(aoi, A.inv_ts));
  if (A.off_qlen >= 0) x[A.off_qlen] = obs_fm(__ll2float_rn(A.queue_len[rbs]), A.inv_F);
  if (A.off_qbytes >= 0) x[A.off_qbytes] = obs_fm(A.queue_bytes[rbs], A.inv_qbytes);
  if (A.off_sinr >= 0) x[A.off_sinr] = obs_fm(sinr, A.inv_db);
  if (A.off_rsrp >= 0) x[A.off_rsrp] = obs_fm(__fsub_rn(rsrp, A.noise_db), A.inv_db);
  if (A.off_last >= 0) x[A.off_last] = newest >= 0 ? 1.0f : 0.0f;
  if (A.off_blocked >= 0) x[A.off_blocked] = blk ? 1.0f : 0.0f;
  if (A.off_los >= 0) x[A.off_los] = los ? 1.0f : 0.0f;
}

}  // namespace inb

extern "C" int inb_net_obs(const InbObsArgs* args, void* cuda_stream) {
  if (args == nullptr) return -1;
  const InbObsArgs& a = *args;
  if (a.E < 0 || a.R < 1 || a.F < 1 || a.F > INB_MAX_F || a.G < 1 || a.K < 0 || a.dim < 0) return -2;
  if (a.E == 0) return 0;
  if (a.newest == nullptr || a.t == nullptr || a.delivered == nullptr || a.cap == nullptr || a.delay == nullptr ||
      a.last_cap == nullptr || (a.dim > 0 && a.x == nullptr) || (a.off_serv >= 0 && a.serving == nullptr) ||
      (a.off_qlen >= 0 && a.queue_len == nullptr) || (a.off_qbytes >= 0 && a.queue_bytes == nullptr) ||
      a.sinr_db == nullptr || (a.K > 0 && a.hist == nullptr) || (a.tag_delivered != nullptr && a.det_env == nullptr))
    return -3;
  const int offs[] = {a.off_mask, a.off_delay, a.off_aoi, a.off_qlen, a.off_qbytes, a.off_sinr, a.off_rsrp,
                      a.off_serv, a.off_last, a.off_hist, a.off_blocked, a.off_los};
  const int wid[] = {a.F, a.F, 1, 1, 1, 1, 1, a.G, 1, a.K, 1, 1};
  for (int i = 0; i < 12; ++i)
    if (offs[i] >= 0 && offs[i] + wid[i] > a.dim) return -4;
  const long long n = (long long)a.E * a.R;
  const cudaStream_t s = (cudaStream_t)cuda_stream;
  if (a.F <= 16) {
    const long long th = n * 16;
    inb::net_obs_kernel<16><<<(unsigned)((th + 255) / 256), 256, 0, s>>>(a);
  } else {
    const long long th = n * 32;
    inb::net_obs_kernel<32><<<(unsigned)((th + 255) / 256), 256, 0, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -100;
}
