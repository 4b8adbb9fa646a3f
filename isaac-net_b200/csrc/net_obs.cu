// Network observation packing of one control step (the Isaac-side consumer of the step dict), in one launch.
//
// isaac_net/isaac/net_module.py:340-374 (NetModule.step's post-processing on the engine's own radio) and
// isaac_net/isaac/obs.py:48-87 (NetObs.update): the freshness state last_cap = max(last_cap, newest), the age of
// information, delays in seconds, RSRP, the defaults of blocked / los, tag_delivered, the delay history (the delay of
// the robot's newest delivered message shifted in front) and the selected features, normalised, into x [E,R,dim].
//
// Mapping: a block of 256 threads packs RB consecutive robots (RB = 256 / 128 / 64 / 32, the most whose x rows fit
// a 96 KB shared-memory tile).  (1) Frame stage: FW lanes per robot (FW = 16 or 32), a lane per frame slot (two with
// F > 32), so the [E,R,F] step-dict arrays are read and delay_s written coalesced; the newest delivered message is a
// segmented (capture step, slot) arg-max over the lanes, ties to the lowest slot as torch.argmax; the per-frame
// feature columns go to the tile.  (2) Robot stage: a thread per robot reads the per-robot fields coalesced, updates
// last_cap and the delay history and writes the scalar columns to the tile.  (3) The tile, RB whole rows of x, is
// stored with 16-byte writes.  Float arithmetic follows torch's CUDA rules op by op: a float tensor
// times a python scalar is a float32 multiply by the scalar rounded to float32, a division by a python scalar is a
// multiply by its float32 reciprocal (inv_* below, computed by the caller), int64 -> float32 rounds to nearest,
// clamp propagates NaN.
#include <atomic>
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

constexpr int OBS_THREADS = 256;
constexpr int OBS_TILE_BYTES = 96 * 1024;

template <int FW>
__global__ void __launch_bounds__(OBS_THREADS) net_obs_kernel(const InbObsArgs A, int RB) {
  extern __shared__ float tile[];                   // [RB][dim] rows of x
  __shared__ float s_dwin[OBS_THREADS];             // delay of the robot's newest delivered message
  __shared__ unsigned char s_any[OBS_THREADS];      // the robot had a delivery this step
  const long long NER = (long long)A.E * A.R;
  const long long rb0 = (long long)blockIdx.x * RB;
  const int nrb = (int)(NER - rb0 < RB ? NER - rb0 : RB);
  const int F = A.F, dim = A.dim;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int RPW = 32 / FW;                      // robots per warp and pass
  const unsigned seg = FW >= 32 ? 0xFFFFFFFFu : (((1u << FW) - 1u) << (lane / FW * FW));
  const int l = lane % FW;
  // ---- (1) frame stage: each warp takes NPASS groups of RPW robots at a time, all their loads issued before the
  // first reduction (the loads of a group are independent of the others': latency overlaps instead of adding up)
  constexpr int NPASS = 4, STRIDE = (OBS_THREADS / 32) * RPW;
  for (int base = warp * RPW; base < nrb; base += STRIDE * NPASS) {   // warp-uniform trip count
    bool dl[NPASS][2];
    float dd[NPASS][2];
    long long ck[NPASS][2];
#pragma unroll
    for (int q = 0; q < NPASS; ++q) {
      const int rl = base + q * STRIDE + lane / FW;
      const long long fb = (rb0 + (rl < nrb ? rl : 0)) * F;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int f = l + j * FW;
        const bool in = rl < nrb && f < F;
        dl[q][j] = in && A.delivered[fb + f] != 0;
        dd[q][j] = in ? obs_fm(A.delay[fb + f], A.step_dt) : 0.0f;
        ck[q][j] = in ? A.cap[fb + f] : 0;
      }
    }
#pragma unroll
    for (int q = 0; q < NPASS; ++q) {
      const int rl = base + q * STRIDE + lane / FW;
      const bool live = rl < nrb;
      const long long fb = (rb0 + (live ? rl : 0)) * F;
      long long best = LLONG_MIN;
      int best_f = 0x7FFFFFFF;
      bool any = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int f = l + j * FW;
        if (!live || f >= F) continue;
        if (A.delay_s) A.delay_s[fb + f] = dd[q][j];
        dd[q][j] = obs_nan0(dd[q][j]);
        any = any || dl[q][j];
        const long long key = dl[q][j] ? ck[q][j] : -(1LL << 62);
        if (key > best || (key == best && f < best_f)) {
          best = key;
          best_f = f;
        }
      }
#pragma unroll
      for (int o = FW / 2; o > 0; o >>= 1) {   // segmented arg-max: largest key, lowest slot on ties
        const long long ob = __shfl_xor_sync(0xFFFFFFFFu, best, o, FW);
        const int of = __shfl_xor_sync(0xFFFFFFFFu, best_f, o, FW);
        if (ob > best || (ob == best && of < best_f)) {
          best = ob;
          best_f = of;
        }
      }
      any = (__ballot_sync(0xFFFFFFFFu, any) & seg) != 0u;
      const int owner = best_f % FW, jw = best_f / FW;   // the delay of the winning slot, from its lane
      const float mine = jw == 0 ? dd[q][0] : dd[q][1];
      const float dwin = __shfl_sync(0xFFFFFFFFu, mine, owner, FW);
      if (!live) continue;
      if (l == 0) {
        s_dwin[rl] = dwin;
        s_any[rl] = any ? 1 : 0;
      }
      float* const row = tile + (size_t)rl * dim;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int f = l + j * FW;
        if (f >= F) continue;
        if (A.off_mask >= 0) row[A.off_mask + f] = dl[q][j] ? 1.0f : 0.0f;
        if (A.off_delay >= 0) row[A.off_delay + f] = dl[q][j] ? obs_clamp01(obs_fm(dd[q][j], A.inv_ts)) : 0.0f;
      }
    }
  }
  __syncthreads();
  // ---- (2) robot stage
  for (int rl = tid; rl < nrb; rl += OBS_THREADS) {
    const long long rb = rb0 + rl;
    const long long e = rb / A.R;
    float* const row = tile + (size_t)rl * dim;
    const long long newest = A.newest[rb];
    long long lc = A.last_cap[rb];
    lc = newest > lc ? newest : lc;
    A.last_cap[rb] = lc;
    if (A.last_cap_out) A.last_cap_out[rb] = lc;
    const float aoi = obs_fm(__ll2float_rn(A.t[e] + 1 - lc), A.step_dt);
    if (A.aoi_s) A.aoi_s[rb] = aoi;
    const float sinr = A.sinr_db[rb];
    const float rsrp = __fadd_rn(sinr, A.noise_db);
    if (A.rsrp_dbm) A.rsrp_dbm[rb] = rsrp;
    const bool blk = A.blocked != nullptr ? A.blocked[rb] != 0 : false;
    const bool los = A.los != nullptr ? A.los[rb] != 0 : !blk;
    if (A.blocked_out) A.blocked_out[rb] = blk ? 1 : 0;
    if (A.los_out) A.los_out[rb] = los ? 1 : 0;
    if (A.delivered_any) A.delivered_any[rb] = newest >= 0 ? 1 : 0;
    if (A.tag_delivered != nullptr && A.cur_tag != nullptr && rb % A.R == 0)
      A.tag_delivered[e] = (A.det_env[e] != 0 && A.cur_tag[e] >= 0) ? 1 : 0;
    if (A.K > 0 && A.hist != nullptr) {   // the newest delivered message's delay shifted in front
      float* const h = A.hist + rb * A.K;
      if (s_any[rl]) {
        for (int k = A.K - 1; k > 0; --k) h[k] = h[k - 1];
        h[0] = obs_clamp01(obs_fm(s_dwin[rl], A.inv_ts));
      }
      if (A.off_hist >= 0)
        for (int k = 0; k < A.K; ++k) row[A.off_hist + k] = h[k];
    }
    if (A.off_serv >= 0) {
      long long sv = A.serving[rb];
      sv = sv < 0 ? 0 : (sv > A.G - 1 ? A.G - 1 : sv);
      for (int g = 0; g < A.G; ++g) row[A.off_serv + g] = g == sv ? 1.0f : 0.0f;
    }
    if (A.off_aoi >= 0) row[A.off_aoi] = obs_clamp01(obs_fm(aoi, A.inv_ts));
    if (A.off_qlen >= 0) row[A.off_qlen] = obs_fm(__ll2float_rn(A.queue_len[rb]), A.inv_F);
    if (A.off_qbytes >= 0) row[A.off_qbytes] = obs_fm(A.queue_bytes[rb], A.inv_qbytes);
    if (A.off_sinr >= 0) row[A.off_sinr] = obs_fm(sinr, A.inv_db);
    if (A.off_rsrp >= 0) row[A.off_rsrp] = obs_fm(__fsub_rn(rsrp, A.noise_db), A.inv_db);
    if (A.off_last >= 0) row[A.off_last] = newest >= 0 ? 1.0f : 0.0f;
    if (A.off_blocked >= 0) row[A.off_blocked] = blk ? 1.0f : 0.0f;
    if (A.off_los >= 0) row[A.off_los] = los ? 1.0f : 0.0f;
  }
  __syncthreads();
  // ---- (3) the tile's rows of x, 16-byte stores where the addresses allow
  if (dim == 0) return;
  float* const xg = A.x + rb0 * dim;
  const int n = nrb * dim;
  if ((reinterpret_cast<uintptr_t>(xg) & 15u) == 0u) {
    const int n4 = n / 4;
    for (int i = tid; i < n4; i += OBS_THREADS)
      reinterpret_cast<float4*>(xg)[i] = reinterpret_cast<const float4*>(tile)[i];
    for (int i = n4 * 4 + tid; i < n; i += OBS_THREADS) xg[i] = tile[i];
  } else {
    for (int i = tid; i < n; i += OBS_THREADS) xg[i] = tile[i];
  }
}

}  // namespace inb

extern "C" int inb_net_obs(const InbObsArgs* args, void* cuda_stream) {
  if (args == nullptr) return -1;
  const InbObsArgs& a = *args;
  // at most 64 frame slots: two per lane of a robot's 32 lanes
  if (a.E < 0 || a.R < 1 || a.F < 1 || a.F > 64 || a.G < 1 || a.K < 0 || a.dim < 0) return -2;
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
  int RB = inb::OBS_THREADS;   // robots per block: the most whose x rows fit the shared-memory tile
  while (RB > 32 && (size_t)RB * a.dim * sizeof(float) > (size_t)inb::OBS_TILE_BYTES) RB /= 2;
  const size_t smem = (size_t)RB * a.dim * sizeof(float);
  if (smem > (size_t)inb::OBS_TILE_BYTES) return -2;   // x rows wider than 768 features
  const long long n = (long long)a.E * a.R;
  const unsigned grid = (unsigned)((n + RB - 1) / RB);
  const cudaStream_t s = (cudaStream_t)cuda_stream;
  // dynamic shared memory above 48 KB needs an opt-in, once per device
  static std::atomic<bool> opted[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -100;
  if (!opted[dev].load()) {
    if (cudaFuncSetAttribute(inb::net_obs_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             inb::OBS_TILE_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(inb::net_obs_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             inb::OBS_TILE_BYTES) != cudaSuccess)
      return -100;
    opted[dev].store(true);
  }
  if (a.F <= 16)
    inb::net_obs_kernel<16><<<grid, inb::OBS_THREADS, smem, s>>>(a, RB);
  else
    inb::net_obs_kernel<32><<<grid, inb::OBS_THREADS, smem, s>>>(a, RB);
  return cudaGetLastError() == cudaSuccess ? 0 : -100;
}
