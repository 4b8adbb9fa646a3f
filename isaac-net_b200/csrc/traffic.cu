// Traffic arrivals of one control step on the device: periodic, video and bursty models.
//
// inb_traffic_step reproduces TrafficGen.step (isaac_net/core/traffic.py:408-430) with _Stream._step
// (traffic.py:301-365) for every robot in one thread, including the random stream: the reference draws each uniform
// as a float64 torch.rand([E, R]) call on the engine's CUDA torch.Generator, i.e. curand Philox4x32-10 keyed by the
// generator seed, in torch's grid-stride layout (ATen DistributionTemplates.h: `stride` = 256 x blocks threads,
// element li served by thread li % stride on its (li / stride) / 2-th curand_uniform2_double call, component
// (li / stride) % 2, at the call's Philox offset; the value 1.0 is mapped to 0.0).  Every call advances the offset by
// `inc`, and the number of calls per step does not depend on the data, so draw d of step n sits at offset
// off0 + (n ndraws + d) inc.  A thread computes a draw only where its value is used (Philox is counter based, so
// skipping draws changes nothing), and a bursty model's event loop stops at its first iteration that changes no
// state (every later iteration would see the same state and also change nothing).
//
// Float64 arithmetic follows the reference op by op with round-to-nearest intrinsics: exponential draws are
// (-log1p(-u)) * mean, slots are floor(max(t, 0) * (1 / slot_ms)) (torch's CUDA division by a python scalar).
//
// With InbTrafficArgs.counter the uniforms come instead from the opt-in counter-keyed stream (CounterU below): the
// same models and the same draw indices d, each uniform a function of (seed key, global env id, episode, the robot's
// step count, d, robot), so the arrivals of an env do not depend on which engine (shard) steps it.
#include <cmath>
#include <cstdint>
#include <curand_kernel.h>

#include "isaac_net_b200.h"
#include "nr_common.cuh"

namespace inb {

constexpr uint32_t CH_TRAFFIC = 0x54u;   // counter-RNG channel of the counter-keyed traffic stream's step draws

struct Philox {
  unsigned long long seed, base;  // base: offset of draw 0 of this step
  long long inc;
  unsigned long long sub;         // the torch thread (curand subsequence) that serves this element
  unsigned long long call_off;    // 4 x the index of that thread's curand_uniform2_double call
  int comp;                       // which double of the pair

  __device__ double u(long long d) const {
    curandStatePhilox4_32_10_t st;
    curand_init(seed, sub, base + (unsigned long long)(d * inc) + call_off, &st);
    const double2 v = curand_uniform2_double(&st);
    const double x = comp ? v.y : v.x;
    return x == 1.0 ? 0.0 : x;
  }
  // _Source._expo: -log1p(-u) * mean_ms
  __device__ double expo(long long d, double mean) const { return __dmul_rn(-log1p(-u(d)), mean); }

  // the draws of element li (robot r) in its n-th step
  __device__ static Philox make(const InbTrafficArgs& A, long long li, long long n, int r) {
    Philox p;
    p.seed = A.seed;
    p.base = A.off0 + (unsigned long long)(n * A.ndraws * A.inc);
    p.inc = A.inc;
    p.sub = (unsigned long long)(li % A.stride);
    const long long q = li / A.stride;
    p.call_off = (unsigned long long)(q >> 1) * 4ull;
    p.comp = (int)(q & 1);
    return p;
  }
};

// The counter-keyed stream: uniform d = 53 bits from the element hashes 2r, 2r + 1 of stream d under the key
// (s0, env id, episode, CH_TRAFFIC, step count); exact in float64, in [0, 1)
struct CounterU {
  uint32_t kenv, r2;
  __device__ double u(long long d) const {
    const uint32_t base = key_stream(kenv, (uint32_t)d);
    const uint32_t h0 = elem(base, r2), h1 = elem(base, r2 + 1u);
    return (double)(h0 >> 5) * 67108864.0 * 0x1p-53 + (double)(h1 >> 6) * 0x1p-53;
  }
  __device__ double expo(long long d, double mean) const { return __dmul_rn(-log1p(-u(d)), mean); }
  __device__ static CounterU make(const InbTrafficArgs& A, long long li, long long n, int r) {
    const long long e = li / A.R;
    CounterU c;
    c.kenv = key_env(A.s0, A.env_id[e], A.episode[e], CH_TRAFFIC, n);
    c.r2 = 2u * (uint32_t)r;
    return c;
  }
};

template <class Rng>
__global__ void __launch_bounds__(256) traffic_step_kernel(const InbTrafficArgs A) {
  const long long li = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)A.E * A.R;
  if (li >= total) return;
  const int r = (int)(li % A.R);
  const int M = A.M;
  const double T = A.step_ms;

  const long long n = A.calls[li];
  A.calls[li] = n + 1;
  const Rng rng = Rng::make(A, li, n, r);

  // columns of this robot before sorting: emission time, validity, bytes, model
  double t_c[INB_MAX_M];
  float b_c[INB_MAX_M];
  uint8_t v_c[INB_MAX_M];
  int8_t s_c[INB_MAX_M];

  long long d0 = 0;  // first draw of the current model in this step
  for (int k = 0; k < A.n_src; ++k) {
    const InbTrafficSource& S = A.src[k];
    const bool msk = S.mask[r] != 0;
    if (S.kind == 0 || S.kind == 1) {
      double nom = S.nom[li], nxt = S.nxt[li];
      long long cnt = S.cnt[li];
      for (int w = 0; w < S.width; ++w) {
        const bool hit = (nxt < T) && msk;
        double size = S.size;
        if (S.kind == 1 && S.gop_n > 0) size = (cnt % S.gop_n == 0) ? S.gop_i : S.gop_p;
        const int c = S.col + w;
        v_c[c] = hit; t_c[c] = nxt; b_c[c] = (float)size; s_c[c] = (int8_t)k;
        cnt += hit ? 1 : 0;
        if (hit) {
          nom = __dadd_rn(nom, S.period);
          nxt = __dadd_rn(nom, __dmul_rn(rng.u(d0 + w), S.jitter));
        }
      }
      if ((nxt < T) && msk) atomicAdd((unsigned long long*)S.deferred, 1ull);
      S.nom[li] = __dsub_rn(nom, T);
      S.nxt[li] = __dsub_rn(nxt, T);
      S.cnt[li] = cnt;
      d0 += S.width;
    } else {
      const int nb = S.nb;
      const int per = S.off_ms > 0.0 ? 4 : 3;  // draws per loop iteration: burst iat, ON, [OFF], toggle iat
      bool on = S.on[li] != 0;
      double t_tog = S.t_tog[li], t_bur = S.t_bur[li];
      double times[INB_MAX_M];
      for (int b = 0; b < nb; ++b) times[b] = INFINITY;
      int cnt = 0;
      for (int it = 0; it < S.loops; ++it) {
        const double t_b = on ? t_bur : INFINITY;
        const bool due = msk && on && (t_b <= t_tog) && (t_b < T);
        const bool burst = due && cnt < nb;
        const bool blocked = due && cnt >= nb;
        const bool tog = msk && !burst && !blocked && (t_tog < T) && (t_tog < t_b);
        if (!burst && !tog) break;
        const long long d = d0 + (long long)it * per;
        if (burst) {
          times[cnt] = t_b;
          cnt += 1;
          t_bur = __dadd_rn(t_bur, rng.expo(d, S.iat));
        }
        if (tog) {
          const bool now_on = !on;
          double dt;
          if (now_on) dt = rng.expo(d + 1, S.on_ms);
          else dt = per == 4 ? rng.expo(d + 2, S.off_ms) : INFINITY;
          const double new_tog = __dadd_rn(t_tog, dt);
          if (now_on) t_bur = __dadd_rn(t_tog, rng.expo(d + per - 1, S.iat));
          t_tog = new_tog;
          on = now_on;
        }
      }
      const double t_b = on ? t_bur : INFINITY;
      if (msk && fmin(t_b, t_tog) < T) atomicAdd((unsigned long long*)S.deferred, 1ull);
      S.on[li] = on;
      S.t_bur[li] = __dsub_rn(t_bur, T);
      S.t_tog[li] = __dsub_rn(t_tog, T);
      for (int b = 0; b < nb; ++b)
        for (int j = 0; j < S.burst; ++j) {
          const int c = S.col + b * S.burst + j;
          v_c[c] = isfinite(times[b]); t_c[c] = times[b]; b_c[c] = (float)S.size; s_c[c] = (int8_t)k;
        }
      d0 += (long long)S.loops * per;
    }
  }

  // sort by key (valid ? slot : N) * M + column (distinct keys: the order is unique), insertion sort
  int key[INB_MAX_M], slot[INB_MAX_M];
  for (int c = 0; c < M; ++c) {
    const double t = v_c[c] ? t_c[c] : 0.0;
    long long sl = (long long)floor(__dmul_rn(fmax(t, 0.0), A.inv_slot_ms));
    sl = sl < 0 ? 0 : (sl > A.N - 1 ? A.N - 1 : sl);
    slot[c] = (int)sl;
    key[c] = (v_c[c] ? (int)sl : A.N) * M + c;
  }
  int order[INB_MAX_M];
  for (int c = 0; c < M; ++c) {
    int j = c;
    while (j > 0 && key[order[j - 1]] > key[c]) { order[j] = order[j - 1]; --j; }
    order[j] = c;
  }
  for (int m = 0; m < M; ++m) {
    const int c = order[m];
    const InbTrafficSource& S = A.src[s_c[c]];
    const long long at = li * M + m;
    A.valid[at] = v_c[c];
    A.det[at] = (uint8_t)(S.det != 0);
    A.nbytes[at] = b_c[c];
    A.slot[at] = slot[c];
    A.tag[at] = S.tag;
    A.prio[at] = S.prio;
    A.dline[at] = S.dline;
  }
}

}  // namespace inb

extern "C" int inb_traffic_step(const InbTrafficArgs* args, void* stream) {
  if (args == nullptr) return -1;
  const InbTrafficArgs& A = *args;
  if (A.E <= 0 || A.R <= 0 || A.M <= 0 || A.M > INB_MAX_M || A.n_src <= 0 || A.n_src > INB_MAX_SRC || A.N <= 0)
    return -2;
  if (A.calls == nullptr) return -3;
  if (A.counter ? (A.env_id == nullptr || A.episode == nullptr) : (A.stride <= 0 || A.inc <= 0)) return -3;
  int cols = 0;
  for (int k = 0; k < A.n_src; ++k) {
    const InbTrafficSource& S = A.src[k];
    if (S.kind < 0 || S.kind > 2 || S.mask == nullptr || S.deferred == nullptr || S.col != cols) return -4;
    if (S.kind == 2 && (S.nb * S.burst != S.width || S.nb > INB_MAX_M || S.loops < 0)) return -5;
    cols += S.width;
  }
  if (cols != A.M) return -6;
  const long long total = (long long)A.E * A.R;
  const int block = 256;
  const long long grid = (total + block - 1) / block;
  if (A.counter)
    inb::traffic_step_kernel<inb::CounterU><<<(unsigned)grid, block, 0, (cudaStream_t)stream>>>(A);
  else
    inb::traffic_step_kernel<inb::Philox><<<(unsigned)grid, block, 0, (cudaStream_t)stream>>>(A);
  return cudaGetLastError() == cudaSuccess ? 0 : -100;
}
