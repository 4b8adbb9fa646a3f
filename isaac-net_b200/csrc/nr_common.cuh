// Shared device helpers of the B200 NR engine kernels.
//
// Numerics: every floating-point operation of the MAC path is written with an explicit round-to-nearest intrinsic
// (__fmul_rn, __fadd_rn, ...), so the compiler never contracts a multiply and an add into one FMA.  The reference
// evaluates each tensor operation separately, rounding after every op; the kernels round exactly there too.
// Transcendentals call CUDA's own functions (logf, log10f, expf, powf, cosf, sqrtf), the ones torch's CUDA kernels
// call for the same tensor ops.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "isaac_net_b200.h"

namespace inb {

constexpr uint32_t M32 = 0xFFFFFFFFu;
constexpr uint32_t C1 = 0x21F0AAADu, C2 = 0x735A2D97u, GOLD = 0x9E3779B9u;
constexpr uint32_t CH_STEP = 2u, CH_RESET = 3u;
constexpr int SITE_FADING = 1, SITE_BLER_UL = 2, SITE_BLER_DL = 3, SITE_H0 = 4, SITE_KPHI = 6;
constexpr long long BIGI = 1LL << 62;

__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double dm(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double da(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsb(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double ddv(double a, double b) { return __ddiv_rn(a, b); }

// torch.clamp semantics: NaN propagates
__device__ __forceinline__ float clampf_t(float x, float lo, float hi) {
  return isnan(x) ? x : fminf(fmaxf(x, lo), hi);
}
__device__ __forceinline__ float clamp_min_t(float x, float lo) { return isnan(x) ? x : fmaxf(x, lo); }

// ---------------------------------------------------------------- counter RNG (lowbias32 key chain)
// isaac_net/core/proto/rng.py:42-60, 164-185: mix32 = lowbias32, salt(v) = mix32(v) + GOLD, key chain over
// (seed, env, episode, channel, counter, stream), element hash = two rounds over base + i * GOLD.
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= C1;
  x ^= x >> 15;
  x *= C2;
  x ^= x >> 15;
  return x;
}
__device__ __forceinline__ uint32_t salt(uint32_t v) { return mix32(v) + GOLD; }
__device__ __forceinline__ uint32_t key_env(uint32_t s0, int64_t env, int64_t ep, uint32_t channel, int64_t ctr) {
  uint32_t h = mix32(s0 ^ salt((uint32_t)env));
  h = mix32(h ^ salt((uint32_t)ep));
  h = mix32(h ^ salt(channel));
  return mix32(h ^ salt((uint32_t)ctr));
}
__device__ __forceinline__ uint32_t key_stream(uint32_t kenv, uint32_t stream) { return mix32(kenv ^ salt(stream)); }
__device__ __forceinline__ uint32_t elem(uint32_t base, uint32_t i) { return mix32(mix32(base + i * GOLD) ^ base); }

constexpr float INV24 = 5.9604644775390625e-08f;  // 2^-24, exact

__device__ __forceinline__ float uniform_at(uint32_t base, uint32_t i) {
  return fm((float)(elem(base, i) >> 8), INV24);
}
// Box-Muller cosine branch on hash elements 2i, 2i+1: sqrt(-2 log u1) cos(2 pi u2), u1 in (0, 1]
__device__ __forceinline__ float normal_at(uint32_t base, uint32_t i, float two_pi) {
  uint32_t h1 = elem(base, 2u * i), h2 = elem(base, 2u * i + 1u);
  float u1 = fm((float)((h1 >> 8) + 1u), INV24);
  float u2 = fm((float)(h2 >> 8), INV24);
  return fm(sqrtf(fm(-2.0f, logf(u1))), cosf(fm(two_pi, u2)));
}

// ---------------------------------------------------------------- large-scale channel formulas
// Received power (dBm) of one link at 2-D distance d2 (floored at 1 m) with the shadowing value `field` (dB, the
// plane-wave sum times its amplitude): TR 38.901 UMi / UMa LOS path loss (isaac_net/core/channels/tr38901.py:148-170)
// plus sigma_SF times the unit field (radio_model 0 / 1), or log-distance path loss minus the field (radio_model 2,
// isaac_net/core/radio.py:265-273), each in the reference's op order.
__device__ __forceinline__ float formula_rx(const InbParams& p, float d2, float field) {
  if (p.radio_model <= 1) {
    const float d3 = sqrtf(fa(fm(d2, d2), p.hh2));
    const float lg = log10f(d3);
    const float pl = (d2 <= p.dbp) ? fa(fa(p.pl_a, fm(p.pl_n1, lg)), p.fc_term)
                                   : fs(fa(fa(p.pl_a, fm(40.0f, lg)), p.fc_term), p.pl_b_term);
    return fa(p.ue_tx, -fa(pl, fm(p.sigma_sf, field)));
  }
  const float pl = fa(p.pl_const, fm(p.pl_10n, log10f(d2)));
  return fs(fs(p.ue_tx, pl), field);
}

// Phase k . x of one plane wave at (x, y), rounded as the reference's CPU einsum rounds it: one fused multiply-add
// over the x product (its BLAS path) or two rounded products and a rounded sum (its plain loop for small matrices)
__device__ __forceinline__ float wave_phase(float x, float y, float kx, float ky, bool fused) {
  return fused ? __fmaf_rn(y, ky, fm(x, kx)) : fa(fm(x, kx), fm(y, ky));
}

// The envs [e0, e1) of one launch of a step (the entry points launch the whole batch)
struct Range {
  int e0 = 0, e1 = 0;
};

// an output pointer of InbOutputs: absolute, or a byte offset from the block address `base` (InbStepArgs.o_base)
template <typename T>
__device__ __forceinline__ T* out_ptr(T* p, long long base) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + base);
}

}  // namespace inb
