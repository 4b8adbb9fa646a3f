// Fused NR uplink MAC of one control step (sm_100a): traffic enqueue and arrival gate, large-scale radio, and the K
// scheduled slots (SR, candidate selection, retransmission admission, RBG-by-RBG PF / RR allocation, EESM link
// adaptation, HARQ decode and update, OLLA, PF averages, RLC in-order delivery).  The AR(1) fading of the step runs
// before it (nr_fading.cu) and the end-of-step finish (delivery / timeout / drop masks, outputs, FIFO compaction)
// after it (nr_finish.cu), as separate launches on the same stream.
//
// Thread mapping: one thread per robot; the R robots of an env form a group of GW lanes (GW = next power of two >= R,
// at least 16).  GW <= 32: 128 / GW envs per 128-thread block, group collectives are segmented warp shuffles.
// GW > 32: one env per block of GW threads, collectives go through shared memory.  Every lane of a group runs the
// same control flow (ghost lanes r >= R and ghost envs e >= E carry neutral values and store nothing), because the
// schedule of a control step is the same for every env.  A branch that holds a collective is taken on a warp-uniform
// condition, so full-mask shuffles are always reached by all 32 lanes at the same call site.
//
// The AR(1) fading of the step runs before this kernel (nr_fading.cu): the CSI and the fading gain of the u-th UL
// row are rows u and u + 1 of the gain buffer [n_ul + 1][E R][S].  Per-RBG work (rates, link adaptation, the decode
// SINR) is only needed for the robots that want or use RBGs in a slot: a warp serves a few such robots one at a time
// with a lane per RBG (or per MCS), and several at once with a lane per robot; their per-RBG vectors (rate, PF metric,
// link-adaptation SINR, the optional per-RBG SNR input) live in shared memory, laid out [vector][RBG][thread] with an
// odd row stride, so a warp reading a row or a column is conflict-free.  Counters accumulate in shared memory, one block of words per env.
//
// Semantics follow isaac-net v0.2.0 (file:line in the comments); reductions over the RBG axis are left-to-right sums
// (the oracle's "seq" mode), ties in every argmax resolve to the lowest robot / process index (torch.max / argmin),
// and the retransmission ranking is a stable descending sort.
#pragma once
#include <cfloat>
#include <cmath>
#include <cstdint>

#include "nr_bsr.cuh"
#include "nr_common.cuh"

namespace inb {

struct SmemGroup {
  unsigned long long red[2][4];   // per-warp partial maxima (GW up to 128: 4 warps), double-buffered
  unsigned long long redc[2][INB_MAX_C][4];   // per-cell partial (max, lowest lane) pairs (GW > 32)
  uint32_t redf[2][INB_MAX_C][4];             // per-cell partial flags (GW > 32)
  float rkey[128];
  int32_t rnsb[128];
  int32_t rserv[128];
  uint32_t rmask[4];              // per-warp ballot of the robots with a retransmission (GW > 32)
  int32_t bc[2][INB_MAX_C];       // per-cell value broadcast by one lane (GW > 32), double-buffered
};

// float -> order-preserving u32 (non-NaN inputs)
__device__ __forceinline__ uint32_t fkey(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

template <int GW>
struct Grp {
  // max over the group's lanes (lane = robot index)
  __device__ static unsigned long long max_u64(unsigned long long x, SmemGroup* sm, int& par) {
    constexpr int W = GW < 32 ? GW : 32;
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) {
      unsigned long long v = __shfl_xor_sync(0xFFFFFFFFu, x, o, W);
      x = v > x ? v : x;
    }
    if constexpr (GW > 32) {
      int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
      if (lane == 0) sm->red[par][wid] = x;
      __syncthreads();
      unsigned long long m = sm->red[par][0];
#pragma unroll
      for (int w = 1; w < GW / 32; ++w) m = sm->red[par][w] > m ? sm->red[par][w] : m;
      par ^= 1;
      return m;
    } else {
      return x;
    }
  }
  __device__ static unsigned gmask() {   // this lane's group within its warp (GW <= 32)
    if constexpr (GW >= 32) {
      return 0xFFFFFFFFu;
    } else {
      return ((1u << GW) - 1u) << ((threadIdx.x & 31) / GW * GW);
    }
  }
  __device__ static bool any(bool v, SmemGroup* sm, int& par) {
    if constexpr (GW > 32) {
      return max_u64(v ? 1ull : 0ull, sm, par) != 0ull;
    } else {
      return (__ballot_sync(0xFFFFFFFFu, v) & gmask()) != 0u;
    }
  }
  // the group's maximum of `key` (mx) and the lowest lane (robot index) holding it
  __device__ static int argmax_u32(uint32_t key, uint32_t& mx, SmemGroup* sm, int& par) {
    const int lane = threadIdx.x & 31;
    if constexpr (GW <= 32) {
      uint32_t m = 0u;
      if constexpr (GW == 32) {
        m = __reduce_max_sync(0xFFFFFFFFu, key);
      } else {
#pragma unroll
        for (int gq = 0; gq < 32 / GW; ++gq) {   // one full-warp reduction per group; each lane keeps its own
          const uint32_t v = __reduce_max_sync(0xFFFFFFFFu, lane / GW == gq ? key : 0u);
          if (lane / GW == gq) m = v;
        }
      }
      const unsigned win = __ballot_sync(0xFFFFFFFFu, key == m) & gmask();
      mx = m;
      return __ffs(win) - 1 - (lane / GW * GW) % 32;
    } else {
      const int wid = threadIdx.x >> 5;
      const uint32_t m = __reduce_max_sync(0xFFFFFFFFu, key);
      const int wl = __ffs(__ballot_sync(0xFFFFFFFFu, key == m)) - 1;
      if (lane == 0) sm->red[par][wid] = ((unsigned long long)m << 32) | (unsigned)(255 - (wid * 32 + wl));
      __syncthreads();
      unsigned long long b = sm->red[par][0];
#pragma unroll
      for (int w = 1; w < GW / 32; ++w) b = sm->red[par][w] > b ? sm->red[par][w] : b;
      par ^= 1;
      mx = (uint32_t)(b >> 32);
      return 255 - (int)(b & 0xFFu);
    }
  }
  // Per cell: the maximum of `key` over the group's lanes of cell c (c < C <= NC) with the lowest lane holding it
  // (mx, return value), and whether a lane of cell c has `flag` (anyf); the lanes of cell c must have keys > 0.
  // As argmax_u32 / any of each cell, but with GW > 32 one block barrier serves every cell and both results.
  // anyc (optional, GW > 32): whether any cell of the block has a lane with a non-negative key (a candidate of the
  // allocation rounds), read from the same shared-memory partials
  template <int NC>
  __device__ static int argmax_cell(uint32_t key, bool flag, int c, int C, uint32_t& mx, bool& anyf, SmemGroup* sm,
                                    int& par, bool* anyc = nullptr) {
    if constexpr (GW <= 32) {
      int w = 0;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        uint32_t m;
        const int wi = argmax_u32(c == cc ? key : 0u, m, sm, par);
        const bool a = any(flag && c == cc, sm, par);
        if (cc == c) { w = wi; mx = m; anyf = a; }
      }
      return w;
    } else {
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        const uint32_t kk = c == cc ? key : 0u;
        const uint32_t m = __reduce_max_sync(0xFFFFFFFFu, kk);
        const unsigned bl = __ballot_sync(0xFFFFFFFFu, c == cc && kk == m);
        const unsigned fl = __ballot_sync(0xFFFFFFFFu, flag && c == cc);
        if (lane == 0) {
          sm->redc[par][cc][wid] = bl ? (((unsigned long long)m << 32) | (unsigned)(255 - (wid * 32 + __ffs(bl) - 1)))
                                      : 0ull;
          sm->redf[par][cc][wid] = fl != 0u ? 1u : 0u;
        }
      }
      __syncthreads();
      unsigned long long b = sm->redc[par][c][0];
      uint32_t f = sm->redf[par][c][0];
#pragma unroll
      for (int w = 1; w < GW / 32; ++w) {
        b = sm->redc[par][c][w] > b ? sm->redc[par][c][w] : b;
        f |= sm->redf[par][c][w];
      }
      if (anyc != nullptr) {
        bool a = false;
#pragma unroll
        for (int cc = 0; cc < NC; ++cc)
          for (int w = 0; w < GW / 32; ++w)
            a = a || (cc < C && fkey_inv((uint32_t)(sm->redc[par][cc][w] >> 32)) >= 0.0f);
        *anyc = a;
      }
      par ^= 1;
      mx = (uint32_t)(b >> 32);
      anyf = f != 0u;
      return 255 - (int)(b & 0xFFu);
    }
  }
  // whether a group (cell) of the warp (GW <= 32: one ballot of each lane's own result `own`) or of the block
  // (GW > 32: the block-wide value `blk` an argmax already read from shared memory) has a candidate
  __device__ static bool any_candidate(bool own, bool blk) {
    if constexpr (GW > 32) {
      return blk;
    } else {
      return __ballot_sync(0xFFFFFFFFu, own) != 0u;
    }
  }
  // true on every lane of the warp (GW <= 32) or block (GW > 32) when any lane there has v; a block barrier for
  // GW > 32 (which also orders shared-memory writes before it with reads after it)
  __device__ static bool any_sync(bool v) {
    if constexpr (GW > 32) {
      return __syncthreads_or(v) != 0;
    } else {
      return __ballot_sync(0xFFFFFFFFu, v) != 0u;
    }
  }
  // OR of v over the group's lanes of cell c (this lane's cell); a block barrier for GW > 32
  template <int NC>
  __device__ static uint32_t or_cell(uint32_t v, int c, int C, SmemGroup* sm, int& par) {
    const int lane = threadIdx.x & 31;
    if constexpr (GW <= 32) {
      uint32_t res = 0u;
#pragma unroll
      for (int gq = 0; gq < 32 / GW; ++gq) {
#pragma unroll
        for (int cc = 0; cc < NC; ++cc) {
          if (cc >= C) continue;
          const bool mine = lane / GW == gq && c == cc;
          const uint32_t o = __reduce_or_sync(0xFFFFFFFFu, mine ? v : 0u);
          if (mine) res = o;
        }
      }
      return res;
    } else {
      const int wid = threadIdx.x >> 5;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        const uint32_t o = __reduce_or_sync(0xFFFFFFFFu, c == cc ? v : 0u);
        if (lane == 0) sm->redf[par][cc][wid] = o;
      }
      __syncthreads();
      uint32_t res = 0u;
#pragma unroll
      for (int w = 0; w < GW / 32; ++w) res |= sm->redf[par][c][w];
      par ^= 1;
      return res;
    }
  }
  // whether the sum of v (>= 0) over the group's lanes of some cell (this lane's cell c < C <= NC) exceeds lim: the
  // same on every lane of the warp (GW <= 32: every group's and cell's sum by warp reductions) or of the block
  // (GW > 32: per-warp partial sums through shared memory, one block barrier)
  template <int NC>
  __device__ static bool any_cell_sum_over(int v, int c, int C, int lim, SmemGroup* sm, int& par) {
    const int lane = threadIdx.x & 31;
    bool over = false;
    if constexpr (GW <= 32) {
#pragma unroll
      for (int gq = 0; gq < 32 / GW; ++gq) {
#pragma unroll
        for (int cc = 0; cc < NC; ++cc) {
          if (cc >= C) continue;
          const unsigned t = __reduce_add_sync(0xFFFFFFFFu, (lane / GW == gq && c == cc) ? (unsigned)v : 0u);
          over = over || t > (unsigned)lim;
        }
      }
    } else {
      const int wid = threadIdx.x >> 5;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        const unsigned t = __reduce_add_sync(0xFFFFFFFFu, c == cc ? (unsigned)v : 0u);
        if (lane == 0) sm->redf[par][cc][wid] = t;
      }
      __syncthreads();
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        unsigned t = 0u;
#pragma unroll
        for (int w = 0; w < GW / 32; ++w) t += sm->redf[par][cc][w];
        over = over || t > (unsigned)lim;
      }
      par ^= 1;
    }
    return over;
  }
  // as two_or_more_uniform, counting the lanes of each cell (cell index c < C) separately
  __device__ static bool two_or_more_in_a_cell_uniform(bool v, int c, int C) {
    bool multi = false;
    for (int cc = 0; cc < C; ++cc) multi = two_or_more_uniform(v && c == cc) || multi;
    return multi;
  }
  // true on every lane of the warp (GW <= 32) or block (GW > 32) when some group there has two or more lanes with v
  __device__ static bool two_or_more_uniform(bool v) {
    if constexpr (GW > 32) {
      return __syncthreads_count(v) >= 2;
    } else {
      const unsigned b = __ballot_sync(0xFFFFFFFFu, v);
      const int lane = threadIdx.x & 31;
      const unsigned gm = GW == 32 ? 0xFFFFFFFFu : (((1u << GW) - 1u) << (lane / GW * GW));
      return __ballot_sync(0xFFFFFFFFu, __popc(b & gm) >= 2) != 0u;
    }
  }
  // condition of a branch that contains collectives: uniform over the whole warp (GW < 32 packs several envs in a
  // warp, and full-mask shuffles must be reached by every lane of the warp at the same call site)
  __device__ static bool any_uniform(bool v, SmemGroup* sm, int& par) {
    if constexpr (GW > 32) {
      return any(v, sm, par);
    } else {
      return __ballot_sync(0xFFFFFFFFu, v) != 0u;
    }
  }
};

// Out-of-line IEEE divisions (each inline __fdiv_rn / __ddiv_rn carries its own ~2 KB slow path): one copy in the
// kernel instead of one per call site keeps the (long, branchy) kernel within the instruction cache.
static __device__ __noinline__ float x_fdv(float a, float b) { return fdv(a, b); }      // IEEE a / b
static __device__ __noinline__ double x_ddv(double a, double b) { return ddv(a, b); }  // IEEE a / b

// ------------------------------------------------------------------------------------------------ PHY helpers
// PHY.bler_lookup (isaac_net/core/phy.py:271-285), CUDA torch semantics: division by a python scalar is a multiply
// by the float32 reciprocal.
struct BlerGrid {
  const float* tab;
  int C, G, M;
  float s0, inv_ds;
  int32_t* status;
};

#ifdef INB_CHECK
// debug build: out-of-range index -> record (code << 24 | low bits of the index) once in the status word and use 0
__device__ __forceinline__ long long ck(long long i, long long n, int code, int32_t* status) {
  if (i < 0 || i >= n) {
    if (status != nullptr) atomicCAS(status, 0, (code << 24) | (int)(i & 0xFFFFFF) | 0x40000000);
    return 0;
  }
  return i;
}
#endif

static __device__ __noinline__ float bler_lookup(const BlerGrid bg, int mcs, float sinr, int i0, float wi) {
  const int C = bg.C, G = bg.G;
  const float* __restrict__ tab = bg.tab;
  float s = isnan(sinr) ? -30.0f : sinr;
  float x = clampf_t(fm(fs(s, bg.s0), bg.inv_ds), 0.0f, (float)(G - 1));
  int j0 = (int)floorf(x);
  if (j0 > G - 2) j0 = G - 2;
  float wj = fs(x, (float)j0);
  long long b0 = ((long long)mcs * C + i0) * (long long)G;
#ifdef INB_CHECK
  if (b0 < 0 || b0 + G + j0 + 1 >= (long long)bg.M * C * G) {
    if (bg.status != nullptr) atomicCAS(bg.status, 0, (11 << 24) | 0x40000000);
    b0 = 0;
    j0 = 0;
  }
#endif
  float omj = fs(1.0f, wj);
  float lo = fa(fm(__ldg(tab + b0 + j0), omj), fm(__ldg(tab + b0 + j0 + 1), wj));
  float hi = fa(fm(__ldg(tab + b0 + G + j0), omj), fm(__ldg(tab + b0 + G + j0 + 1), wj));
  return fa(fm(lo, fs(1.0f, wi)), fm(hi, wi));
}

// code-block index / weight of a code-block size (PHY._cidx, phy.py:263-269)
__device__ __forceinline__ void cidx(const InbParams& p, float cbs, int& i0, float& wi) {
  float x = clampf_t(fm(fs(cbs, p.c0_cbs), p.inv_dc), 0.0f, (float)(p.C_axis - 1));
  int i = (int)floorf(x);
  if (i > p.C_axis - 2) i = p.C_axis - 2;
  i0 = i;
  wi = fs(x, (float)i);
}

// LDPC segmentation (phy.py:109-119) in float64: (code-block size incl. CRC, number of code blocks)
__device__ __forceinline__ void segment(long long tbs, float r32, float& cbs, float& ncb) {
  double t = (double)tbs, r = (double)r32;
  bool bg2 = (t <= 292.0) || ((t <= 3824.0) && (r <= 0.67)) || (r <= 0.25);
  double kcb = bg2 ? 3840.0 : 8448.0;
  double b = da(t, t > 3824.0 ? 24.0 : 16.0);
  double c = (b <= kcb) ? 1.0 : ceil(x_ddv(b, dsb(kcb, 24.0)));
  double bp = (c > 1.0) ? da(b, dm(24.0, c)) : b;
  cbs = (float)x_ddv(bp, c);
  ncb = (float)c;
}

// linear -> dB with the reference's NaN / inf mapping (phy.py:137-139)
__device__ __forceinline__ float db_of(float lin) {
  if (isnan(lin)) return -30.0f;
  float v = fm(10.0f, log10f(fmaxf(lin, 1e-6f)));
  if (isnan(v)) return -30.0f;
  if (isinf(v)) return v > 0.0f ? 60.0f : -30.0f;
  return v;
}

// EESM effective SINR (dB) of one MCS over the won RBGs (PHY.eff_sinr / eff_sinr_all, phy.py:311-336):
// x_s = -lin_s / beta + log(w_s) on won RBGs, logsumexp as max + the left-to-right sum of exp(x - max),
// eff = -beta (lse - lnw).  The kernel evaluates it with one lane per RBG (warp_max, ordered_sum below).

// warp-wide max (fmaxf: order-independent) and the sum of lane values over the set bits of `won` in ascending lane
// order (the left-to-right RBG sum of the serial code; lanes outside `won` would add +0.0, which changes nothing)
__device__ __forceinline__ float warp_max(float x) {
  // order-preserving keys (NaN ranks as -inf, which fmaxf would skip; no -0.0 reaches here: every x is a sum with a
  // non-negative log(w) term), one warp reduction
  const uint32_t k = __reduce_max_sync(0xFFFFFFFFu, fkey(isnan(x) ? -INFINITY : x));
  return fkey_inv(k);
}
__device__ __forceinline__ float ordered_sum(float e, uint32_t won) {
  float acc = 0.0f;
  bool first = true;
  for (uint32_t m = won; m; m &= m - 1u) {
    const float v = __shfl_sync(0xFFFFFFFFu, e, __ffs(m) - 1);
    acc = first ? v : fa(acc, v);
    first = false;
  }
  return acc;
}

// the in-order pointer: lowest byte still owned by an undecoded process, or `sent` (MacLink.ack_ptr, mac.py:194-197);
// pend = bit mask of the processes in state 1
__device__ __forceinline__ long long ack_ptr(const InbState& st, long long eP, uint32_t pend, long long sent,
                                             long long floor_) {
  long long ack = sent;
  while (pend) {
    const int q = __ffs(pend) - 1;
    pend &= pend - 1u;
    const long long hh = st.h_hi[eP + q];
    if (hh > floor_) {
      long long ll = st.h_lo[eP + q];
      ll = ll > floor_ ? ll : floor_;
      ack = ll < ack ? ll : ack;
    }
  }
  return ack;
}

// highest MCS <= mcs_max whose 10 % BLER threshold the estimate meets, else 0 (PHY.mcs_at, phy.py:302-304);
// binary search when the thresholds are non-decreasing (checked on the host), else a linear scan
__device__ __forceinline__ int mcs_at(const float* thr, int mcs_max, bool mono, float x) {
  if (mono) {
    if (!(x >= thr[0])) return 0;
    int lo = 0, hi = mcs_max;   // invariant: thr[lo] <= x
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (x >= thr[mid]) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
  int m = 0;
  for (int mm = 0; mm <= mcs_max; ++mm)
    if (x >= thr[mm]) m = mm;
  return m;
}

// ------------------------------------------------------------------------------------------------ the step kernel
// SV: the scheduler variant.  1 is the round-robin scheduler's instance (its allocation by runs; the other
// schedulers' per-RBG rounds are left out of it, and it out of theirs, which keeps each instance's code smaller); 2 is
// the PF instance with pf_update = "rbg" (the per-RBG metric over the bytes granted so far); 0 is every other case.
// NCT: the number of cells; NCT > 1 (MC) adds the A3 association and handover, per-cell schedulers, UL power control
// and interference.  BSR: the SR / BSR grant pipeline (p.bsr_on) replaces the lumped SR grant; compiled only into the
// instances that run it, so the other instances carry none of its code.  DL: the downlink link (one cell; DlMac,
// isaac_net/core/mac_dl.py:1-49) on the same slot machinery: its own state, queue, arrivals and counters, the DL data
// rows and CQI reports of the schedule (InbParams.rows_dl), the scheduler's estimate from the last CQI report (the
// MCS threshold SINR the UE reported, csi = thr[m] - ref), no power split, HARQ-ACK timing (an ACKed process waits in
// state 2 until its HARQ-ACK reaches the gNB, a NACK until then too), the BLER_DL draws.
template <int GW, int NCT, int SV, bool BSR, bool DL>
__global__ void __launch_bounds__(GW > 32 ? GW : 128, GW > 32 ? 896 / GW : 7)
    nr_step_kernel(const InbStepArgs A, const int e_begin, const int e_end) {
  constexpr bool MC = NCT > 1;   // several cells
  constexpr int NC = NCT;        // cells this instance is compiled for (== p.C)
  constexpr bool RRK = SV == 1;  // round-robin allocation by runs (p.sched == 2)
  constexpr bool PFR = SV == 2;  // per-RBG PF metric and update (p.pf_rbg)
  constexpr int NT = GW > 32 ? GW : 128;
  constexpr int NP = NT + 1;   // row stride of the shared vectors: a warp reading one column across rows is
                               // conflict-free as well as a warp reading one row
  const InbParams& p = A.p;
  __shared__ SmemGroup smem_all[GW > 32 ? 1 : 128 / GW];
  __shared__ float s_lw[INB_MAX_S], s_lw10[INB_MAX_S], s_w[INB_MAX_S];
  __shared__ float s_thr[INB_MAX_MCS], s_se[INB_MAX_MCS], s_beta[INB_MAX_MCS], s_rate[INB_MAX_MCS];
  __shared__ unsigned long long s_ctr[GW > 32 ? 1 : 128 / GW][INB_NCTR];
  constexpr int NG = GW > 32 ? 1 : 128 / GW;   // groups (envs) per block
  __shared__ float s_fld[NG][NC][INB_MAX_KF][3];   // the env's plane waves per cell: kx, ky, phi
  // several cells: per env, the gNBs' N+I per PRB (mW) and its dB value at the start of the slot, this slot's
  // interference accumulator and N+I (dB)
  __shared__ float s_ni[MC ? NG : 1][NC][MC ? INB_MAX_S : 1], s_nidb[MC ? NG : 1][NC][MC ? INB_MAX_S : 1];
  __shared__ float s_if[MC ? NG : 1][NC][MC ? INB_MAX_S : 1], s_nadb[MC ? NG : 1][NC][MC ? INB_MAX_S : 1];
  extern __shared__ float dyn[];   // [2 or 3][S][NP]: rate / -lin, PF metric, ref (optional)
  const int tid = threadIdx.x;
  const int gpb = GW > 32 ? 1 : 128 / GW;
  const int gi = GW > 32 ? 0 : tid / GW;
  const int r = GW > 32 ? tid : tid % GW;
  SmemGroup* sm = &smem_all[gi];
  const long long e = (long long)e_begin + (long long)blockIdx.x * gpb + gi;   // envs [e_begin, e_end) of the launch
  const int R = p.R, S = p.S, P = p.P, F = p.F;
  const bool env_ok = e < e_end;
  const bool act = env_ok && r < R;
  int par = 0;
  for (int i = tid; i < S; i += NT) {
    s_lw[i] = A.t.lw[i];
    s_lw10[i] = A.t.lw10[i];
    s_w[i] = A.t.w[i];
  }
  for (int i = tid; i < p.MCS; i += NT) {
    s_thr[i] = A.t.thr_ref[i];
    s_se[i] = A.t.se[i];
    s_beta[i] = A.t.beta[i];
    s_rate[i] = A.t.rate[i];
  }
  float* const d_x = dyn;                            // rate (bytes per RBG), later -SINR_lin of the grant
  float* const d_m = dyn + (size_t)S * NP;           // PF metric rate / max(avg, 1e-9)
  float* const d_ref = dyn + (size_t)2 * S * NP;     // per-RBG reference SINR input
  float* v_x = d_x + tid;
  float* v_m = d_m + tid;
  float* v_ref = d_ref + tid;
  unsigned long long* const sc = s_ctr[gi];
  for (int i = r; i < INB_NCTR; i += GW) sc[i] = 0ull;
  const int C = MC ? p.C : 1;
  if (A.pos != nullptr && A.pathgain_in == nullptr && env_ok) {
    for (int i = r; i < C * p.Kf * 3; i += GW) {
      const int cc = i / (p.Kf * 3), k = (i / 3) % p.Kf, q = i % 3;
      const long long fo = ((long long)cc * p.E + e) * p.Kf + k;
      s_fld[gi][cc][k][q] = q < 2 ? A.t.fk[fo * 2 + q] : A.t.fphi[fo];
    }
  }
  if constexpr (MC) {
    if (env_ok) {
      for (int i = r; i < C * S; i += GW) {
        s_ni[gi][i / S][i % S] = A.s.ni_ul[e * C * S + i];
        s_if[gi][i / S][i % S] = 0.0f;
      }
    }
  }
  const int lane = tid & 31;
  const int wbase = tid - lane;                      // thread index of lane 0 of this warp
  const bool ref_vec = A.ul_ref_in != nullptr;
  __syncthreads();

  const long long er = act ? e * R + r : 0;
  const long long eP = er * P, eF = er * F, eS = er * S;
  const InbState& st = A.s;
  const long long T = (A.T_dev != nullptr) ? *A.T_dev : p.T;
#ifdef INB_CHECK
  const long long NER = (long long)p.E * R, NERF = NER * F, NERP = NER * P, NERS = NER * S, NERM = NER * p.M;
  const long long NFK = (long long)p.E * p.Kf, GCAP = A.gain_cap;
  const long long NLA = (long long)(p.nprb + 1) * p.MCS * (p.la_sets > 1 ? p.la_sets : 1);
#define CK(i, n, code) ck((i), (n), (code), A.status)
#else
#define CK(i, n, code) (i)
#endif

  // ---------------- per-robot scalars
  long long sent = 0, floor_ = 0, bsr = 0, sr_t = -1, last_tx = -1, enq = 0;
  float olla = 0.0f, avg = 100.0f;
  if (act) {
    sent = st.sent[CK(er, NER, 1)]; floor_ = st.floor_[CK(er, NER, 1)]; bsr = st.bsr[CK(er, NER, 1)]; sr_t = st.sr_t[CK(er, NER, 1)]; last_tx = st.last_tx[CK(er, NER, 1)];
    enq = st.enq[CK(er, NER, 1)]; olla = st.olla[CK(er, NER, 1)]; avg = st.avg[CK(er, NER, 1)];
  }
  float last_nprb = 0.0f;   // PRBs of the last PUSCH (ul_amc_alloc = "previous")
  if (act && p.amc_prev) last_nprb = st.last_nprb[CK(er, NER, 1)];
  // HARQ process states as bit masks (state 1: holds a TB awaiting its retransmission or ACK; state 0: free)
  uint32_t pend = 0u, freem = 0u, ackm = 0u;   // ackm (DL): state 2, decoded and waiting for its HARQ-ACK
  auto harq_state = [&](long long hs, int q) {
    if (hs == 1) pend |= 1u << q;
    else if (hs == 0) freem |= 1u << q;
    else if (DL && hs == 2) ackm |= 1u << q;
  };
#ifndef INB_CHECK
  // a robot's P states are contiguous: 16-byte loads where P is even and the array 16-byte aligned
  const bool vec_h = (P & 1) == 0 && (reinterpret_cast<uintptr_t>(st.h_state) & 15u) == 0;
#else
  const bool vec_h = false;
#endif
  if (act && vec_h) {
    const longlong2* hv = reinterpret_cast<const longlong2*>(st.h_state + eP);
#pragma unroll 4
    for (int q2 = 0; q2 < P / 2; ++q2) {
      const longlong2 v = hv[q2];
      harq_state(v.x, 2 * q2);
      harq_state(v.y, 2 * q2 + 1);
    }
  } else if (act) {
    for (int q = 0; q < P; ++q) harq_state(st.h_state[CK(eP + q, NERP, 4)], q);
  }
  const long long last_hid = env_ok ? A.last_hid[CK(e, p.E, 10)] : 0;

  // ---------------- traffic enqueue (NREngine._inject / _enqueue, engine.py:191-244; FrameQueue.add, queues.py:87-103)
  long long g_end[INB_MAX_M];
  int g_slot[INB_MAX_M];
  const int M = p.M;
  const long long n0 = enq;
  const long long base = enq;
  long long n_acc = 0;
  int cnt_q = 0;
  if (act) {
#ifndef INB_CHECK
    if ((F & 1) == 0 && (reinterpret_cast<uintptr_t>(st.cap) & 15u) == 0) {   // 16-byte loads, as the HARQ states
      const longlong2* cv = reinterpret_cast<const longlong2*>(st.cap + eF);
#pragma unroll 4
      for (int f2 = 0; f2 < F / 2; ++f2) {
        const longlong2 v = cv[f2];
        cnt_q += (v.x >= 0 ? 1 : 0) + (v.y >= 0 ? 1 : 0);
      }
    } else
#endif
    {
#pragma unroll 8
      for (int f = 0; f < F; ++f) cnt_q += st.cap[CK(eF + f, NERF, 3)] >= 0 ? 1 : 0;
    }
    for (int m = 0; m < M; ++m) {
      const long long em = er * M + m;
      const bool v = A.a.valid[CK(em, NERM, 7)] != 0;
      const float nbf = A.a.nbytes[CK(em, NERM, 7)];
      if (v && (cnt_q < F) && (nbf > 0.0f)) {
        const long long nb = (long long)rintf(nbf);
        const long long at = eF + cnt_q;
        st.cap[CK(at, NERF, 3)] = T;
        st.start[CK(at, NERF, 3)] = enq;
        st.end_[CK(at, NERF, 3)] = enq + nb;
        st.lost[CK(at, NERF, 3)] = 0;
        st.fin[CK(at, NERF, 3)] = INFINITY;
        // a generated DL message carries cls = -tag, at most -1 (NREngine._inject_dl, engine.py:660-662)
        st.cls[CK(at, NERF, 3)] = DL ? -(A.a.tag[CK(em, NERM, 7)] > 1 ? A.a.tag[CK(em, NERM, 7)] : 1) : 0;
        st.det[CK(at, NERF, 3)] = A.a.det[CK(em, NERM, 7)] != 0 ? 1 : 0;
        st.hid[CK(at, NERF, 3)] = last_hid;
        st.off[CK(at, NERF, 3)] = dm((double)A.a.slot[CK(em, NERM, 7)], p.inv_N_d);
        st.tag[CK(at, NERF, 3)] = A.a.tag[CK(em, NERM, 7)];
        st.prio[CK(at, NERF, 3)] = A.a.prio[CK(em, NERM, 7)];
        st.dline[CK(at, NERF, 3)] = A.a.dline[CK(em, NERM, 7)];
        enq += nb;
        cnt_q += 1;
        n_acc += 1;
      }
      g_end[m] = enq;
      g_slot[m] = v ? (int)A.a.slot[CK(em, NERM, 7)] : p.N;
    }
  }
  const long long full_enq = enq;
  if (M > 0) enq = base;

  // ---------------- large-scale radio: path gain of every link (one per cell)
  float pg_c[NC];
#pragma unroll
  for (int cc = 0; cc < NC; ++cc) pg_c[cc] = 0.0f;
  if (act) {
    if (A.pathgain_in != nullptr) {
#pragma unroll
      for (int cc = 0; cc < NC; ++cc)
        if (cc < C) pg_c[cc] = A.pathgain_in[CK(er * C + cc, NER * C, 1)];
    } else if (A.pos != nullptr) {
      const float px = A.pos[CK(er * 2, NER * 2, 2)], py = A.pos[CK(er * 2 + 1, NER * 2, 2)];
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        const float dx = fs(px, A.t.gnb[cc * 2]), dy = fs(py, A.t.gnb[cc * 2 + 1]);
        const float d2 = fmaxf(sqrtf(fa(fm(dx, dx), fm(dy, dy))), 1.0f);
        // shadowing: amp * sum_k cos(k . x + phi) (channels/fields.py:61-64), the field of (env, cell)
        float cs = 0.0f;
#pragma unroll 4
        for (int k = 0; k < p.Kf; ++k) {
          const float* f3 = s_fld[gi][cc][k];
          const float arg = fa(wave_phase(px, py, f3[0], f3[1], p.field_fma != 0), f3[2]);
          const float cv = cosf(arg);
          cs = k == 0 ? cv : fa(cs, cv);
        }
        pg_c[cc] = fs(formula_rx(p, d2, fm(p.amp, cs)), p.ue_tx);
      }
    }
  }
  float pg = pg_c[0];
  // ---------------- several cells: association and the A3 plan of this step (CellAssociation.associate / plan,
  // radio.py:398-432): RSRP rx = pg + ue_tx; fire slot k_ho inside the step (or -1) toward the strongest neighbour
  int serv = 0, k_ho = -1, tgt = 0, csi_src = -1;   // csi_src: -1 the stored CSI, -2 zeros (after a handover), u row
  bool fired = false;
  long long ho_end = 0, n_ho = 0;
  if constexpr (MC) {
    if (act) {
      float rx[NC];
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) rx[cc] = fa(pg_c[cc], p.ue_tx);
      serv = (int)st.serv[CK(er, NER, 1)];
      if (A.s.pending[CK(e, p.E, 10)]) {              // argmax, first index on ties
        serv = 0;
#pragma unroll
        for (int cc = 1; cc < NC; ++cc)
          if (cc < C && rx[cc] > rx[serv]) serv = cc;
      }
      ho_end = st.ho_end[CK(er, NER, 1)];
      n_ho = st.n_ho[CK(er, NER, 1)];
      float rs = rx[0], best = 0.0f;
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) if (cc == serv) rs = rx[cc];
      int bc = 0;                                     // max over the other cells, first index on ties
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
        if (cc >= C) continue;
        const float v = cc == serv ? -INFINITY : rx[cc];
        if (cc == 0 || v > best) { best = v; bc = cc; }
      }
      bool cond = best > fa(fa(rs, p.a3_off), p.a3_hyst);
      if (p.has_floor) cond = cond && (best >= p.floor_rx);
      const long long cand = st.a3_cand[CK(er, NER, 1)], cnt0 = st.a3_cnt[CK(er, NER, 1)];
      const long long cnt = (cond && bc == cand) ? cnt0 : 0;
      long long k_fire = (long long)p.ttt - cnt - 1;
      k_fire = k_fire < 0 ? 0 : k_fire;
      const bool fire = cond && k_fire < p.N;
      st.a3_cnt[CK(er, NER, 1)] = (cond && !fire) ? cnt + p.N : 0;
      st.a3_cand[CK(er, NER, 1)] = (cond && !fire) ? bc : -1;
      k_ho = fire ? (int)k_fire : -1;
      tgt = bc;
    }
  }
  // ul_ref = ue_tx - 10 log10(snr_ref_prbs) + pg - N_prb (NRNet.step_rx, nr_engine.py:613-632); with several cells
  // ul_ref = (ue_tx - 10 log10(snr_ref_prbs) + pg_serving) - N+I_serving(dB) per RBG (nr_engine.py:770-772), the
  // first sum kept in ref_pg and the N+I term read from the env's shared row of the slot
  float ref_pg = MC ? 0.0f : fs(fa(p.ul_ref0, pg), p.noise_prb);
  const float sinr_obs = fs(fa(pg, p.ue_tx), p.sub_noise);
  if (ref_vec) {
    for (int s = 0; s < S; ++s) v_ref[s * NP] = act ? A.ul_ref_in[CK(eS + s, NERS, 5)] : 0.0f;
  }
#define REF(s) (MC ? fs(ref_pg, s_nidb[MC ? gi : 0][MC ? serv : 0][s]) : (ref_vec ? v_ref[(s) * NP] : ref_pg))
  // the per-RBG reference of robot a (lane a of this warp) from lane s
#define REF_A(s, ta, ref_a, serv_a) (MC ? fs(ref_a, s_nidb[MC && GW <= 32 ? (ta) / GW : 0][MC ? (serv_a) : 0][s]) \
                                        : (ref_vec ? d_ref[(s) * NP + (ta)] : ref_a))

  // ---------------- CSI / fading gain rows of the step (written by the fading kernel)
  const long long NERr = (long long)p.E * R;
  const long long plane = (long long)S * NERr * C;   // one gain row: [E R][C][S] (C = 1: [E R][S])
  int u = 0;   // UL rows done
  // several cells: gain-row index of link (robot a, cell c) RBG s in row `row`; the CSI of robot a
#define GIDX(row, er_a, c, s) ((long long)(row) * plane + ((er_a) * C + (c)) * S + (s))
#define CSI_A(src, er_a, c, s) ((src) == -1 ? st.csi[CK((er_a) * S + (s), NERS, 5)] \
                               : ((src) == -2 ? 0.0f : A.gain[CK(GIDX((src), (er_a), (c), (s)), GCAP, 13)]))
  // PHR cap n_max = floor(snr_ref_prbs * 10^((mean(ul_ref) - phr_min) / 10) / w[0]).clamp(1, S) (mac_ul.py:165-168),
  // the mean as a left-to-right sum times float32(1 / S)
  int n_max = S;
  if (p.phr_cap && !MC) {
    float sum = 0.0f;
    for (int s = 0; s < S; ++s) sum = s == 0 ? REF(0) : fa(sum, REF(s));
    const float x = fm(fs(fm(sum, p.inv_S), p.phr_min), 0.1f);
    const float nmp = fm((float)p.ref_prbs, powf(10.0f, x));
    n_max = (int)clampf_t(floorf(x_fdv(nmp, s_w[0])), 1.0f, (float)S);
  }

  const uint32_t kenv = env_ok ? key_env(p.s0, A.env_id[CK(e, p.E, 10)], A.episode[CK(e, p.E, 10)], CH_STEP, A.rng_ctr[CK(e, p.E, 10)]) : 0u;
  const bool thr_mono = p.thr_mono != 0;
  const BlerGrid bgrid = {A.t.bler, p.C_axis, p.G_axis, p.MCS, p.s0_snr, p.inv_ds, A.status};


  // RLC scan start: the first frame neither lost nor finished, and its end byte (frames are in stream order, and
  // within a step a frame's end never changes, so the cached end decides whether a slot can deliver anything)
  const int nvalid = cnt_q;
  int f_scan = 0;
  long long end_scan = LLONG_MAX;
  bool q_dirty = false;   // frames were marked lost in this slot: the scan start may move
  auto rescan = [&]() {
    while (f_scan < nvalid && (st.lost[CK(eF + f_scan, NERF, 3)] != 0 || !isinf(st.fin[CK(eF + f_scan, NERF, 3)]))) ++f_scan;
    end_scan = f_scan < nvalid ? st.end_[CK(eF + f_scan, NERF, 3)] : LLONG_MAX;
  };
  if (act) rescan();

  // ---- handover of this robot at slot g_sw (CellAssociation.switch, radio.py:434-444; MacLink.handover,
  // mac.py:557-582; UlMac.handover, mac_ul.py:238-243): the target cell serves from g_sw + ho_int on; HARQ combining
  // restarts (or, under RLC UM or ho_rlc = "flush", the TBs in flight are lost, and flush drops every queued frame
  // not completed); OLLA, the PF average and the CSI start afresh; a pending SR is dropped; BSR = unsent bytes
  auto handover = [&](long long g_sw) {
    serv = tgt;
    ho_end = g_sw + p.ho_int;
    n_ho += 1;
    if (p.harq_drop || p.ho_flush) {
      for (int f = 0; f < F; ++f) {
        const long long at = eF + f;
        const bool valid = st.cap[CK(at, NERF, 3)] >= 0 && isinf(st.fin[CK(at, NERF, 3)]) && !st.lost[CK(at, NERF, 3)];
        if (!valid) continue;
        bool ov = p.ho_flush != 0;
        for (uint32_t m_ = pend; m_ && !ov; m_ &= m_ - 1u) {
          const int q = __ffs(m_) - 1;
          ov = st.start[CK(at, NERF, 3)] < st.h_hi[CK(eP + q, NERP, 4)] && st.end_[CK(at, NERF, 3)] > st.h_lo[CK(eP + q, NERP, 4)];
        }
        if (ov) {
          st.lost[CK(at, NERF, 3)] = 1;
          atomicAdd(sc + INB_CTR_LOST_FRAMES, 1ull);
        }
      }
      if (p.ho_flush) sent = enq;
      for (uint32_t m_ = pend; m_; m_ &= m_ - 1u) st.h_state[CK(eP + __ffs(m_) - 1, NERP, 4)] = 0;
      freem |= pend;
      pend = 0u;
      q_dirty = true;
    } else {
      for (uint32_t m_ = pend; m_; m_ &= m_ - 1u) {
        const int q = __ffs(m_) - 1;
        st.h_ntx[CK(eP + q, NERP, 4)] = 0;
        st.h_comb[CK(eP + q, NERP, 4)] = 0.0f;
      }
    }
    olla = 0.0f;
    avg = 100.0f;
    csi_src = -2;
    sr_t = -1;
    bsr = enq - sent;
    if constexpr (BSR) bsr_handover(st, p, er, enq, sent);
  };


  // ======================================================================= slot loop (nr_engine.py:656-667)
  for (int k = 0; k < p.K_rows; ++k) {
    // uls: the data symbols of this link's slot (the DL instance: the row's DL data symbols); srf: SR opportunity
    const int rel = p.rows[k][0], uls = DL ? p.rows_dl[k][0] : p.rows[k][1], srf = DL ? 0 : p.rows[k][2];
    const long long g = T * p.N + rel;
    if constexpr (MC) {   // A3 handovers due by this slot fire before it (nr_engine.py:748-752)
      if (act && k_ho >= 0 && k_ho <= rel && !fired) {
        handover(T * p.N + k_ho);
        fired = true;
      }
    }
    // ---- arrival gate (NREngine._open_gate, engine.py:176-183)
    if ((srf || uls) && M > 0 && act) {
      long long vis = base;
      for (int m = 0; m < M; ++m) {
        const long long v = g_slot[m] <= rel ? g_end[m] : base;
        vis = v > vis ? v : vis;
      }
      enq = vis > base ? vis : base;
    }
    // ---- DL CQI report (DlMac.cqi_report, mac_dl.py:28-39; NRNet.step, nr_engine.py:660-661), before the row's DL
    // data slot: per RBG the highest MCS (<= the DL cap) whose threshold the SINR ref + gain meets; the gNB keeps that
    // MCS's threshold SINR, csi = thr[m] - ref
    if constexpr (DL) {
      if (p.rows_dl[k][1] && act) {
        const long long gq = (long long)(p.n_ul_rows + 1 + p.rows_dl[k][3]) * plane + er * S;
        for (int s = 0; s < S; ++s) {
          const float rs = REF(s);
          const int m = mcs_at(s_thr, p.mcs_max, thr_mono, fa(rs, A.gain[CK(gq + s, GCAP, 13)]));
          st.csi[CK(eS + s, NERS, 5)] = fs(s_thr[m], rs);
        }
      }
    }
    // ---- SR (UlMac.sr_step, mac_ul.py:66-71; the BSR pipeline's, mac_ul.py:280-287)
    if (srf && act) {
      if constexpr (BSR) bsr_sr_step(st, er, enq, sent, g, sr_t);
      if (!BSR && (enq - sent > 0) && bsr <= 0 && sr_t < 0) sr_t = g;
    }
    if (!uls) continue;

    // =================================================================== data slot (MacLink.slot, mac.py:228-508)
    const long long unsent = enq - sent;
    // the CSI of this decision is gain row u (the gain of the previous UL row), this row's fading gain is row u + 1;
    // the DL instance reads its CSI state (the CQI reports) and the row's DL gain row
    const long long g_csi = (long long)u * plane;
    const long long g_gain = DL ? (long long)(p.n_ul_rows + 1 + p.rows_dl[k][3]) * plane : g_csi + plane;
    if constexpr (DL) {   // DL processes whose HARQ-ACK has reached the gNB become free (mac.py:238-239)
      for (uint32_t m_ = ackm; m_; m_ &= m_ - 1u) {
        const int q = __ffs(m_) - 1;
        if (st.h_ready[CK(eP + q, NERP, 4)] <= g) {
          st.h_state[CK(eP + q, NERP, 4)] = 0;
          ackm &= ~(1u << q);
          freem |= 1u << q;
        }
      }
    }
    // lumped SR grant (mac_ul.py:140-147), or the BSR pipeline's bootstrap grant and matured reports
    long long need_bsr = 0;
    if constexpr (BSR) {
      if (act) need_bsr = bsr_pre_slot(st, p, er, enq, g, sr_t);
    } else if (!DL && sr_t >= 0 && g - sr_t >= p.sr_delay) {
      bsr = bsr < 1 ? 1 : bsr;
      sr_t = -1;
    }
    // candidates: earliest ready NACKed process, else the first free one (mac.py:241-253)
    int rx_p = 0, p_new = freem ? __ffs(freem) - 1 : -1;
    long long best_ready = BIGI;
    bool has_rx = false;
    const bool pending = pend != 0u;
    for (uint32_t m_ = pend; m_; m_ &= m_ - 1u) {
      const int q = __ffs(m_) - 1;
      const long long rd = st.h_ready[CK(eP + q, NERP, 4)];
      if (rd <= g) {
        has_rx = true;
        if (rd < best_ready) { best_ready = rd; rx_p = q; }
      }
    }
    const bool any_free = p_new >= 0;
    if (p_new < 0) p_new = 0;
    const long long need = DL ? unsent : (BSR ? need_bsr : (bsr < unsent ? bsr : unsent));   // DL: MacLink._need
    bool new_el = act && any_free && need > 0 && !has_rx;
    float pcv = -INFINITY;   // power-control backoff (dB), -inf without power control
    if constexpr (MC) {
      // the env's N+I in dB of this slot, the serving link's reference, power control and the PHR cap.  The previous
      // slot's decode reads s_nidb with no barrier after it, so every warp of the env must be past it first.
      if constexpr (GW > 32) __syncthreads(); else __syncwarp();
      for (int i = r; i < C * S; i += GW) s_nidb[gi][i / S][i % S] = fm(10.0f, log10f(s_ni[gi][i / S][i % S]));
      float pg_s = pg_c[0];
#pragma unroll
      for (int cc = 1; cc < NC; ++cc) if (cc == serv) pg_s = pg_c[cc];
      ref_pg = fa(pg_s, p.ue_tx_ref);
      const float rx_s = fa(pg_s, p.ue_tx);
      if (p.pc_on) pcv = fs(p.ue_tx, fa(p.pc_p0, fm(p.pc_alpha, fs(p.ue_tx, rx_s))));
      if (p.phr_cap) {
        const float x = fm(fs(fs(rx_s, p.sub_noise), p.phr_min), 0.1f);
        const float nmp = fm((float)p.ref_prbs, powf(10.0f, x));
        n_max = (int)clampf_t(floorf(x_fdv(nmp, s_w[0])), 1.0f, (float)S);
      }
      const bool ok = g >= ho_end;              // outside the handover interruption (mac.py:249-251)
      has_rx = has_rx && ok;
      new_el = new_el && ok;
      if constexpr (GW > 32) __syncthreads(); else __syncwarp();
    }
    const int rx_nsb = has_rx ? (int)st.h_nsb[CK(eP + rx_p, NERP, 4)] : 0;
    // scheduler estimate with OLLA -> rate (bytes per RBG) (mac.py:255-266, mac_ul.py:154-171) and the scheduler
    // metric per RBG: PF rate / avg, maxCI rate, RR slot age (mac.py:267-275).  Only robots that may want RBGs use
    // them; those are few, so the warp evaluates one such robot at a time with one lane per RBG.
    const float re_prb = (float)min(12 * uls - p.dmrs - p.oh, 156);
    const float avg_den = fmaxf(avg, 1e-9f);
    const float rr_metric = (float)(g - last_tx);
    {
      const uint32_t wm0 = __ballot_sync(0xFFFFFFFFu, has_rx || new_el);
      if (MC ? __popc(wm0) >= 6 : __popc(wm0) * 4 > S * 3) {
        // many robots of the warp want RBGs (loaded cells: the multi-cell configs, a saturated uplink): each lane
        // evaluates its own robot, RBG by RBG (the same expressions), instead of one robot at a time (measured:
        // one cell from three quarters of S robots on, several cells from six)
        if (has_rx || new_el) {
          // the rates first (no call in the loop, so the CSI loads of several RBGs are in flight together), then the
          // PF metrics
          for (int s = 0; s < S; ++s) {
            float est;
            if constexpr (MC) {
              est = fa(fs(REF(s), fmaxf(s_lw10[s], pcv)), CSI_A(csi_src, er, serv, s));
            } else if constexpr (DL) {   // DlMac._sched_estimate (mac_dl.py:41-42): ref + csi
              est = fa(REF(s), st.csi[CK(eS + s, NERS, 5)]);
            } else {
              est = fa(fs(REF(s), s_lw10[s]), A.gain[CK(g_csi + er * S + s, GCAP, 13)]);
            }
            const float eo = p.olla_on ? fa(est, olla) : fa(est, 0.0f);
            const int m = mcs_at(s_thr, p.mcs_max, thr_mono, eo);
            v_x[s * NP] = fm(fm(fm(s_se[m], re_prb), s_w[s]), 0.125f);
          }
          if (p.sched == 0)
            for (int s = 0; s < S; ++s) v_m[s * NP] = x_fdv(v_x[s * NP], avg_den);
        }
      } else {
        // the CSI of robot a on this lane's RBG (every lane calls it: it shuffles); the next robot's is loaded while
        // the warp works on this one
        auto csi_of = [&](int a) {
          const long long ra = __shfl_sync(0xFFFFFFFFu, er, a) * S;
          const int serv_a = MC ? __shfl_sync(0xFFFFFFFFu, serv, a) : 0;
          const int csrc_a = MC ? __shfl_sync(0xFFFFFFFFu, csi_src, a) : 0;
          float v = 0.0f;
          if (lane < S) {
            const int s = lane;
            if constexpr (MC) {
              v = CSI_A(csrc_a, ra / S, serv_a, s);
            } else if constexpr (DL) {
              v = st.csi[CK(ra + s, NERS, 5)];
            } else {
              v = A.gain[CK(g_csi + ra + s, GCAP, 13)];
            }
          }
          return v;
        };
        float csi_next = wm0 ? csi_of(__ffs(wm0) - 1) : 0.0f;
        for (uint32_t wm = wm0; wm; wm &= wm - 1u) {
          const int a = __ffs(wm) - 1;
          const float csi_a = csi_next;
          const uint32_t later = wm & (wm - 1u);
          if (later) csi_next = csi_of(__ffs(later) - 1);
          const int ta = wbase + a;
          const float ref_a = __shfl_sync(0xFFFFFFFFu, ref_pg, a);
          const float olla_a = __shfl_sync(0xFFFFFFFFu, olla, a);
          const float avgd_a = __shfl_sync(0xFFFFFFFFu, avg_den, a);
          const int serv_a = MC ? __shfl_sync(0xFFFFFFFFu, serv, a) : 0;
          const float pc_a = MC ? __shfl_sync(0xFFFFFFFFu, pcv, a) : 0.0f;
          if (lane < S) {
            const int s = lane;
            const float refs = REF_A(s, ta, ref_a, serv_a);
            float est;
            if constexpr (MC) {   // one RBG at the power-control PSD (mac_ul.py:160-161)
              est = fa(fs(refs, fmaxf(s_lw10[s], pc_a)), csi_a);
            } else if constexpr (DL) {
              est = fa(refs, csi_a);
            } else {
              est = fa(fs(refs, s_lw10[s]), csi_a);
            }
            const float eo = p.olla_on ? fa(est, olla_a) : fa(est, 0.0f);
            const int m = mcs_at(s_thr, p.mcs_max, thr_mono, eo);
            const float rt = fm(fm(fm(s_se[m], re_prb), s_w[s]), 0.125f);
            d_x[s * NP + ta] = rt;
            if (p.sched == 0) d_m[s * NP + ta] = x_fdv(rt, avgd_a);
          }
        }
      }
      __syncwarp();
    }
#define RATE(s) v_x[(s) * NP]
#define METRIC(s) (p.sched == 2 ? rr_metric : (p.sched == 1 ? RATE(s) : v_m[(s) * NP]))
    // the allocation's metric of RBG s: with pf_update = "rbg" the PF rate over the average moved by the bytes this
    // robot has been granted so far in the slot (MacLink._rbg_metric, mac.py:526-532), else the slot metric
    const float pf_base = fm(p.pf_a, avg);
    float got = 0.0f;
#define AMET(s) (PFR ? x_fdv(RATE(s), fmaxf(fa(pf_base, fm(p.pf_b, got)), 1e-9f)) : METRIC(s))
    if (p.tdma) {
      // 5G-LENA UL HARQ (ul_retx_sched = "tdma", mac.py:279-299): one retransmission per slot and cell, the oldest
      // NACK (earliest ready slot of its process; lowest robot on ties, torch.argmin) first, and no new data in a
      // cell that has one.  Key: 1 + the slots since it became ready, so the arg-max is the arg-min of ready.
      const long long age = g - best_ready;
      const uint32_t key = has_rx ? (uint32_t)(age < 0xFFFFFFFELL ? age : 0xFFFFFFFELL) + 1u : 0u;
      uint32_t mx = 0u;
      bool anyrx = false;
      const int wl = Grp<GW>::template argmax_cell<NC>(key, has_rx, serv, C, mx, anyrx, sm, par);
      const bool adm = has_rx && wl == r;
      if (anyrx) new_el = false;
      if (adm && p.lena_ctr && rx_nsb < S) atomicAdd(sc + INB_CTR_RETX_BLOCK, 1ull);
      has_rx = adm;
    } else if (Grp<GW>::template any_cell_sum_over<NC>(has_rx ? rx_nsb : 0, serv, C, S, sm, par)) {
      // retransmission admission: rank by metric sum (stable, descending), admit while RBG counts fit
      // (mac.py:300-312).  Where the retransmissions of every cell need S RBGs or fewer in all, each one's count
      // plus those ranked before it fits, so all are admitted and the ranking is skipped (the branch's condition).
      float rkey = -1.0f;
      if (has_rx) {
        float sum = 0.0f;
        for (int s = 0; s < S; ++s) sum = s == 0 ? METRIC(0) : fa(sum, METRIC(s));
        rkey = sum;
      }
      const int mine = has_rx ? rx_nsb : 0;
      int before = 0;   // several cells: the ranking runs inside each cell (mac.py:313-319)
      // only robots with a retransmission hold RBGs in this count (the others have mine = 0)
      if constexpr (GW <= 32) {
        const int gb = lane / GW * GW;   // lane of robot 0 of this group
#pragma unroll 1
        for (unsigned hm = __ballot_sync(0xFFFFFFFFu, has_rx); hm; hm &= hm - 1u) {
          const int jl = __ffs(hm) - 1;
          const float kj = __shfl_sync(0xFFFFFFFFu, rkey, jl);
          const int nj = __shfl_sync(0xFFFFFFFFu, mine, jl);
          const int sj = MC ? __shfl_sync(0xFFFFFFFFu, serv, jl) : 0;
          const int j = jl - gb;
          if (jl >= gb && j < GW && (!MC || sj == serv) && (kj > rkey || (kj == rkey && j < r))) before += nj;
        }
      } else {
        sm->rkey[r] = rkey;
        sm->rnsb[r] = mine;
        sm->rserv[r] = serv;
        const unsigned hm = __ballot_sync(0xFFFFFFFFu, has_rx);
        if (lane == 0) sm->rmask[r >> 5] = hm;
        __syncthreads();
#pragma unroll 1
        for (int w = 0; w < GW / 32; ++w) {
          for (unsigned m_ = sm->rmask[w]; m_; m_ &= m_ - 1u) {
            const int j = w * 32 + __ffs(m_) - 1;
            const float kj = sm->rkey[j];
            if ((!MC || sm->rserv[j] == serv) && (kj > rkey || (kj == rkey && j < r))) before += sm->rnsb[j];
          }
        }
        __syncthreads();
      }
      has_rx = has_rx && (before + mine <= S);
    }
    const int want_cnt = has_rx ? rx_nsb : (new_el ? n_max : 0);
    const bool lex = p.retx_priority != 0;
    const float prio = lex ? fm(1e9f, has_rx ? 1.0f : 0.0f) : 0.0f;
    // greedy allocation RBG by RBG (mac.py:322-351); key = (retx wanting, metric + prio, lowest robot).  RBGs only
    // move while at least one robot wants them, so where no group of the warp (block) has two candidates the only
    // candidate takes each RBG it still wants, which is what the argmax rounds give; else the rounds run.
    uint32_t won = 0u;
    int cnt = 0;
    float left = (float)need;
    // several cells: one scheduler per cell on the same RBGs (mac.py:335-345), the argmax over the cell's robots
    const bool contested = MC ? Grp<GW>::two_or_more_in_a_cell_uniform(act && want_cnt > 0, serv, C)
                              : Grp<GW>::two_or_more_uniform(act && want_cnt > 0);
    // the retransmission mask below can only act where a retransmission competes (uniform over the warp / block)
    const bool lex_mask = lex && contested && Grp<GW>::any_sync(act && has_rx);
    if (contested && RRK) {
      // Round robin (the RRK instance, p.sched == 2): a robot's metric (slots since its last transmission) is the
      // same on every RBG, so the RBG by RBG argmax of the generic rounds (the other instances) keeps picking one
      // robot until it stops wanting, then the next: each
      // round here finds a cell's winner once (the same key, the same candidates, the same lowest-index tie rule;
      // with retransmission priority the retransmissions are the candidates while one of them wants) and the winner
      // takes RBGs from the cell's cursor on while it still wants, exactly the RBGs the per-RBG rounds give it.
      int cur = 0;   // next RBG of this lane's cell (the same on every lane of the cell)
      bool live = true;
#pragma unroll 1
      for (;;) {
        const bool want = act && (cnt < want_cnt) && (has_rx || left > 0.0f);
        float mkey = want ? fa(rr_metric, prio) : -1.0f;
        if (lex_mask) {
          const bool wr = want && has_rx;
          bool any_wr = false;
          uint32_t mx_;
          Grp<GW>::template argmax_cell<NC>(1u, wr, serv, C, mx_, any_wr, sm, par);
          if (any_wr && !wr) mkey = -1.0f;
        }
        uint32_t mx;
        bool unused;
        const int w = Grp<GW>::template argmax_cell<NC>(fkey(mkey), false, serv, C, mx, unused, sm, par);
        const bool has = live && cur < S && fkey_inv(mx) >= 0.0f;
        int ncur = cur;
        if (has && w == r) {
          int s = cur;
          while (s < S && cnt < want_cnt && (has_rx || left > 0.0f)) {
            won |= 1u << s;
            cnt += 1;
            if (!has_rx) left = fs(left, RATE(s));
            ++s;
          }
          ncur = s;
          if constexpr (GW > 32) sm->bc[par][serv] = ncur;
        }
        bool progress;
        if constexpr (GW > 32) {
          progress = Grp<GW>::any_sync(has);
          if (has) cur = sm->bc[par][serv];
          par ^= 1;
        } else {
          const int nc_w = __shfl_sync(0xFFFFFFFFu, ncur, (lane / GW) * GW + w);
          progress = Grp<GW>::any_sync(has);
          if (has) cur = nc_w;
        }
        live = has;
        if (!progress) break;
      }
      if (!lex) {
        // retransmissions that won fewer RBGs than their TB needs release them to the new-data robots of their
        // cell, which take the released RBGs in RBG order by the same rule (mac.py:353-379)
        const bool short_ = has_rx && (__popc(won) != rx_nsb);
        const uint32_t rel_rs = short_ ? won : 0u;
        if (short_) won = 0u;
        cnt = __popc(won);
        uint32_t rs = Grp<GW>::template or_cell<NC>(rel_rs, serv, C, sm, par);   // this cell's released RBGs
        if (Grp<GW>::any_sync(rs != 0u)) {
          bool live2 = true;
#pragma unroll 1
          for (;;) {
            const bool want = act && (cnt < want_cnt) && new_el && (left > 0.0f);
            const float mkey = want ? rr_metric : -1.0f;
            uint32_t mx;
            bool unused;
            const int w = Grp<GW>::template argmax_cell<NC>(fkey(mkey), false, serv, C, mx, unused, sm, par);
            const bool has = live2 && rs != 0u && fkey_inv(mx) >= 0.0f;
            uint32_t nrs = rs;
            if (has && w == r) {
              while (nrs != 0u && cnt < want_cnt && left > 0.0f) {
                const int s = __ffs(nrs) - 1;
                nrs &= nrs - 1u;
                won |= 1u << s;
                cnt += 1;
                left = fs(left, RATE(s));
              }
              if constexpr (GW > 32) sm->bc[par][serv] = (int32_t)nrs;
            }
            bool progress;
            if constexpr (GW > 32) {
              progress = Grp<GW>::any_sync(has);
              if (has) rs = (uint32_t)sm->bc[par][serv];
              par ^= 1;
            } else {
              const uint32_t nrs_w = __shfl_sync(0xFFFFFFFFu, nrs, (lane / GW) * GW + w);
              progress = Grp<GW>::any_sync(has);
              if (has) rs = nrs_w;
            }
            live2 = has;
            if (!progress) break;
          }
        }
      }
    } else if (contested && !RRK) {
#pragma unroll 1
      for (int s = 0; s < S; ++s) {
        const bool want = act && (cnt < want_cnt) && (has_rx || left > 0.0f);
        float mkey = want ? fa(AMET(s), prio) : -1.0f;
        if (lex_mask) {   // while a retransmission wants RBG s, the new-data robots of the cell are masked out
          const bool wr = want && has_rx;
          bool any_wr = false;
          if constexpr (MC) {
            uint32_t mx_;
            Grp<GW>::template argmax_cell<NC>(1u, wr, serv, C, mx_, any_wr, sm, par);   // every lane takes part
          } else {
            any_wr = Grp<GW>::any(wr, sm, par);
          }
          if (any_wr && !wr) mkey = -1.0f;
        }
        bool oh, more;
        if constexpr (MC) {
          uint32_t mx;
          bool unused, anyc = true;
          const int w = Grp<GW>::template argmax_cell<NC>(fkey(mkey), false, serv, C, mx, unused, sm, par, &anyc);
          oh = (w == r) && (fkey_inv(mx) >= 0.0f);
          more = Grp<GW>::any_candidate(fkey_inv(mx) >= 0.0f, anyc);
        } else {
          uint32_t mx;
          const int w = Grp<GW>::argmax_u32(fkey(mkey), mx, sm, par);
          oh = (w == r) && (fkey_inv(mx) >= 0.0f);
          more = Grp<GW>::any_candidate(fkey_inv(mx) >= 0.0f, fkey_inv(mx) >= 0.0f);
        }
        if (oh) {
          won |= 1u << s;
          cnt += 1;
          if (PFR) got = fa(got, RATE(s));
          if (!has_rx) left = fs(left, RATE(s));
        }
        // `want` does not depend on s and only ever turns off: once no robot of the warp (block) is a candidate,
        // no later round gives an RBG, so every lane leaves the rounds together
        if (!more) break;
      }
      if (!lex) {
        // retransmissions that won fewer RBGs than their TB needs release them to the new-data robots (mac.py:353-379)
        const bool short_ = has_rx && (__popc(won) != rx_nsb);
        const uint32_t rel_rs = short_ ? won : 0u;
        if (short_) won = 0u;
        cnt = __popc(won);
#pragma unroll 1
        for (int s = 0; s < S; ++s) {
          const bool want = act && (cnt < want_cnt) && new_el && (left > 0.0f);
          const float mkey = want ? AMET(s) : -1.0f;
          uint32_t mx;
          bool av;
          bool anyc = true;
          const int w = Grp<GW>::template argmax_cell<NC>(fkey(mkey), ((rel_rs >> s) & 1u) != 0u, serv, C, mx, av, sm,
                                                          par, &anyc);
          const bool oh = (w == r) && (fkey_inv(mx) >= 0.0f) && av;
          const bool more = Grp<GW>::any_candidate(fkey_inv(mx) >= 0.0f, anyc);
          if (oh) {
            won |= 1u << s;
            cnt += 1;
            if (PFR) got = fa(got, RATE(s));
            left = fs(left, RATE(s));
          }
          if (!more) break;   // as in the rounds above: no candidate now, none later
        }
      }
    } else {
      if (act && want_cnt > 0) {
#pragma unroll 1
        for (int s = 0; s < S && cnt < want_cnt; ++s) {
          if (!(has_rx || left > 0.0f)) break;
          if (fa(AMET(s), prio) >= 0.0f) {
            won |= 1u << s;
            cnt += 1;
            if (PFR) got = fa(got, RATE(s));
            if (!has_rx) left = fs(left, RATE(s));
          }
        }
      }
      // a short retransmission releases its RBGs; with no other candidate nobody takes them
      if (!lex && has_rx && (__popc(won) != rx_nsb)) won = 0u;
    }
#undef AMET
#undef METRIC
#undef RATE
    const int n_sb = __popc(won);
    float n_prb = 0.0f;
    for (int s = 0; s < S; ++s)
      if ((won >> s) & 1u) n_prb = fa(n_prb, s_w[s]);
    const bool tx_rx = has_rx && (n_sb == rx_nsb) && (n_sb > 0);
    const bool tx_new = new_el && (n_sb > 0);
    const bool tx = tx_rx || tx_new;
    // power split over the grant (UlMac._split, mac_ul.py:173-180)
    // (the DL has none: est_tx = est and the decode SINR ref + gain, mac_dl.py:44-45; ref - 0 is ref exactly)
    // (ul_power = "whole_band": a fixed PSD, the same split for every grant, mac_ul.py:173-176)
    float split = DL ? 0.0f : (p.whole_band ? p.wb_db : fm(10.0f, log10f(clamp_min_t(fm(n_prb, p.inv_ref_prbs), 1e-3f))));
    if constexpr (MC) split = fmaxf(split, pcv);   // at least the power-control backoff (mac_ul.py:176-180)
    // The transmitting robots of a slot are few: the warp serves them one at a time, with one lane per RBG for the
    // EESM normalization (and the decode SINR below) and one lane per MCS for link adaptation.
    float lnw = 0.0f;
    int mcs_new = 0;
    long long tbs_new = 0;
    uint32_t la_serial = __ballot_sync(0xFFFFFFFFu, tx);   // robots served one at a time below
    bool rest_only = false;                                // ... for the lane-per-MCS search only
    // the CSI of this lane's robot on RBG s_ (the scheduler's, as the estimate above read it)
#define CSI_OWN(s_) (MC ? CSI_A(csi_src, er, serv, (s_)) \
                        : (DL ? st.csi[CK(eS + (s_), NERS, 5)] : A.gain[CK(g_csi + er * S + (s_), GCAP, 13)]))
    // Several robots of the warp transmit: unless one of them holds many more RBGs than there are transmitters, each
    // lane evaluates its own robot's per-RBG work (a chain per won RBG, all lanes at once) for link adaptation and the
    // decode SINR, instead of the warp serving the robots one at a time (one chain per robot, a lane per RBG).  The
    // same expressions in the same order (the max order-free, the sums left to right over the won RBGs).
    const int k_tx = __popc(la_serial);
    const int won_max = (int)__reduce_max_sync(0xFFFFFFFFu, tx ? (unsigned)__popc(won) : 0u);
    // (measured: one cell, any two or more transmitters whose largest grant is under 5 k_tx - 4 RBGs; several cells,
    // where the loaded cells grant many RBGs per robot, six or more for link adaptation and, with the per-RBG rounds of
    // PF, for the decode and the interference (config 3: 4.88 -> 3.75 ms per step); with several cells and round robin,
    // whose runs give a few robots most of the band, the decode and the interference stay one robot at a time (config
    // 5: 5.38 vs 5.52 ms)).  The same on every lane of the warp.
    const bool lane_one = k_tx >= 2 && won_max + 4 <= 5 * k_tx;
    const bool lane_own = MC ? k_tx >= 6 : lane_one;                                   // link adaptation
    const bool lane_dec = MC ? (!RRK && k_tx >= 6 && won_max <= k_tx) : lane_one;   // decode SINR, interference
    // The RBGs whose EESM chooses a new TB's MCS: the grant, or with ul_amc_alloc = "previous" and the whole-band
    // PSD every RBG of the band (mac.py:393-400); lnw_la is the logsumexp of log(w) over them (lnw: over the grant,
    // for the decode).  Compiled into the per-RBG PF instance only, the scheduler of the 5G-LENA switch set (the host
    // refuses the combination with the others): elsewhere its code cost 1-3 % of the step.
    const bool la_band = PFR && !DL && p.whole_band && p.amc_prev;
    const uint32_t band = S >= 32 ? 0xFFFFFFFFu : ((1u << S) - 1u);
    float lnw_la = 0.0f;
    {
      // link adaptation: grant, lnw and the top MCS per lane; only robots whose top MCS fails take the lane-per-MCS
      // search below, with their -SINR_lin already in their column
      if (lane_own) {
        bool more = false;
        if (tx) {
          uint32_t kmx = 0u;
          for (uint32_t bb = won; bb; bb &= bb - 1u) kmx = max(kmx, fkey(s_lw[__ffs(bb) - 1]));
          const float lmx = fkey_inv(kmx);
          const float lm0 = isinf(lmx) ? 0.0f : lmx;
          float sw = 0.0f;
          for (uint32_t bb = won; bb; bb &= bb - 1u) {
            const float ev = expf(fs(s_lw[__ffs(bb) - 1], lm0));
            sw = bb == won ? ev : fa(sw, ev);
          }
          lnw = fa(logf(sw), lm0);
          if (tx_new) {
            const uint32_t lam = la_band ? band : won;
            lnw_la = lnw;
            if (lam != won) {
              uint32_t kml = 0u;
              for (uint32_t bb = lam; bb; bb &= bb - 1u) kml = max(kml, fkey(s_lw[__ffs(bb) - 1]));
              const float lml = fkey_inv(kml);
              const float lm0l = isinf(lml) ? 0.0f : lml;
              float swl = 0.0f;
              for (uint32_t bb = lam; bb; bb &= bb - 1u) {
                const float ev = expf(fs(s_lw[__ffs(bb) - 1], lm0l));
                swl = bb == lam ? ev : fa(swl, ev);
              }
              lnw_la = fa(logf(swl), lm0l);
            }
            const float off_ = p.olla_on ? olla : 0.0f;
            for (uint32_t bb = lam; bb; bb &= bb - 1u) {
              const int s_ = __ffs(bb) - 1;
              const float est_tx = fa(fs(REF(s_), split), CSI_OWN(s_));
              v_x[s_ * NP] = -powf(10.0f, fm(clampf_t(est_tx, -30.0f, 60.0f), 0.1f));
            }
            // the TBS row of this grant (the DL: in the table set of this slot's DL data symbols), and the row the
            // MCS is chosen on (the last PUSCH's PRBs under ul_amc_alloc = "previous", mac.py:393-400)
            const long long tab0_ = DL ? (long long)p.dl_nsym_tab[uls] * (p.nprb + 1) * p.MCS : 0;
            const long long trow_g = tab0_ + (long long)(int)n_prb * p.MCS;
            const long long trow = (p.amc_prev && last_nprb > 0.0f) ? (long long)(int)last_nprb * p.MCS : trow_g;
            int mtop = -1, n_cand = 0;
            for (int m = min(p.mcs_max, p.MCS - 1); m >= 0; --m) {
              if (A.t.la_tbs[CK(trow + m, NLA, 9)] > 0) {
                if (mtop < 0) mtop = m;
                ++n_cand;
                if (n_cand > 1) break;
              }
            }
            int chosen = -1;
            if (mtop >= 0) {
              const float beta = s_beta[mtop];
              uint32_t kx = 0u;
              for (uint32_t bb = lam; bb; bb &= bb - 1u) {
                const int s_ = __ffs(bb) - 1;
                const float x = fa(x_fdv(v_x[s_ * NP], beta), s_lw[s_]);
                kx = max(kx, fkey(isnan(x) ? -INFINITY : x));
              }
              const float mx = fkey_inv(kx);
              const float m0 = isinf(mx) ? 0.0f : mx;
              float se = 0.0f;
              for (uint32_t bb = lam; bb; bb &= bb - 1u) {
                const int s_ = __ffs(bb) - 1;
                const float ev = expf(fs(fa(x_fdv(v_x[s_ * NP], beta), s_lw[s_]), m0));
                se = bb == lam ? ev : fa(se, ev);
              }
              const float lse = fa(logf(se), m0);
              const float eff = fa(db_of(fm(-beta, fs(lse, lnw_la))), off_);
              const float b = bler_lookup(bgrid, mtop, eff, A.t.la_i0[CK(trow + mtop, NLA, 9)],
                                          A.t.la_wi[CK(trow + mtop, NLA, 9)]);
              const float tbler = fs(1.0f, powf(fs(1.0f, b), A.t.la_ncb[CK(trow + mtop, NLA, 9)]));
              if (tbler <= p.target) chosen = mtop;
            }
            if (chosen >= 0 || n_cand <= 1) {
              mcs_new = chosen < 0 ? 0 : chosen;
              tbs_new = A.t.la_tbs[CK(trow_g + mcs_new, NLA, 9)];
            } else {
              more = true;
            }
          }
        }
        la_serial = __ballot_sync(0xFFFFFFFFu, more);
        rest_only = true;
      }
    }
    for (uint32_t tm = la_serial; tm; tm &= tm - 1u) {
      const int a = __ffs(tm) - 1;
      const int ta = wbase + a;
      const long long ra = __shfl_sync(0xFFFFFFFFu, er, a) * S;
      const uint32_t won_a = __shfl_sync(0xFFFFFFFFu, won, a);
      const bool in = lane < S && ((won_a >> lane) & 1u);
      const float lw_l = lane < S ? s_lw[lane] : 0.0f;
      // logsumexp of log(w) over the grant
      float lnw_a;
      if (rest_only) {
        lnw_a = __shfl_sync(0xFFFFFFFFu, lnw, a);
      } else {
        const float lmx = warp_max(in ? lw_l : -INFINITY);
        const float lm0 = isinf(lmx) ? 0.0f : lmx;
        lnw_a = fa(logf(ordered_sum(in ? expf(fs(lw_l, lm0)) : 0.0f, won_a)), lm0);
        if (lane == a) lnw = lnw_a;
      }
      if (__shfl_sync(0xFFFFFFFFu, tx_new ? 1 : 0, a)) {
        // ---- link adaptation of a new TB (PHY.select_mcs, phy.py:339-350): the highest MCS <= mcs_max with a TBS
        // whose TB BLER at the EESM SINR (+ OLLA) meets the target, else 0; MCS scanned downward (the first that
        // passes is the highest), the EESM of each with one lane per RBG of lam_a (the grant, or the whole band)
        const uint32_t lam_a = la_band ? band : won_a;
        const bool in_l = lane < S && ((lam_a >> lane) & 1u);
        float lnw_l = lnw_a;
        if (lam_a != won_a) {
          if (rest_only) {
            lnw_l = __shfl_sync(0xFFFFFFFFu, lnw_la, a);
          } else {
            const float lml = warp_max(in_l ? lw_l : -INFINITY);
            const float lm0l = isinf(lml) ? 0.0f : lml;
            lnw_l = fa(logf(ordered_sum(in_l ? expf(fs(lw_l, lm0l)) : 0.0f, lam_a)), lm0l);
          }
        }
        const float split_a = __shfl_sync(0xFFFFFFFFu, split, a);
        const float ref_a = __shfl_sync(0xFFFFFFFFu, ref_pg, a);
        const float off_a = __shfl_sync(0xFFFFFFFFu, p.olla_on ? olla : 0.0f, a);
        const float nprb_a = __shfl_sync(0xFFFFFFFFu, n_prb, a);
        const float lnp_a = __shfl_sync(0xFFFFFFFFu, last_nprb, a);
        const int serv_a = MC ? __shfl_sync(0xFFFFFFFFu, serv, a) : 0;
        const int csrc_a = MC ? __shfl_sync(0xFFFFFFFFu, csi_src, a) : 0;
        float ng = 0.0f;   // -10^(clamp(est, -30, 60) / 10) of this lane's RBG
        if (in_l && !rest_only) {
          const int s = lane;
          const float refs = REF_A(s, ta, ref_a, serv_a);
          const float csi_s = MC ? CSI_A(csrc_a, ra / S, serv_a, s)
                                 : (DL ? st.csi[CK(ra + s, NERS, 5)] : A.gain[CK(g_csi + ra + s, GCAP, 13)]);
          const float est_tx = fa(fs(refs, split_a), csi_s);
          ng = -powf(10.0f, fm(clampf_t(est_tx, -30.0f, 60.0f), 0.1f));
        }
        // this grant's TBS row (the DL: in the table set of this slot's DL data symbols)
        const long long tab0 = DL ? (long long)p.dl_nsym_tab[uls] * (p.nprb + 1) * p.MCS : 0;
        const long long trow_g = tab0 + (long long)(int)nprb_a * p.MCS;
        const long long trow = (p.amc_prev && lnp_a > 0.0f) ? (long long)(int)lnp_a * p.MCS : trow_g;   // MCS row
        // candidates: MCS <= mcs_max with a TBS; the highest first (one lane per RBG), which is the usual outcome;
        // if it fails, every other candidate at once (one lane per MCS) and the highest that passes
        const uint32_t cand = __ballot_sync(0xFFFFFFFFu, lane <= p.mcs_max && lane < p.MCS &&
                                                         A.t.la_tbs[CK(trow + (lane < p.MCS ? lane : 0), NLA, 9)] > 0);
        int chosen = -1;
        if (cand && !rest_only) {
          const int m = 31 - __clz(cand);
          const float beta = s_beta[m];
          const float x = in_l ? fa(x_fdv(ng, beta), lw_l) : -INFINITY;
          const float mx = warp_max(x);
          const float m0 = isinf(mx) ? 0.0f : mx;
          const float lse = fa(logf(ordered_sum(in_l ? expf(fs(x, m0)) : 0.0f, lam_a)), m0);
          const float eff = fa(db_of(fm(-beta, fs(lse, lnw_l))), off_a);
          const float b = bler_lookup(bgrid, m, eff, A.t.la_i0[CK(trow + m, NLA, 9)], A.t.la_wi[CK(trow + m, NLA, 9)]);
          const float tbler = fs(1.0f, powf(fs(1.0f, b), A.t.la_ncb[CK(trow + m, NLA, 9)]));
          if (tbler <= p.target) chosen = m;   // the same value on every lane
        }
        const uint32_t rest = chosen < 0 && cand ? cand & ~(1u << (31 - __clz(cand))) : 0u;
        if (rest) {
          // the grant's -SINR_lin into robot a's column (its rates are done; already there in rest_only mode)
          if (in_l && !rest_only) d_x[lane * NP + ta] = ng;
          __syncwarp();
          bool pass = false;
          if ((rest >> lane) & 1u) {
            const int m = lane;
            const float beta = s_beta[m];
            // x_s of this lane's MCS kept in the warp's columns of the PF-metric rows (free once RBGs are allocated)
            float* const xcol = d_m + wbase + lane;
            float mx = -INFINITY;
            for (uint32_t bb = lam_a; bb; bb &= bb - 1u) {
              const int s = __ffs(bb) - 1;
              const float x = fa(x_fdv(d_x[s * NP + ta], beta), s_lw[s]);
              xcol[s * NP] = x;
              mx = fmaxf(mx, x);
            }
            const float m0 = isinf(mx) ? 0.0f : mx;
            float sum = 0.0f;
            bool first = true;
            for (uint32_t bb = lam_a; bb; bb &= bb - 1u) {
              const int s = __ffs(bb) - 1;
              const float e = expf(fs(xcol[s * NP], m0));
              sum = first ? e : fa(sum, e);
              first = false;
            }
            const float lse = fa(logf(sum), m0);
            const float eff = fa(db_of(fm(-beta, fs(lse, lnw_l))), off_a);
            const float b = bler_lookup(bgrid, m, eff, A.t.la_i0[CK(trow + m, NLA, 9)], A.t.la_wi[CK(trow + m, NLA, 9)]);
            const float tbler = fs(1.0f, powf(fs(1.0f, b), A.t.la_ncb[CK(trow + m, NLA, 9)]));
            pass = tbler <= p.target;
          }
          const uint32_t pm = __ballot_sync(0xFFFFFFFFu, pass);
          chosen = pm ? 31 - __clz(pm) : -1;
          __syncwarp();
        }
        if (lane == a) {
          mcs_new = chosen < 0 ? 0 : chosen;
          tbs_new = A.t.la_tbs[CK(trow_g + mcs_new, NLA, 9)];
        }
      }
    }
    long long cap_b = tbs_new / 8 - p.tb_oh;
    cap_b = cap_b < 1 ? 1 : cap_b;
    const long long byt_new = (BSR && tx_new) ? bsr_tb_payload(st, p, er, enq, sent, cap_b, g)
                                                   : (cap_b < unsent ? cap_b : unsent);
    // ---- bind the TB to its HARQ process (mac.py:406-423)
    const int p_tx = tx_rx ? rx_p : p_new;
    const long long hp = eP + p_tx;
    const long long sent_before = sent;
    if (tx_new) {
      st.h_lo[CK(hp, NERP, 4)] = sent;
      st.h_hi[CK(hp, NERP, 4)] = sent + byt_new;
      st.h_mcs[CK(hp, NERP, 4)] = mcs_new;
      st.h_tbs[CK(hp, NERP, 4)] = tbs_new;
      st.h_nsb[CK(hp, NERP, 4)] = n_sb;
      st.h_ntx[CK(hp, NERP, 4)] = 0;
      st.h_comb[CK(hp, NERP, 4)] = 0.0f;
      st.h_state[CK(hp, NERP, 4)] = 1;
      pend |= 1u << p_tx;
      freem &= ~(1u << p_tx);
      sent += byt_new;
    }
    // ---- several cells: this slot's uplink interference at every gNB from the robots the other cells scheduled on
    // the same RBG (NRNet._ul_ici, nr_engine.py:799-816): PSD after power split and control, the link's fading.  At
    // most one robot per cell holds an RBG, so with C <= 3 every (cell, RBG) sum has at most two non-zero terms and
    // its value does not depend on the order of the shared-memory additions.
    if constexpr (MC) {
      if (lane_dec && tx) {   // each lane its own robot's RBGs (see lane_dec); the sums do not depend on the order
#pragma unroll
        for (int cc = 0; cc < NC; ++cc) {
          if (cc >= C || cc == serv) continue;
          const float psd = fs(fs(fa(pg_c[cc], p.ue_tx), p.ref_db), split);
          for (uint32_t bb = won; bb; bb &= bb - 1u) {
            const int s = __ffs(bb) - 1;
            const float prx = powf(10.0f, fm(fa(psd, A.gain[CK(GIDX(u, er, cc, s), GCAP, 13)]), 0.1f));
            atomicAdd(&s_if[gi][cc][s], prx);
          }
        }
      }
      for (uint32_t tm = lane_dec ? 0u : __ballot_sync(0xFFFFFFFFu, tx); tm; tm &= tm - 1u) {
        const int a = __ffs(tm) - 1;
        const int ta = wbase + a;
        const long long er_a = __shfl_sync(0xFFFFFFFFu, er, a);
        const uint32_t won_a = __shfl_sync(0xFFFFFFFFu, won, a);
        const float split_a = __shfl_sync(0xFFFFFFFFu, split, a);
        const int serv_a = __shfl_sync(0xFFFFFFFFu, serv, a);
        const int gi_a = GW > 32 ? 0 : ta / GW;
        float pga[NC];
#pragma unroll
        for (int cc = 0; cc < NC; ++cc) pga[cc] = __shfl_sync(0xFFFFFFFFu, pg_c[cc], a);
        if (lane < S && ((won_a >> lane) & 1u)) {
          const int s = lane;
#pragma unroll
          for (int cc = 0; cc < NC; ++cc) {
            if (cc >= C || cc == serv_a) continue;
            const float psd = fs(fs(fa(pga[cc], p.ue_tx), p.ref_db), split_a);
            const float prx = powf(10.0f, fm(fa(psd, A.gain[CK(GIDX(u, er_a, cc, s), GCAP, 13)]), 0.1f));
            atomicAdd(&s_if[gi_a][cc][s], prx);
          }
        }
      }
      if constexpr (GW > 32) __syncthreads(); else __syncwarp();
      for (int i = r; i < C * S; i += GW) {
        const int cc = i / S, s = i % S;
        const float ni_now = fa(s_if[gi][cc][s], p.noise_mw);
        s_nadb[gi][cc][s] = fm(10.0f, log10f(ni_now));
        s_ni[gi][cc][s] = p.li_alpha == 1.0f ? ni_now : fa(fm(p.li_alpha, ni_now), fm(p.li_beta, s_ni[gi][cc][s]));
        s_if[gi][cc][s] = 0.0f;
      }
      if constexpr (GW > 32) __syncthreads(); else __syncwarp();
    }
    // ---- decode on the actual channel, HARQ update (mac.py:424-477)
    bool ok = false, fail = false, exh = false;
    long long served = 0;
    int ntx = 0;
    // the TB's HARQ fields: a new TB's from registers (just bound), a retransmission's from its process
    int mcs = mcs_new;
    long long tbs = tbs_new;
    float comb0 = 0.0f;
    long long lo_tx = sent_before, hi_tx = sent_before + byt_new;
    if (tx_new) ntx = 1;
    if (tx_rx) {
      mcs = (int)st.h_mcs[CK(hp, NERP, 4)];
      tbs = st.h_tbs[CK(hp, NERP, 4)];
      ntx = (int)st.h_ntx[CK(hp, NERP, 4)] + 1;
      comb0 = st.h_comb[CK(hp, NERP, 4)];
      lo_tx = st.h_lo[CK(hp, NERP, 4)];
      hi_tx = st.h_hi[CK(hp, NERP, 4)];
    }
    // EESM SINR of the TB's MCS on this row's channel (PHY.eff_sinr, phy.py:311-321): each lane its own robot's (see
    // lane_dec), or one robot at a time with one lane per RBG
    float eff_tx = 0.0f;
    if (lane_dec && tx) {
      const float beta = s_beta[mcs];
      uint32_t kx = 0u;
      for (uint32_t bb = won; bb; bb &= bb - 1u) {
        const int s = __ffs(bb) - 1;
        float a_;
        if constexpr (MC) {   // this slot's interference replaces the N+I the estimate used (nr_engine.py:815)
          a_ = fa(fs(REF(s), split), A.gain[CK(GIDX(u, er, serv, s), GCAP, 13)]);
          a_ = fs(a_, fs(s_nadb[MC ? gi : 0][serv][s], s_nidb[MC ? gi : 0][serv][s]));
        } else {
          a_ = fa(fs(REF(s), split), A.gain[CK(g_gain + er * S + s, GCAP, 13)]);
        }
        const float negl = -powf(10.0f, fm(clampf_t(a_, -30.0f, 60.0f), 0.1f));
        const float x = fa(x_fdv(negl, beta), s_lw[s]);
        v_x[s * NP] = x;   // this thread's column is free once link adaptation is done
        kx = max(kx, fkey(isnan(x) ? -INFINITY : x));
      }
      const float mx = fkey_inv(kx);
      const float m0 = isinf(mx) ? 0.0f : mx;
      float se = 0.0f;
      for (uint32_t bb = won; bb; bb &= bb - 1u) {
        const float ev = expf(fs(v_x[(__ffs(bb) - 1) * NP], m0));
        se = bb == won ? ev : fa(se, ev);
      }
      const float lse = fa(logf(se), m0);
      eff_tx = db_of(fm(-beta, fs(lse, lnw)));
    }
    for (uint32_t tm = lane_dec ? 0u : __ballot_sync(0xFFFFFFFFu, tx); tm; tm &= tm - 1u) {
      const int a = __ffs(tm) - 1;
      const int ta = wbase + a;
      const long long ra = __shfl_sync(0xFFFFFFFFu, er, a) * S;
      const uint32_t won_a = __shfl_sync(0xFFFFFFFFu, won, a);
      const float split_a = __shfl_sync(0xFFFFFFFFu, split, a);
      const float ref_a = __shfl_sync(0xFFFFFFFFu, ref_pg, a);
      const float lnw_a = __shfl_sync(0xFFFFFFFFu, lnw, a);
      const int serv_a = MC ? __shfl_sync(0xFFFFFFFFu, serv, a) : 0;
      const float beta = s_beta[__shfl_sync(0xFFFFFFFFu, mcs, a)];
      const bool in = lane < S && ((won_a >> lane) & 1u);
      float x = -INFINITY;
      if (in) {
        const int s = lane;
        const float refs = REF_A(s, ta, ref_a, serv_a);
        float a_;
        if constexpr (MC) {   // this slot's interference replaces the N+I the estimate used (nr_engine.py:815)
          const int gi_a = GW > 32 ? 0 : ta / GW;
          a_ = fa(fs(refs, split_a), A.gain[CK(GIDX(u, ra / S, serv_a, s), GCAP, 13)]);
          a_ = fs(a_, fs(s_nadb[gi_a][serv_a][s], s_nidb[gi_a][serv_a][s]));
        } else {
          a_ = fa(fs(refs, split_a), A.gain[CK(g_gain + ra + s, GCAP, 13)]);
        }
        const float negl = -powf(10.0f, fm(clampf_t(a_, -30.0f, 60.0f), 0.1f));
        x = fa(x_fdv(negl, beta), s_lw[s]);
      }
      const float mx = warp_max(x);
      const float m0 = isinf(mx) ? 0.0f : mx;
      const float lse = fa(logf(ordered_sum(in ? expf(fs(x, m0)) : 0.0f, won_a)), m0);
      const float eff = db_of(fm(-beta, fs(lse, lnw_a)));
      if (lane == a) eff_tx = eff;
    }
    if (tx) {
      const float eff = eff_tx;
      const float lin = powf(10.0f, fm(eff, 0.1f));
      const float comb = p.comb_cc ? fa(comb0, lin) : lin;
      const float eff_used = fm(10.0f, log10f(clamp_min_t(comb, 1e-9f)));
      float cbs, ncb;
      segment(tbs, s_rate[mcs], cbs, ncb);
      int i0;
      float wi;
      cidx(p, cbs, i0, wi);
      const float b = bler_lookup(bgrid, mcs, eff_used, i0, wi);
      const float p_err = fs(1.0f, powf(fs(1.0f, b), ncb));
      const float u = uniform_at(key_stream(kenv, (uint32_t)(((DL ? SITE_BLER_DL : SITE_BLER_UL) << 16) | rel)),
                                 (uint32_t)r);
      ok = u >= p_err;
      fail = !ok;
      exh = fail && ntx >= p.max_tx;
      // HARQ times (MacLink._harq_times): UL, an ACK frees the process now and a NACK waits ul_rtt; DL
      // (mac_dl.py:47-49), both wait for the HARQ-ACK slot + gnb_proc_slots, an ACKed process in state 2
      const long long r_ack = T * p.N + p.rows_dl[k][2];
      if (ok) {
        pend &= ~(1u << p_tx);
        if constexpr (DL) {
          st.h_state[CK(hp, NERP, 4)] = 2;
          ackm |= 1u << p_tx;
          st.h_ready[CK(hp, NERP, 4)] = r_ack;
        } else {
          st.h_state[CK(hp, NERP, 4)] = 0;
          freem |= 1u << p_tx;
          st.h_ready[CK(hp, NERP, 4)] = g;
        }
      }
      st.h_ntx[CK(hp, NERP, 4)] = ntx;
      st.h_comb[CK(hp, NERP, 4)] = comb;
      if (fail) st.h_ready[CK(hp, NERP, 4)] = DL ? r_ack : g + p.ul_rtt;
      if (exh) {
        if (!p.harq_drop) {
          st.h_ntx[CK(hp, NERP, 4)] = 0;
          st.h_comb[CK(hp, NERP, 4)] = 0.0f;
          st.h_ready[CK(hp, NERP, 4)] = g + p.rlc_retx;
        } else {
          st.h_state[CK(hp, NERP, 4)] = 0;
          pend &= ~(1u << p_tx);
          freem |= 1u << p_tx;
          for (int f = 0; f < F; ++f) {
            const long long at = eF + f;
            if (st.cap[CK(at, NERF, 3)] >= 0 && st.start[CK(at, NERF, 3)] < hi_tx && st.end_[CK(at, NERF, 3)] > lo_tx) {
              if (!st.lost[CK(at, NERF, 3)]) atomicAdd(sc + INB_CTR_LOST_FRAMES, 1ull);
              st.lost[CK(at, NERF, 3)] = 1;
            }
          }
          q_dirty = true;
        }
      }
      served = ok ? hi_tx - lo_tx : 0;
    }
    if (A.trace != nullptr && act) {
      int64_t* tr = A.trace + (((long long)k * p.E + e) * R + r) * 8;
      tr[0] = bsr; tr[1] = need; tr[2] = won; tr[3] = mcs_new;
      tr[4] = (has_rx ? 1 : 0) | (new_el ? 2 : 0) | (tx_rx ? 4 : 0) | (tx_new ? 8 : 0) | (ok ? 16 : 0);
      tr[5] = sent; tr[6] = n_max; tr[7] = (int64_t)__float_as_uint(left);
    }
    // ---- OLLA, BSR and CSI reports, PF average, RR clock (mac.py:478-485, mac_ul.py:221-236, mac.py:534-554)
    if (p.olla_on) {
      const float up = fm(p.olla_up, ok ? 1.0f : 0.0f), dn = fm(p.olla_dn, fail ? 1.0f : 0.0f);
      olla = clampf_t(fs(fa(olla, up), dn), -10.0f, 10.0f);
    }
    if constexpr (BSR) {
      if (act) bsr_post_slot(st, p, er, enq, sent, g, tx, tx_new, tbs_new);
    } else if (!DL && tx) {
      bsr = enq - sent;
    }
    if constexpr (MC) csi_src = u;   // the serving link's gain of this row is the CSI of the next decision
    ++u;
    if (!PFR && !p.pf_freeze) {
      avg = fmaxf(fa(fm(p.pf_a, avg), fm(p.pf_b, (float)served)), 1e-9f);
    } else {   // MacLink._pf_update's other branch (mac.py:545-552)
      const float upd = PFR ? fm((float)(tbs_new / 8), tx_new ? 1.0f : 0.0f) : (float)served;
      const float na = fmaxf(fa(fm(p.pf_a, avg), fm(p.pf_b, upd)), 1e-9f);
      if (!p.pf_freeze || (need > 0 && !has_rx)) avg = na;
    }
    if (p.sched == 2 && tx) last_tx = g;
    if (p.amc_prev && tx) last_nprb = n_prb;   // mac.py:484
    if (tx) {   // counters (only transmitting robots have any to add)
      if (tx_new && p.lena_ctr) {   // grant accounting of the 5G-LENA switches (mac.py:492-493)
        atomicAdd(sc + INB_CTR_TB_BYTES, (unsigned long long)(tbs_new / 8));
        if (byt_new == 0) atomicAdd(sc + INB_CTR_TB_EMPTY, 1ull);
      }
      if (tx_new) {
        atomicAdd(sc + INB_CTR_TB_NEW, 1ull);
        atomicAdd(sc + INB_CTR_BYTES_NEW, (unsigned long long)byt_new);
        if (pending) atomicAdd(sc + INB_CTR_NEW_WHILE_PENDING, 1ull);
      }
      if (tx_rx) atomicAdd(sc + INB_CTR_TB_RETX, 1ull);
      if (ok) {
        atomicAdd(sc + INB_CTR_TB_OK, 1ull);
        atomicAdd(sc + INB_CTR_BYTES_OK, (unsigned long long)served);
      }
      if (fail) atomicAdd(sc + INB_CTR_TB_FAIL, 1ull);
      if (exh) atomicAdd(sc + INB_CTR_EXHAUST, 1ull);
      atomicAdd(sc + INB_CTR_PRB_USED, (unsigned long long)(long long)n_prb);
      int kx = ntx < p.max_tx ? ntx : p.max_tx;
      kx = kx < 15 ? kx : 15;
      atomicAdd(sc + INB_CTR_RV_TX + kx, 1ull);
      if (ok) atomicAdd(sc + INB_CTR_NTX_HIST + kx, 1ull);
      if (fail) atomicAdd(sc + INB_CTR_RV_FAIL + kx, 1ull);
    }
    // ---- RLC in-order delivery (mac.py:499-503): frames are in stream order, so the completed ones are a prefix
    // the in-order pointer never passes `sent`, so a slot with end_scan > sent delivers nothing
    if (act && (q_dirty || end_scan <= sent)) {
#ifdef INB_CHECK
      CK(eP + P - 1, NERP, 12);
#endif
      const long long ack = end_scan <= sent ? ack_ptr(st, eP, pend, sent, floor_) : LLONG_MIN;
      if (end_scan <= ack) {
        const double fin_val = da(da((double)T, x_ddv((double)(rel + 1), (double)p.N)), p.proc_off);
        for (int f = f_scan; f < nvalid; ++f) {
          const long long at = eF + f;
          if (st.end_[CK(at, NERF, 3)] > ack) break;
          if (!st.lost[CK(at, NERF, 3)] && isinf(st.fin[CK(at, NERF, 3)])) st.fin[CK(at, NERF, 3)] = fin_val;
        }
      }
      rescan();
      q_dirty = false;
    }
  }

  // ======================================================================= step state and outputs
  // (the end-of-step queue work runs in the finish kernel, nr_finish.cu)
  if constexpr (MC) {   // A3 triggers after the last scheduled slot of the step (nr_engine.py:781-784)
    if (act && k_ho >= 0 && !fired) handover(T * p.N + k_ho);
  }
  if (M > 0) enq = full_enq;
  if (act) {
    const InbOutputs& o = A.o;
    const long long ob = A.o_base != nullptr ? *A.o_base : 0;
    if constexpr (MC) {
      // serving-link SINR against the gNB's latest N+I, its mean over the RBGs (NRNet.serving_sinr_db,
      // nr_engine.py:709-713); the CSI, association and path gains of every link
      float sum = 0.0f, pg_s = pg_c[0];
#pragma unroll
      for (int cc = 1; cc < NC; ++cc) if (cc == serv) pg_s = pg_c[cc];
      for (int s = 0; s < S; ++s) sum = s == 0 ? s_ni[gi][serv][0] : fa(sum, s_ni[gi][serv][s]);
      const float snr = fs(fs(fa(pg_s, p.ue_tx), p.ref_db), fm(10.0f, log10f(fm(sum, p.inv_S))));
      out_ptr(o.sinr_db, ob)[CK(er, NER, 1)] = snr;
      out_ptr(o.serving_cell, ob)[CK(er, NER, 1)] = serv;
      if (o.pathgain) {
#pragma unroll
        for (int cc = 0; cc < NC; ++cc)
          if (cc < C) out_ptr(o.pathgain, ob)[CK(er * C + cc, NER * C, 1)] = pg_c[cc];
      }
      if (o.blocked) out_ptr(o.blocked, ob)[CK(er, NER, 1)] = (A.rm.blk[CK(er, NER, 1)] >> serv) & 1;
      for (int s = 0; s < S; ++s) st.csi[CK(eS + s, NERS, 5)] = CSI_A(csi_src, er, serv, s);
      st.serv[CK(er, NER, 1)] = serv;
      st.ho_end[CK(er, NER, 1)] = ho_end;
      st.n_ho[CK(er, NER, 1)] = n_ho;
    } else if (!DL) {
      out_ptr(o.sinr_db, ob)[CK(er, NER, 1)] = sinr_obs;
      if (o.serving_cell) out_ptr(o.serving_cell, ob)[CK(er, NER, 1)] = 0;
      if (o.pathgain) out_ptr(o.pathgain, ob)[CK(er, NER, 1)] = pg;
      if (o.blocked) out_ptr(o.blocked, ob)[CK(er, NER, 1)] = A.rm.blk[CK(er, NER, 1)] & 1;
    }
    if (o.los) out_ptr(o.los, ob)[CK(er, NER, 1)] = (uint8_t)p.los_const;
    if (o.gen_accepted) out_ptr(o.gen_accepted, ob)[CK(er, NER, 1)] = n_acc;
    if (o.gen_bytes) out_ptr(o.gen_bytes, ob)[CK(er, NER, 1)] = full_enq - n0;
    st.sent[CK(er, NER, 1)] = sent; st.floor_[CK(er, NER, 1)] = floor_; st.bsr[CK(er, NER, 1)] = bsr; st.sr_t[CK(er, NER, 1)] = sr_t; st.last_tx[CK(er, NER, 1)] = last_tx;
    st.enq[CK(er, NER, 1)] = enq; st.olla[CK(er, NER, 1)] = olla; st.avg[CK(er, NER, 1)] = avg;
    if (p.amc_prev) st.last_nprb[CK(er, NER, 1)] = last_nprb;
  }
#undef REF
  if constexpr (MC) {   // the env's N+I back to memory; the initial association is done
    if constexpr (GW > 32) __syncthreads(); else __syncwarp();
    if (env_ok) {
      for (int i = r; i < C * S; i += GW) A.s.ni_ul[e * C * S + i] = s_ni[gi][i / S][i % S];
      if (r == 0) A.s.pending[e] = 0;
    }
  }
  // counters: one writer per word and env (an env's counter words are shared by its group only)
  if constexpr (GW > 32) {
    __syncthreads();
  } else {
    __syncwarp();
  }
  if (env_ok) {
    int64_t* c = A.ctr + CK(e, p.E, 10) * INB_NCTR;
    for (int i = r; i < INB_NCTR; i += GW)
      if (sc[i]) atomicAdd((unsigned long long*)&c[i], sc[i]);
  }
  // the step's counter-RNG call ends here (the DL instance runs before this one and leaves it alone)
  if (!DL && env_ok && r == 0) A.rng_ctr[CK(e, p.E, 10)] += 1;
#undef CK
}

}  // namespace inb
