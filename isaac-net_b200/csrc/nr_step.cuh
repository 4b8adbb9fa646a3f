// Fused NR uplink control step (sm_100a): traffic enqueue and arrival gate, large-scale radio, the K scheduled slots
// (AR(1) fading, SR, candidate selection, retransmission admission, RBG-by-RBG PF / RR allocation, EESM link
// adaptation, HARQ decode and update, OLLA, PF averages, RLC in-order delivery) and the end-of-step finish (delivery /
// timeout / drop masks, outputs, FIFO compaction) in ONE launch.
//
// Thread mapping: one thread per robot; the R robots of an env form a group of GW lanes (GW = next power of two >= R,
// at least 16).  GW <= 32: 128 / GW envs per 128-thread block, group collectives are segmented warp shuffles.
// GW > 32: one env per block of GW threads, collectives go through shared memory.  Every lane of a group runs the
// same control flow (ghost lanes r >= R and ghost envs e >= E carry neutral values and store nothing), because the
// schedule of a control step is the same for every env.  A branch that holds a collective is taken on a warp-uniform
// condition, so full-mask shuffles are always reached by all 32 lanes at the same call site.
//
// Per-robot per-RBG vectors (fading state, CSI / gain, rate, link-adaptation SINR) live in shared memory, laid out
// [vector][RBG][thread] so a warp touches 32 consecutive words (no bank conflicts); the RBG loops are not unrolled,
// which keeps the kernel small enough for the instruction cache and its register count low.
//
// Semantics follow isaac-net v0.2.0 (file:line in the comments); reductions over the RBG axis are left-to-right sums
// (the oracle's "seq" mode), ties in every argmax resolve to the lowest robot / process index (torch.max / argmin),
// and the retransmission ranking is a stable descending sort.
#pragma once
#include <cfloat>
#include <cmath>
#include <cstdint>

#include "nr_common.cuh"

namespace inb {

struct SmemGroup {
  unsigned long long red[2][4];   // per-warp partial maxima (GW up to 128: 4 warps), double-buffered
  float rkey[128];
  int32_t rnsb[128];
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
  __device__ static bool any(bool v, SmemGroup* sm, int& par) { return max_u64(v ? 1ull : 0ull, sm, par) != 0ull; }
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
  double c = (b <= kcb) ? 1.0 : ceil(ddv(b, dsb(kcb, 24.0)));
  double bp = (c > 1.0) ? da(b, dm(24.0, c)) : b;
  cbs = (float)ddv(bp, c);
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
// x_s = -lin_s / beta + log(w_s) on won RBGs (-inf elsewhere), logsumexp as max + left-to-right sum of exp(x - max),
// eff = -beta (lse - lnw).  negl[s * NT] = -lin_s.
static __device__ __noinline__ float eesm_db(const float* negl, int NT, const float* __restrict__ lw, uint32_t won, int S,
                                      float beta, float lnw) {
  float mx = -INFINITY;
  for (int s = 0; s < S; ++s)
    if ((won >> s) & 1u) mx = fmaxf(mx, fa(fdv(negl[s * NT], beta), lw[s]));
  const float m0 = isinf(mx) ? 0.0f : mx;
  float sum = 0.0f;
  for (int s = 0; s < S; ++s) {
    float e = ((won >> s) & 1u) ? expf(fs(fa(fdv(negl[s * NT], beta), lw[s]), m0)) : 0.0f;
    sum = s == 0 ? e : fa(sum, e);
  }
  const float lse = fa(logf(sum), m0);
  return db_of(fm(-beta, fs(lse, lnw)));
}

// logsumexp of log(w) over the won RBGs (the EESM normalization)
__device__ __forceinline__ float lnw_of(const float* __restrict__ lw, uint32_t won, int S) {
  float mx = -INFINITY;
  for (int s = 0; s < S; ++s)
    if ((won >> s) & 1u) mx = fmaxf(mx, lw[s]);
  const float m0 = isinf(mx) ? 0.0f : mx;
  float sum = 0.0f;
  for (int s = 0; s < S; ++s) {
    float e = ((won >> s) & 1u) ? expf(fs(lw[s], m0)) : 0.0f;
    sum = s == 0 ? e : fa(sum, e);
  }
  return fa(logf(sum), m0);
}

// the in-order pointer: lowest byte still owned by an undecoded process, or `sent` (MacLink.ack_ptr, mac.py:194-197)
__device__ __forceinline__ long long ack_ptr(const InbState& st, long long eP, int P, long long sent, long long floor_) {
  long long ack = sent;
  for (int q = 0; q < P; ++q) {
    if (st.h_state[eP + q] == 1) {
      const long long hh = st.h_hi[eP + q];
      if (hh > floor_) {
        long long ll = st.h_lo[eP + q];
        ll = ll > floor_ ? ll : floor_;
        ack = ll < ack ? ll : ack;
      }
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
template <int GW>
__global__ void __launch_bounds__(GW > 32 ? GW : 128, GW > 32 ? 512 / GW : 4) nr_step_kernel(const InbStepArgs A) {
  constexpr int NT = GW > 32 ? GW : 128;
  const InbParams& p = A.p;
  __shared__ SmemGroup smem_all[GW > 32 ? 1 : 128 / GW];
  __shared__ float s_lw[INB_MAX_S], s_lw10[INB_MAX_S], s_w[INB_MAX_S];
  __shared__ float s_thr[INB_MAX_MCS], s_se[INB_MAX_MCS], s_beta[INB_MAX_MCS], s_rate[INB_MAX_MCS];
  extern __shared__ float dyn[];   // [5 or 6][S][NT]: hr, hi, csi/gain ping-pong (2), rate / -lin, ref (optional)
  const int tid = threadIdx.x;
  const int gpb = GW > 32 ? 1 : 128 / GW;
  const int gi = GW > 32 ? 0 : tid / GW;
  const int r = GW > 32 ? tid : tid % GW;
  SmemGroup* sm = &smem_all[gi];
  const long long e = (long long)blockIdx.x * gpb + gi;
  const int R = p.R, S = p.S, P = p.P, F = p.F;
  const bool env_ok = e < p.E;
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
  float* v_hr = dyn + tid;
  float* v_hi = dyn + (size_t)S * NT + tid;
  float* v_cg0 = dyn + (size_t)2 * S * NT + tid;
  float* v_cg1 = dyn + (size_t)3 * S * NT + tid;
  float* v_x = dyn + (size_t)4 * S * NT + tid;
  float* v_ref = dyn + (size_t)5 * S * NT + tid;
  const bool ref_vec = A.ul_ref_in != nullptr;
  __syncthreads();

  const long long er = act ? e * R + r : 0;
  const long long eP = er * P, eF = er * F, eS = er * S;
  const InbState& st = A.s;
  const long long T = (A.T_dev != nullptr) ? *A.T_dev : p.T;
#ifdef INB_CHECK
  const long long NER = (long long)p.E * R, NERF = NER * F, NERP = NER * P, NERS = NER * S, NERM = NER * p.M;
  const long long NFK = (long long)p.E * p.Kf, NLA = (long long)(p.nprb + 1) * p.MCS;
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
  const long long epoch = env_ok ? A.epoch[CK(e, p.E, 10)] : 0;
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
    for (int f = 0; f < F; ++f) cnt_q += st.cap[CK(eF + f, NERF, 3)] >= 0 ? 1 : 0;
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
        st.cls[CK(at, NERF, 3)] = 0;
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

  // ---------------- large-scale radio: path gain of the serving link (one cell)
  float pg = 0.0f;
  if (act) {
    if (A.pathgain_in != nullptr) {
      pg = A.pathgain_in[CK(er, NER, 1)];
    } else if (A.pos != nullptr) {
      const float px = A.pos[CK(er * 2, NER * 2, 2)], py = A.pos[CK(er * 2 + 1, NER * 2, 2)];
      const float dx = fs(px, A.t.gnb[0]), dy = fs(py, A.t.gnb[1]);
      const float d2 = fmaxf(sqrtf(fa(fm(dx, dx), fm(dy, dy))), 1.0f);
      // shadowing: amp * sum_k cos(k . x + phi) (channels/fields.py:61-64), the field of (env, cell 0)
      float cs = 0.0f;
      for (int k = 0; k < p.Kf; ++k) {
        const long long fo = e * p.Kf + k;
        const float arg = fa(fa(fm(px, A.t.fk[CK(fo * 2, NFK * 2, 8)]), fm(py, A.t.fk[CK(fo * 2 + 1, NFK * 2, 8)])), A.t.fphi[CK(fo, NFK, 8)]);
        const float c = cosf(arg);
        cs = k == 0 ? c : fa(cs, c);
      }
      const float field = fm(p.amp, cs);
      if (p.radio_model <= 1) {
        // TR 38.901 UMi / UMa LOS path loss (channels/tr38901.py:148-170) + sigma_SF * unit field
        const float d3 = sqrtf(fa(fm(d2, d2), p.hh2));
        const float lg = log10f(d3);
        const float pl = (d2 <= p.dbp) ? fa(fa(p.pl_a, fm(p.pl_n1, lg)), p.fc_term)
                                       : fs(fa(fa(p.pl_a, fm(40.0f, lg)), p.fc_term), p.pl_b_term);
        const float rx = fa(p.ue_tx, -fa(pl, fm(p.sigma_sf, field)));
        pg = fs(rx, p.ue_tx);
      } else {
        // log-distance (radio.py:265-273)
        const float pl = fa(p.pl_const, fm(p.pl_10n, log10f(d2)));
        pg = fs(fs(fs(p.ue_tx, pl), field), p.ue_tx);
      }
    }
  }
  // ul_ref = ue_tx - 10 log10(snr_ref_prbs) + pg - N_prb (NRNet.step_rx, nr_engine.py:613-632)
  const float ref_pg = fs(fa(p.ul_ref0, pg), p.noise_prb);
  const float sinr_obs = fs(fa(pg, p.ue_tx), p.sub_noise);
  if (ref_vec) {
    for (int s = 0; s < S; ++s) v_ref[s * NT] = act ? A.ul_ref_in[CK(eS + s, NERS, 5)] : 0.0f;
  }
#define REF(s) (ref_vec ? v_ref[(s) * NT] : ref_pg)

  // ---------------- fading state and CSI into shared memory
  for (int s = 0; s < S; ++s) {
    float a = 0.0f, b = 0.0f, c = 0.0f;
    if (act) {
      a = st.h[CK((eS + s) * 2, NERS * 2, 6)];
      b = st.h[CK((eS + s) * 2 + 1, NERS * 2, 6)];
      c = st.csi[CK(eS + s, NERS, 5)];
    }
    v_hr[s * NT] = a;
    v_hi[s * NT] = b;
    v_cg0[s * NT] = c;
  }
  float* csi = v_cg0;   // CSI of the previous PUSCH
  float* gain = v_cg1;  // fading gain of this slot
  float kb = 1.0f, ar_ = 0.0f, ai_ = 0.0f;
  if (p.rician && act) {
    // |sqrt(K/(K+1)) e^{j phi} + sqrt(1/(K+1)) h|^2 (NRNet._gain, nr_engine.py:602-611)
    const float k_lin = st.k_lin[CK(er, NER, 1)];
    const float kinv = fdv(1.0f, fa(k_lin, 1.0f));
    const float ka = sqrtf(fm(k_lin, kinv));
    kb = sqrtf(kinv);
    ar_ = fm(ka, st.spec[CK(er * 2, NER * 2, 2)]);
    ai_ = fm(ka, st.spec[CK(er * 2 + 1, NER * 2, 2)]);
  }
  // PHR cap n_max = floor(snr_ref_prbs * 10^((mean(ul_ref) - phr_min) / 10) / w[0]).clamp(1, S) (mac_ul.py:165-168),
  // the mean as a left-to-right sum times float32(1 / S)
  int n_max = S;
  if (p.phr_cap) {
    float sum = 0.0f;
    for (int s = 0; s < S; ++s) sum = s == 0 ? REF(0) : fa(sum, REF(s));
    const float x = fm(fs(fm(sum, p.inv_S), p.phr_min), 0.1f);
    const float nmp = fm((float)p.ref_prbs, powf(10.0f, x));
    n_max = (int)clampf_t(floorf(fdv(nmp, s_w[0])), 1.0f, (float)S);
  }

  const uint32_t kenv = env_ok ? key_env(p.s0, A.env_id[CK(e, p.E, 10)], A.episode[CK(e, p.E, 10)], CH_STEP, A.rng_ctr[CK(e, p.E, 10)]) : 0u;
  const float two_pi = 6.28318548202514648438f;
  const bool thr_mono = p.thr_mono != 0;
  const BlerGrid bgrid = {A.t.bler, p.C_axis, p.G_axis, p.MCS, p.s0_snr, p.inv_ds, A.status};

  long long c_v[10];
#pragma unroll
  for (int i = 0; i < 10; ++i) c_v[i] = 0;
  int c_hist[3][16];
#pragma unroll
  for (int i = 0; i < 16; ++i) { c_hist[0][i] = 0; c_hist[1][i] = 0; c_hist[2][i] = 0; }

  // first frame not yet finished (RLC scan start); frames are in stream order
  const int nvalid = cnt_q;
  int f_scan = 0;
  if (act) {
    while (f_scan < nvalid && (st.lost[CK(eF + f_scan, NERF, 3)] != 0 || !isinf(st.fin[CK(eF + f_scan, NERF, 3)]))) ++f_scan;
  }

  // ======================================================================= slot loop (nr_engine.py:656-667)
  for (int k = 0; k < p.K_rows; ++k) {
    const int rel = p.rows[k][0], uls = p.rows[k][1], srf = p.rows[k][2], fad = p.rows[k][3];
    const long long g = T * p.N + rel;
    // ---- AR(1) fading step and gain (NRNet._evolve / _gain, nr_engine.py:570-611)
    if (p.fading) {
      const uint32_t base_f = key_stream(kenv, (uint32_t)((SITE_FADING << 16) | rel));
      const float rho = p.rowf[k][0], c1 = p.rowf[k][1];
#pragma unroll 1
      for (int s = 0; s < S; ++s) {
        float hr = v_hr[s * NT], hi = v_hi[s * NT];
        if (fad) {
          const uint32_t j = (uint32_t)((r * S + s) * 2);
          const float zr = normal_at(base_f, j, two_pi);
          const float zi = normal_at(base_f, j + 1u, two_pi);
          hr = fa(fm(rho, hr), fm(fm(c1, zr), p.inv_sqrt2));
          hi = fa(fm(rho, hi), fm(fm(c1, zi), p.inv_sqrt2));
          v_hr[s * NT] = hr;
          v_hi[s * NT] = hi;
        }
        float pw;
        if (p.rician) {
          const float xr = fa(ar_, fm(kb, hr)), xi = fa(ai_, fm(kb, hi));
          pw = fa(fm(xr, xr), fm(xi, xi));
        } else {
          pw = fa(fm(hr, hr), fm(hi, hi));
        }
        gain[s * NT] = fm(10.0f, log10f(clamp_min_t(pw, 1e-6f)));
      }
    } else {
      for (int s = 0; s < S; ++s) gain[s * NT] = 0.0f;
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
    // ---- SR (UlMac.sr_step, mac_ul.py:66-71)
    if (srf && (enq - sent > 0) && bsr <= 0 && sr_t < 0) sr_t = g;
    if (!uls) continue;

    // =================================================================== UL data slot (MacLink.slot, mac.py:228-508)
    const long long unsent = enq - sent;
    // lumped SR grant (mac_ul.py:140-147)
    if (sr_t >= 0 && g - sr_t >= p.sr_delay) {
      bsr = bsr < 1 ? 1 : bsr;
      sr_t = -1;
    }
    // candidates: earliest ready NACKed process, else the first free one (mac.py:241-253)
    int rx_p = 0, p_new = -1;
    long long best_ready = BIGI;
    bool has_rx = false, pending = false;
    if (act) {
      for (int q = 0; q < P; ++q) {
        const long long hs = st.h_state[CK(eP + q, NERP, 4)];
        if (hs == 1) {
          pending = true;
          const long long rd = st.h_ready[CK(eP + q, NERP, 4)];
          if (rd <= g) {
            has_rx = true;
            if (rd < best_ready) { best_ready = rd; rx_p = q; }
          }
        } else if (hs == 0 && p_new < 0) {
          p_new = q;
        }
      }
    }
    const bool any_free = p_new >= 0;
    if (p_new < 0) p_new = 0;
    const long long need = bsr < unsent ? bsr : unsent;
    const bool new_el = act && any_free && need > 0 && !has_rx;
    const int rx_nsb = act ? (int)st.h_nsb[CK(eP + rx_p, NERP, 4)] : 0;
    // scheduler estimate with OLLA -> rate (bytes per RBG) (mac.py:255-266, mac_ul.py:154-171)
    const float re_prb = (float)min(12 * uls - p.dmrs - p.oh, 156);
    float* rate = v_x;
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
      const float est = fa(fs(REF(s), s_lw10[s]), csi[s * NT]);
      const float eo = p.olla_on ? fa(est, olla) : fa(est, 0.0f);
      const int m = mcs_at(s_thr, p.mcs_max, thr_mono, eo);
      rate[s * NT] = fm(fm(fm(s_se[m], re_prb), s_w[s]), 0.125f);
    }
    // scheduler metric per RBG: PF rate / avg, maxCI rate, RR slot age (mac.py:267-275)
    const float avg_den = fmaxf(avg, 1e-9f);
    const float rr_metric = (float)(g - last_tx);
#define METRIC(s) (p.sched == 2 ? rr_metric : (p.sched == 1 ? rate[(s) * NT] : fdv(rate[(s) * NT], avg_den)))
    // retransmission admission: rank by metric sum (stable, descending), admit while RBG counts fit (mac.py:300-312)
    if (Grp<GW>::any_uniform(has_rx, sm, par)) {
      float rkey = -1.0f;
      if (has_rx) {
        float sum = 0.0f;
        for (int s = 0; s < S; ++s) sum = s == 0 ? METRIC(0) : fa(sum, METRIC(s));
        rkey = sum;
      }
      const int mine = has_rx ? rx_nsb : 0;
      int before = 0;
      if constexpr (GW <= 32) {
        for (int j = 0; j < GW; ++j) {
          const float kj = __shfl_sync(0xFFFFFFFFu, rkey, j, GW);
          const int nj = __shfl_sync(0xFFFFFFFFu, mine, j, GW);
          if (kj > rkey || (kj == rkey && j < r)) before += nj;
        }
      } else {
        sm->rkey[r] = rkey;
        sm->rnsb[r] = mine;
        __syncthreads();
        for (int j = 0; j < GW; ++j) {
          const float kj = sm->rkey[j];
          if (kj > rkey || (kj == rkey && j < r)) before += sm->rnsb[j];
        }
        __syncthreads();
      }
      has_rx = has_rx && (before + mine <= S);
    }
    const int want_cnt = has_rx ? rx_nsb : (new_el ? n_max : 0);
    const bool lex = p.retx_priority != 0;
    const float prio = lex ? fm(1e9f, has_rx ? 1.0f : 0.0f) : 0.0f;
    // greedy allocation RBG by RBG (mac.py:322-351); key = (retx wanting, metric + prio, lowest robot)
    uint32_t won = 0u;
    int cnt = 0;
    float left = (float)need;
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
      const bool want = act && (cnt < want_cnt) && (has_rx || left > 0.0f);
      const float mkey = want ? fa(METRIC(s), prio) : -1.0f;
      const bool wr = lex && want && has_rx;
      const unsigned long long key = ((unsigned long long)(wr ? 1u : 0u) << 40) |
                                     ((unsigned long long)fkey(mkey) << 8) | (unsigned long long)(255 - r);
      const unsigned long long mx = Grp<GW>::max_u64(key, sm, par);
      const bool oh = (255 - (int)(mx & 0xFFull) == r) && (fkey_inv((uint32_t)((mx >> 8) & 0xFFFFFFFFull)) >= 0.0f);
      if (oh) {
        won |= 1u << s;
        cnt += 1;
      }
      left = fs(left, fm(fm(rate[s * NT], oh ? 1.0f : 0.0f), has_rx ? 0.0f : 1.0f));
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
        const float mkey = want ? METRIC(s) : -1.0f;
        const unsigned long long key = ((unsigned long long)fkey(mkey) << 8) | (unsigned long long)(255 - r);
        const unsigned long long mx = Grp<GW>::max_u64(key, sm, par);
        const bool av = Grp<GW>::any(((rel_rs >> s) & 1u) != 0u, sm, par);
        const bool oh = (255 - (int)(mx & 0xFFull) == r) &&
                        (fkey_inv((uint32_t)((mx >> 8) & 0xFFFFFFFFull)) >= 0.0f) && av;
        if (oh) {
          won |= 1u << s;
          cnt += 1;
        }
        left = fs(left, fm(rate[s * NT], oh ? 1.0f : 0.0f));
      }
    }
#undef METRIC
    const int n_sb = __popc(won);
    float n_prb = 0.0f;
    for (int s = 0; s < S; ++s)
      if ((won >> s) & 1u) n_prb = fa(n_prb, s_w[s]);
    const bool tx_rx = has_rx && (n_sb == rx_nsb) && (n_sb > 0);
    const bool tx_new = new_el && (n_sb > 0);
    const bool tx = tx_rx || tx_new;
    // power split over the grant (UlMac._split, mac_ul.py:173-180)
    const float split = fm(10.0f, log10f(clamp_min_t(fm(n_prb, p.inv_ref_prbs), 1e-3f)));
    float* negl = v_x;    // -10^(clamp(sinr, -30, 60) / 10) per RBG (the rates are no longer needed)
    const float lnw = tx ? lnw_of(s_lw, won, S) : 0.0f;
    // ---- link adaptation of a new TB (PHY.select_mcs, phy.py:339-350): highest passing MCS, scanned downward
    int mcs_new = 0;
    long long tbs_new = 0;
    if (tx_new) {
      const long long trow = (long long)(int)n_prb * p.MCS;
      for (int s = 0; s < S; ++s) {
        const float est_tx = fa(fs(REF(s), split), csi[s * NT]);
        negl[s * NT] = -powf(10.0f, fm(clampf_t(est_tx, -30.0f, 60.0f), 0.1f));
      }
      const float off = p.olla_on ? olla : 0.0f;
      int chosen = -1;
      for (int m = p.mcs_max; m >= 0; --m) {
        if (A.t.la_tbs[CK(trow + m, NLA, 9)] <= 0) continue;
        const float eff = fa(eesm_db(negl, NT, s_lw, won, S, s_beta[m], lnw), off);
        const float b = bler_lookup(bgrid, m, eff, A.t.la_i0[CK(trow + m, NLA, 9)], A.t.la_wi[CK(trow + m, NLA, 9)]);
        const float tbler = fs(1.0f, powf(fs(1.0f, b), A.t.la_ncb[CK(trow + m, NLA, 9)]));
        if (tbler <= p.target) { chosen = m; break; }
      }
      mcs_new = chosen < 0 ? 0 : chosen;
      tbs_new = A.t.la_tbs[CK(trow + mcs_new, NLA, 9)];
    }
    long long cap_b = tbs_new / 8 - p.tb_oh;
    cap_b = cap_b < 1 ? 1 : cap_b;
    const long long byt_new = cap_b < unsent ? cap_b : unsent;
    // ---- bind the TB to its HARQ process (mac.py:406-423)
    const int p_tx = tx_rx ? rx_p : p_new;
    const long long hp = eP + p_tx;
    if (tx_new) {
      st.h_lo[CK(hp, NERP, 4)] = sent;
      st.h_hi[CK(hp, NERP, 4)] = sent + byt_new;
      st.h_mcs[CK(hp, NERP, 4)] = mcs_new;
      st.h_tbs[CK(hp, NERP, 4)] = tbs_new;
      st.h_nsb[CK(hp, NERP, 4)] = n_sb;
      st.h_ntx[CK(hp, NERP, 4)] = 0;
      st.h_comb[CK(hp, NERP, 4)] = 0.0f;
      st.h_state[CK(hp, NERP, 4)] = 1;
      sent += byt_new;
    }
    // ---- decode on the actual channel, HARQ update (mac.py:424-477)
    bool ok = false, fail = false, exh = false;
    long long served = 0;
    int ntx = 0;
    if (tx) {
      const int mcs = (int)st.h_mcs[CK(hp, NERP, 4)];
      const long long tbs = st.h_tbs[CK(hp, NERP, 4)];
      ntx = (int)st.h_ntx[CK(hp, NERP, 4)] + 1;
      for (int s = 0; s < S; ++s) {
        const float a_ = fa(fs(REF(s), split), gain[s * NT]);
        negl[s * NT] = -powf(10.0f, fm(clampf_t(a_, -30.0f, 60.0f), 0.1f));
      }
      const float eff = eesm_db(negl, NT, s_lw, won, S, s_beta[mcs], lnw);
      const float lin = powf(10.0f, fm(eff, 0.1f));
      const float comb = p.comb_cc ? fa(st.h_comb[CK(hp, NERP, 4)], lin) : lin;
      const float eff_used = fm(10.0f, log10f(clamp_min_t(comb, 1e-9f)));
      float cbs, ncb;
      segment(tbs, s_rate[mcs], cbs, ncb);
      int i0;
      float wi;
      cidx(p, cbs, i0, wi);
      const float b = bler_lookup(bgrid, mcs, eff_used, i0, wi);
      const float p_err = fs(1.0f, powf(fs(1.0f, b), ncb));
      const float u = uniform_at(key_stream(kenv, (uint32_t)((SITE_BLER_UL << 16) | rel)), (uint32_t)r);
      ok = u >= p_err;
      fail = !ok;
      exh = fail && ntx >= p.max_tx;
      if (ok) {
        st.h_state[CK(hp, NERP, 4)] = 0;
        st.h_ready[CK(hp, NERP, 4)] = g;
      }
      st.h_ntx[CK(hp, NERP, 4)] = ntx;
      st.h_comb[CK(hp, NERP, 4)] = comb;
      if (fail) st.h_ready[CK(hp, NERP, 4)] = g + p.ul_rtt;
      const long long lo_tx = st.h_lo[CK(hp, NERP, 4)], hi_tx = st.h_hi[CK(hp, NERP, 4)];
      if (exh) {
        if (!p.harq_drop) {
          st.h_ntx[CK(hp, NERP, 4)] = 0;
          st.h_comb[CK(hp, NERP, 4)] = 0.0f;
          st.h_ready[CK(hp, NERP, 4)] = g + p.rlc_retx;
        } else {
          st.h_state[CK(hp, NERP, 4)] = 0;
          for (int f = 0; f < F; ++f) {
            const long long at = eF + f;
            if (st.cap[CK(at, NERF, 3)] >= 0 && st.start[CK(at, NERF, 3)] < hi_tx && st.end_[CK(at, NERF, 3)] > lo_tx) {
              if (!st.lost[CK(at, NERF, 3)]) c_v[9] += 1;
              st.lost[CK(at, NERF, 3)] = 1;
            }
          }
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
    if (tx) bsr = enq - sent;
    {
      float* t_ = csi;    // the gain of this slot is the CSI of the next decision
      csi = gain;
      gain = t_;
    }
    avg = fmaxf(fa(fm(p.pf_a, avg), fm(p.pf_b, (float)served)), 1e-9f);
    if (p.sched == 2 && tx) last_tx = g;
    if (act) {
      c_v[0] += tx_new; c_v[1] += tx_rx; c_v[2] += ok; c_v[3] += fail; c_v[4] += exh;
      c_v[5] += served; c_v[6] += tx_new ? byt_new : 0; c_v[7] += (tx_new && pending);
      c_v[8] += tx ? (long long)n_prb : 0;
      if (tx) {
        int kx = ntx < p.max_tx ? ntx : p.max_tx;
        kx = kx < 15 ? kx : 15;
        c_hist[1][kx] += 1;
        if (ok) c_hist[0][kx] += 1;
        if (fail) c_hist[2][kx] += 1;
      }
    }
    // ---- RLC in-order delivery (mac.py:499-503): frames are in stream order, so the completed ones are a prefix
    if (act) {
      CK(eP + P - 1, NERP, 12);
      const long long ack = ack_ptr(st, eP, P, sent, floor_);
      const double fin_val = da(da((double)T, ddv((double)(rel + 1), (double)p.N)), p.proc_off);
      for (int f = f_scan; f < nvalid; ++f) {
        const long long at = eF + f;
        if (st.end_[CK(at, NERF, 3)] > ack) break;
        if (!st.lost[CK(at, NERF, 3)] && isinf(st.fin[CK(at, NERF, 3)])) st.fin[CK(at, NERF, 3)] = fin_val;
      }
      while (f_scan < nvalid && (st.lost[CK(eF + f_scan, NERF, 3)] != 0 || !isinf(st.fin[CK(eF + f_scan, NERF, 3)]))) ++f_scan;
    }
  }

  // ======================================================================= finish (nr_engine.py:843-888)
  if (M > 0) enq = full_enq;
  bool det_hit = false;
  if (act) {
    const InbOutputs& o = A.o;
    const long long ack_end = ack_ptr(st, eP, P, sent, floor_);
    const double lim = da((double)(T + 1), 1e-9);
    long long newest = -1;
    uint64_t gone_mask = 0ull;
    for (int f = 0; f < F; ++f) {
      const long long at = eF + f;
      const long long cap = st.cap[CK(at, NERF, 3)];
      const bool valid = cap >= 0;
      const double fin = st.fin[CK(at, NERF, 3)];
      const bool delivered = valid && fin <= lim;
      const bool timed = p.purge && valid && isinf(fin) && ((T + 1 - cap) >= p.timeout);
      const bool dropped = valid && st.lost[CK(at, NERF, 3)] && (st.end_[CK(at, NERF, 3)] <= ack_end) && !timed;
      if (delivered && cap > newest) newest = cap;
      if (delivered && st.det[CK(at, NERF, 3)] && st.hid[CK(at, NERF, 3)] == last_hid) det_hit = true;
      const double off = st.off[CK(at, NERF, 3)];
      o.delivered[CK(at, NERF, 3)] = delivered;
      o.timed_out[CK(at, NERF, 3)] = timed;
      o.dropped[CK(at, NERF, 3)] = dropped;
      o.cap[CK(at, NERF, 3)] = valid ? cap - epoch : -1;
      o.cls[CK(at, NERF, 3)] = valid ? st.cls[CK(at, NERF, 3)] : 0;
      const float delay = (float)dsb(dsb(fin, (double)cap), off);
      o.delay[CK(at, NERF, 3)] = delivered ? delay : NAN;
      o.arrival[CK(at, NERF, 3)] = valid ? da((double)(cap - epoch), off) : NAN;
      o.arrival_slot[CK(at, NERF, 3)] = valid ? (long long)rint(dm(off, (double)p.N)) : -1;
      o.tag[CK(at, NERF, 3)] = valid ? st.tag[CK(at, NERF, 3)] : 0;
      o.priority[CK(at, NERF, 3)] = valid ? st.prio[CK(at, NERF, 3)] : 0;
      o.bytes[CK(at, NERF, 3)] = valid ? st.end_[CK(at, NERF, 3)] - st.start[CK(at, NERF, 3)] : 0;
      const double dl = st.dline[CK(at, NERF, 3)];
      const bool late = delivered && (dm((double)delay, p.ctl_ms) > dl);
      o.deadline_miss[CK(at, NERF, 3)] = late || ((timed || dropped) && isfinite(dl));
      if (delivered || timed || dropped || !valid) gone_mask |= 1ull << f;
    }
    // compaction: surviving frames first (stable), then the freed slots in index order (queues.py:105-110)
    int order[INB_MAX_F];
    int n_keep = 0;
    for (int f = 0; f < F; ++f)
      if (!((gone_mask >> f) & 1ull)) order[n_keep++] = f;
    {
      int n = n_keep;
      for (int f = 0; f < F; ++f)
        if ((gone_mask >> f) & 1ull) order[n++] = f;
    }
    if (gone_mask != ((F >= 64) ? ~0ull : ((1ull << F) - 1ull)) || n_keep > 0) {
      auto perm64 = [&](int64_t* a, bool is_cap) {
        long long tmp[INB_MAX_F];
        for (int f = 0; f < F; ++f) {
          const int src = order[f];
          tmp[f] = (is_cap && ((gone_mask >> src) & 1ull)) ? -1 : a[CK(eF + src, NERF, 3)];
        }
        for (int f = 0; f < F; ++f) a[CK(eF + f, NERF, 3)] = tmp[f];
      };
      auto permd = [&](double* a) {
        double tmp[INB_MAX_F];
        for (int f = 0; f < F; ++f) tmp[f] = a[CK(eF + order[f], NERF, 3)];
        for (int f = 0; f < F; ++f) a[CK(eF + f, NERF, 3)] = tmp[f];
      };
      auto perm8 = [&](uint8_t* a) {
        uint8_t tmp[INB_MAX_F];
        for (int f = 0; f < F; ++f) tmp[f] = a[CK(eF + order[f], NERF, 3)];
        for (int f = 0; f < F; ++f) a[CK(eF + f, NERF, 3)] = tmp[f];
      };
      perm64(st.cap, true);
      perm64(st.start, false); perm64(st.end_, false); perm64(st.cls, false); perm64(st.hid, false);
      perm64(st.tag, false); perm64(st.prio, false);
      perm8(st.lost); perm8(st.det);
      permd(st.fin); permd(st.off); permd(st.dline);
    } else {
      for (int f = 0; f < F; ++f) st.cap[CK(eF + f, NERF, 3)] = -1;
    }
    // stream floor, send pointer, HARQ processes holding only purged bytes (MacLink.compact, mac.py:598-616)
    floor_ = n_keep > 0 ? st.start[CK(eF, NERF, 3)] : enq;
    sent = sent > floor_ ? sent : floor_;
    for (int q = 0; q < P; ++q) {
      const long long hq = eP + q;
      if (st.h_state[CK(hq, NERP, 4)] == 1 && st.h_hi[CK(hq, NERP, 4)] <= floor_ && st.h_hi[CK(hq, NERP, 4)] > st.h_lo[CK(hq, NERP, 4)]) {
        st.h_state[CK(hq, NERP, 4)] = 0; st.h_ready[CK(hq, NERP, 4)] = 0; st.h_ntx[CK(hq, NERP, 4)] = 0; st.h_comb[CK(hq, NERP, 4)] = 0.0f;
      }
    }
    bsr = bsr < enq - sent ? bsr : enq - sent;
    const long long qb = enq - ack_ptr(st, eP, P, sent, floor_);
    o.newest[CK(er, NER, 1)] = newest >= 0 ? newest - epoch : -1;
    o.queue_len[CK(er, NER, 1)] = n_keep;
    o.queue_bytes[CK(er, NER, 1)] = (float)(qb > 0 ? qb : 0);
    o.sinr_db[CK(er, NER, 1)] = sinr_obs;
    if (o.pathgain) o.pathgain[CK(er, NER, 1)] = pg;
    o.gen_accepted[CK(er, NER, 1)] = n_acc;
    o.gen_bytes[CK(er, NER, 1)] = full_enq - n0;
    // ---- state back to memory
    st.sent[CK(er, NER, 1)] = sent; st.floor_[CK(er, NER, 1)] = floor_; st.bsr[CK(er, NER, 1)] = bsr; st.sr_t[CK(er, NER, 1)] = sr_t; st.last_tx[CK(er, NER, 1)] = last_tx;
    st.enq[CK(er, NER, 1)] = enq; st.olla[CK(er, NER, 1)] = olla; st.avg[CK(er, NER, 1)] = avg;
    for (int s = 0; s < S; ++s) {
      st.csi[CK(eS + s, NERS, 5)] = csi[s * NT];
      st.h[CK((eS + s) * 2, NERS * 2, 6)] = v_hr[s * NT];
      st.h[CK((eS + s) * 2 + 1, NERS * 2, 6)] = v_hi[s * NT];
    }
  }
#undef REF
  // det_env and counters: group reductions, then one writer per group
  const bool det_any = Grp<GW>::any(det_hit, sm, par);
  if (env_ok && r == 0) A.o.det_env[CK(e, p.E, 10)] = det_any ? 1 : 0;
  if (act) {
    int64_t* c = A.ctr + CK(e, p.E, 10) * INB_NCTR;
#pragma unroll
    for (int i = 0; i < 10; ++i)
      if (c_v[i]) atomicAdd((unsigned long long*)&c[i], (unsigned long long)c_v[i]);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (c_hist[0][i]) atomicAdd((unsigned long long*)&c[INB_CTR_NTX_HIST + i], (unsigned long long)c_hist[0][i]);
      if (c_hist[1][i]) atomicAdd((unsigned long long*)&c[INB_CTR_RV_TX + i], (unsigned long long)c_hist[1][i]);
      if (c_hist[2][i]) atomicAdd((unsigned long long*)&c[INB_CTR_RV_FAIL + i], (unsigned long long)c_hist[2][i]);
    }
  }
  if (env_ok && r == 0) A.rng_ctr[CK(e, p.E, 10)] += 1;
#undef CK
}

}  // namespace inb
