// Fused NR uplink control step (sm_100a): traffic enqueue and arrival gate, large-scale radio, the K scheduled slots
// (AR(1) fading, SR, candidate selection, retransmission admission, RBG-by-RBG PF / RR allocation, EESM link
// adaptation, HARQ decode and update, OLLA, PF averages, RLC in-order delivery) and the end-of-step finish (delivery /
// timeout / drop masks, outputs, FIFO compaction) in ONE launch.
//
// Thread mapping: one thread per robot; the R robots of an env form a group of GW lanes (GW = next power of two >= R,
// at least 16).  GW <= 32: 128 / GW envs per 128-thread block, group collectives are segmented warp shuffles.
// GW > 32: one env per block of GW threads, collectives go through shared memory.  Every lane of a group runs the
// same control flow (ghost lanes r >= R and ghost envs e >= E carry neutral values and store nothing), because the
// schedule of a control step is the same for every env.
//
// Semantics follow isaac-net v0.2.0 (file:line in the comments); reductions over the RBG axis are left-to-right sums
// (the oracle's "seq" mode), ties in every argmax resolve to the lowest robot / process index (torch.max / argmin),
// and the retransmission ranking is a stable descending sort.
#include <cfloat>
#include <cmath>
#include <cstdint>

#pragma once
#include "nr_common.cuh"

namespace inb {

struct SmemGroup {
  unsigned long long red[2][4];   // per-warp partial maxima (GW up to 128: 4 warps), double-buffered
  float rkey[128];
  int32_t rnsb[128];
  int32_t flag[2];
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
  // lane = robot index within the group
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
  __device__ static bool any(bool v, SmemGroup* sm, int& par) {
    unsigned long long m = max_u64(v ? 1ull : 0ull, sm, par);
    return m != 0ull;
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
  __device__ static long long sum_i64(long long x, SmemGroup* sm, int& par);
};

struct Ctr {
  long long v[10];
  int hist_ok[INB_MAX_P > 16 ? 16 : 16];
  int hist_tx[16];
  int hist_fail[16];
};

// ------------------------------------------------------------------------------------------------ BLER lookup
// PHY.bler_lookup (isaac_net/core/phy.py:271-285), CUDA torch semantics: division by a python scalar is a multiply
// by the float32 reciprocal.
__device__ __forceinline__ float bler_lookup(const InbParams& p, const float* __restrict__ tab, int mcs, float sinr,
                                             int i0, float wi) {
  const int C = p.C_axis, G = p.G_axis;
  float s = isnan(sinr) ? -30.0f : sinr;
  float x = clampf_t(fm(fs(s, p.s0_snr), p.inv_ds), 0.0f, (float)(G - 1));
  float jf = floorf(x);
  int j0 = (int)jf;
  if (j0 > G - 2) j0 = G - 2;
  float wj = fs(x, (float)j0);
  long long b0 = ((long long)mcs * C + i0) * (long long)G;
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

// EESM effective SINR of one MCS over the won RBGs (PHY.eff_sinr / eff_sinr_all, phy.py:311-336), sequential sums.
// negl[s] = -lin[s] (lin = 10^(clamp(sinr,-30,60)/10)); lnw = logsumexp of log(w) over the won RBGs.
template <int SM>
__device__ __forceinline__ float eesm_db(const float (&negl)[SM], const float* __restrict__ lw, uint32_t won, int S,
                                         float beta, float lnw) {
  float xs[SM];
  float mx = -INFINITY;
#pragma unroll
  for (int s = 0; s < SM; ++s) {
    if (s < S) {
      float x = ((won >> s) & 1u) ? fa(fdv(negl[s], beta), lw[s]) : -INFINITY;
      xs[s] = x;
      mx = fmaxf(mx, x);
    }
  }
  float m0 = isinf(mx) ? 0.0f : mx;
  float sum = 0.0f;
  bool first = true;
#pragma unroll
  for (int s = 0; s < SM; ++s) {
    if (s < S) {
      float e = expf(fs(xs[s], m0));
      sum = first ? e : fa(sum, e);
      first = false;
    }
  }
  float lse = fa(logf(sum), m0);
  float eff = fm(-beta, fs(lse, lnw));
  return db_of(eff);
}

template <int SM>
__device__ __forceinline__ float lnw_of(const float* __restrict__ lw, uint32_t won, int S) {
  float mx = -INFINITY;
#pragma unroll
  for (int s = 0; s < SM; ++s)
    if (s < S && ((won >> s) & 1u)) mx = fmaxf(mx, lw[s]);
  float m0 = isinf(mx) ? 0.0f : mx;
  float sum = 0.0f;
  bool first = true;
#pragma unroll
  for (int s = 0; s < SM; ++s) {
    if (s < S) {
      float e = ((won >> s) & 1u) ? expf(fs(lw[s], m0)) : 0.0f;
      sum = first ? e : fa(sum, e);
      first = false;
    }
  }
  return fa(logf(sum), m0);
}

// ------------------------------------------------------------------------------------------------ the step kernel
template <int GW, int SM>
__global__ void __launch_bounds__(GW > 32 ? GW : 128) nr_step_kernel(const InbStepArgs A) {
  const InbParams& p = A.p;
  __shared__ SmemGroup smem_all[GW > 32 ? 1 : 128 / GW];
  __shared__ float s_lw[INB_MAX_S], s_lw10[INB_MAX_S], s_w[INB_MAX_S];
  __shared__ float s_thr[INB_MAX_MCS], s_se[INB_MAX_MCS], s_beta[INB_MAX_MCS], s_rate[INB_MAX_MCS];
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
  for (int i = tid; i < S; i += blockDim.x) {
    s_lw[i] = A.t.lw[i];
    s_lw10[i] = A.t.lw10[i];
    s_w[i] = A.t.w[i];
  }
  for (int i = tid; i < p.MCS; i += blockDim.x) {
    s_thr[i] = A.t.thr_ref[i];
    s_se[i] = A.t.se[i];
    s_beta[i] = A.t.beta[i];
    s_rate[i] = A.t.rate[i];
  }
  __syncthreads();

  const long long er = act ? e * R + r : 0;
  const long long eP = er * P, eF = er * F, eS = er * S;
  const InbState& st = A.s;

  // ---------------- per-robot scalars
  long long sent = 0, floor_ = 0, bsr = 0, sr_t = -1, last_tx = -1, enq = 0;
  float olla = 0.0f, avg = 100.0f;
  if (act) {
    sent = st.sent[er]; floor_ = st.floor_[er]; bsr = st.bsr[er]; sr_t = st.sr_t[er]; last_tx = st.last_tx[er];
    enq = st.enq[er]; olla = st.olla[er]; avg = st.avg[er];
  }
  const long long T = p.T;
  const long long epoch = env_ok ? A.epoch[e] : 0;
  const long long last_hid = env_ok ? A.last_hid[e] : 0;

  // ---------------- traffic enqueue (NREngine._inject / _enqueue, engine.py:191-244; FrameQueue.add, queues.py:87-103)
  long long g_end[INB_MAX_M];
  int g_slot[INB_MAX_M];
  const int M = p.M;
  const long long n0 = enq;
  const long long base = enq;
  long long n_acc = 0;
  int cnt_q = 0;
  if (act) {
    for (int f = 0; f < F; ++f) cnt_q += st.cap[eF + f] >= 0 ? 1 : 0;
  }
  for (int m = 0; m < M; ++m) {
    if (!act) break;
    const long long em = er * M + m;
    bool v = A.a.valid[em] != 0;
    float nbf = A.a.nbytes[em];
    bool acc = v && (cnt_q < F) && (nbf > 0.0f);
    if (acc) {
      int i = cnt_q < F - 1 ? cnt_q : F - 1;
      long long nb = (long long)rintf(nbf);
      long long at = eF + i;
      st.cap[at] = T;
      st.start[at] = enq;
      st.end_[at] = enq + nb;
      st.lost[at] = 0;
      st.fin[at] = INFINITY;
      st.cls[at] = 0;
      st.det[at] = (A.a.det[em] != 0 && v) ? 1 : 0;
      st.hid[at] = last_hid;
      st.off[at] = dm((double)A.a.slot[em], p.inv_N_d);
      st.tag[at] = A.a.tag[em];
      st.prio[at] = A.a.prio[em];
      st.dline[at] = A.a.dline[em];
      enq += nb;
      cnt_q += 1;
      n_acc += 1;
    }
    g_end[m] = enq;
    g_slot[m] = v ? (int)A.a.slot[em] : p.N;
  }
  const long long full_enq = enq;
  if (M > 0) enq = base;

  // ---------------- large-scale radio: path gain and the reference SINR of every RBG
  float pg = 0.0f;
  if (act) {
    if (A.pathgain_in != nullptr) {
      pg = A.pathgain_in[er];
    } else if (A.pos != nullptr) {
      const float px = A.pos[er * 2], py = A.pos[er * 2 + 1];
      const float gx = A.t.gnb[0], gy = A.t.gnb[1];
      const float dx = fs(px, gx), dy = fs(py, gy);
      const float d2 = fmaxf(sqrtf(fa(fm(dx, dx), fm(dy, dy))), 1.0f);
      // shadowing: amp * sum_k cos(k . x + phi) (channels/fields.py:61-64), field of (env, cell 0)
      float cs = 0.0f;
      const int Kf = p.Kf;
      for (int k = 0; k < Kf; ++k) {
        const long long fo = e * Kf + k;
        float kx = A.t.fk[fo * 2], ky = A.t.fk[fo * 2 + 1];
        float arg = fa(fa(fm(px, kx), fm(py, ky)), A.t.fphi[fo]);
        float c = cosf(arg);
        cs = k == 0 ? c : fa(cs, c);
      }
      float field = fm(p.amp, cs);
      if (p.radio_model <= 1) {
        // TR 38.901 UMi / UMa LOS path loss (channels/tr38901.py:148-170) + sigma_SF * unit field
        float d3 = sqrtf(fa(fm(d2, d2), p.hh2));
        float lg = log10f(d3);
        float pl = (d2 <= p.dbp) ? fa(fa(p.pl_a, fm(p.pl_n1, lg)), p.fc_term)
                                 : fs(fa(fa(p.pl_a, fm(40.0f, lg)), p.fc_term), p.pl_b_term);
        float sf = fm(p.sigma_sf, field);
        float rx = fa(p.ue_tx, -fa(pl, sf));
        pg = fs(rx, p.ue_tx);
      } else {
        // log-distance (radio.py:265-273)
        float pl = fa(p.pl_const, fm(p.pl_10n, log10f(d2)));
        float rx = fs(fs(p.ue_tx, pl), field);
        pg = fs(rx, p.ue_tx);
      }
    }
  }
  // ul_ref = ue_tx - 10 log10(snr_ref_prbs) + pg - N_prb (NRNet.step_rx, nr_engine.py:613-632)
  float ref[SM];
  const float ref_pg = fs(fa(p.ul_ref0, pg), p.noise_prb);
#pragma unroll
  for (int s = 0; s < SM; ++s) ref[s] = ref_pg;
  if (act && A.ul_ref_in != nullptr) {
#pragma unroll
    for (int s = 0; s < SM; ++s)
      if (s < S) ref[s] = A.ul_ref_in[eS + s];
  }
  const float sinr_obs = fs(fa(pg, p.ue_tx), p.sub_noise);

  // ---------------- fading state and CSI
  float hr[SM], hi[SM], csi[SM], gain[SM];
#pragma unroll
  for (int s = 0; s < SM; ++s) {
    hr[s] = 0.0f; hi[s] = 0.0f; csi[s] = 0.0f; gain[s] = 0.0f;
    if (act && s < S) {
      hr[s] = st.h[(eS + s) * 2];
      hi[s] = st.h[(eS + s) * 2 + 1];
      csi[s] = st.csi[eS + s];
    }
  }
  float k_lin = 0.0f, sp_r = 1.0f, sp_i = 0.0f;
  if (act && p.rician) {
    k_lin = st.k_lin[er];
    sp_r = st.spec[er * 2];
    sp_i = st.spec[er * 2 + 1];
  }
  float phr_ref_mean = 0.0f;  // mean over RBGs of ul_ref (PHR cap), left-to-right sum times float32(1/S)
  {
    float sum = 0.0f;
#pragma unroll
    for (int s = 0; s < SM; ++s)
      if (s < S) sum = s == 0 ? ref[s] : fa(sum, ref[s]);
    phr_ref_mean = fm(sum, p.inv_S);
  }
  int n_max = S;
  if (p.phr_cap) {
    // n_max = floor(snr_ref_prbs * 10^((mean(ul_ref) - phr_min) / 10) / w[0]).clamp(1, S) (mac_ul.py:165-168)
    float x = fm(fs(phr_ref_mean, p.phr_min), 0.1f);
    float nmp = fm((float)p.ref_prbs, powf(10.0f, x));
    float q = floorf(fdv(nmp, s_w[0]));
    q = clampf_t(q, 1.0f, (float)S);
    n_max = (int)q;
  }

  // counter RNG keys of this env's step draws
  const uint32_t kenv = env_ok ? key_env(p.s0, A.env_id[e], A.episode[e], CH_STEP, A.rng_ctr[e]) : 0u;
  const float two_pi = 6.28318548202514648438f;

  Ctr ctr;
#pragma unroll
  for (int i = 0; i < 10; ++i) ctr.v[i] = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) { ctr.hist_ok[i] = 0; ctr.hist_tx[i] = 0; ctr.hist_fail[i] = 0; }

  // first frame not yet finished (RLC scan start); frames are in stream order
  int f_scan = 0;
  int nvalid = cnt_q;
  if (act) {
    while (f_scan < nvalid && (st.lost[eF + f_scan] != 0 || !isinf(st.fin[eF + f_scan]))) ++f_scan;
  }

  // ======================================================================= slot loop (nr_engine.py:656-667)
  for (int k = 0; k < p.K_rows; ++k) {
    const int rel = p.rows[k][0], uls = p.rows[k][1], srf = p.rows[k][2], fad = p.rows[k][3];
    const long long g = T * p.N + rel;
    // ---- AR(1) fading step (NRNet._evolve / _gain, nr_engine.py:570-611)
    if (p.fading) {
      if (fad) {
        const uint32_t base_f = key_stream(kenv, (uint32_t)((SITE_FADING << 16) | rel));
        const float rho = p.rowf[k][0], c1 = p.rowf[k][1];
#pragma unroll
        for (int s = 0; s < SM; ++s) {
          if (s < S) {
            uint32_t j = (uint32_t)((r * S + s) * 2);
            float zr = normal_at(base_f, j, two_pi);
            float zi = normal_at(base_f, j + 1u, two_pi);
            hr[s] = fa(fm(rho, hr[s]), fm(fm(c1, zr), p.inv_sqrt2));
            hi[s] = fa(fm(rho, hi[s]), fm(fm(c1, zi), p.inv_sqrt2));
          }
        }
      }
      if (p.rician) {
        float kinv = fdv(1.0f, fa(k_lin, 1.0f));
        float ka = sqrtf(fm(k_lin, kinv)), kb = sqrtf(kinv);
        float ar_ = fm(ka, sp_r), ai_ = fm(ka, sp_i);
#pragma unroll
        for (int s = 0; s < SM; ++s) {
          if (s < S) {
            float xr = fa(ar_, fm(kb, hr[s])), xi = fa(ai_, fm(kb, hi[s]));
            gain[s] = fm(10.0f, log10f(clamp_min_t(fa(fm(xr, xr), fm(xi, xi)), 1e-6f)));
          }
        }
      } else {
#pragma unroll
        for (int s = 0; s < SM; ++s)
          if (s < S) gain[s] = fm(10.0f, log10f(clamp_min_t(fa(fm(hr[s], hr[s]), fm(hi[s], hi[s])), 1e-6f)));
      }
    }
    // ---- arrival gate (NREngine._open_gate, engine.py:176-183)
    if ((srf || uls) && M > 0 && act) {
      long long vis = base;
      for (int m = 0; m < M; ++m) {
        long long v = g_slot[m] <= rel ? g_end[m] : base;
        vis = v > vis ? v : vis;
      }
      enq = vis > base ? vis : base;
    }
    // ---- SR (UlMac.sr_step, mac_ul.py:66-71)
    if (srf) {
      if ((enq - sent > 0) && bsr <= 0 && sr_t < 0) sr_t = g;
    }
    if (!uls) continue;

    // =================================================================== UL data slot (MacLink.slot, mac.py:228-508)
    const long long unsent = enq - sent;
    // lumped SR grant (mac_ul.py:140-147)
    if (sr_t >= 0 && g - sr_t >= p.sr_delay) {
      bsr = bsr < 1 ? 1 : bsr;
      sr_t = -1;
    }
    // candidates: earliest ready NACKed process, else the first free one
    int rx_p = 0, p_new = -1;
    long long best_ready = BIGI;
    bool has_rx = false, pending = false;
    if (act) {
      for (int q = 0; q < P; ++q) {
        long long hs = st.h_state[eP + q];
        if (hs == 1) {
          pending = true;
          long long rd = st.h_ready[eP + q];
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
    const int rx_nsb = act ? (int)st.h_nsb[eP + rx_p] : 0;
    // scheduler estimate with OLLA, rate and metric per RBG (mac.py:255-275, mac_ul.py:154-171)
    float rate[SM], metric[SM];
    const float re_prb = (float)min(12 * uls - p.dmrs - p.oh, 156);
#pragma unroll
    for (int s = 0; s < SM; ++s) {
      rate[s] = 0.0f; metric[s] = 0.0f;
      if (s < S) {
        float est = fa(fs(ref[s], s_lw10[s]), csi[s]);
        float eo = p.olla_on ? fa(est, olla) : fa(est, 0.0f);
        int m = 0;
        for (int mm = 0; mm <= p.mcs_max; ++mm)
          if (eo >= s_thr[mm]) m = mm;
        rate[s] = fm(fm(fm(s_se[m], re_prb), s_w[s]), 0.125f);
        if (p.sched == 2)
          metric[s] = (float)(g - last_tx);
        else if (p.sched == 1)
          metric[s] = rate[s];
        else
          metric[s] = fdv(rate[s], fmaxf(avg, 1e-9f));
      }
    }
    // retransmission admission: rank by metric sum (stable, descending), admit while RBG counts fit (mac.py:300-312)
    if (Grp<GW>::any_uniform(has_rx, sm, par)) {
      float rkey = -1.0f;
      if (has_rx) {
        float sum = 0.0f;
#pragma unroll
        for (int s = 0; s < SM; ++s)
          if (s < S) sum = s == 0 ? metric[s] : fa(sum, metric[s]);
        rkey = sum;
      }
      const int mine = has_rx ? rx_nsb : 0;
      int before = 0;
      if constexpr (GW <= 32) {
        for (int j = 0; j < GW; ++j) {
          float kj = __shfl_sync(0xFFFFFFFFu, rkey, j, GW);
          int nj = __shfl_sync(0xFFFFFFFFu, mine, j, GW);
          if (kj > rkey || (kj == rkey && j < r)) before += nj;
        }
      } else {
        sm->rkey[r] = rkey;
        sm->rnsb[r] = mine;
        __syncthreads();
        for (int j = 0; j < GW; ++j) {
          float kj = sm->rkey[j];
          if (kj > rkey || (kj == rkey && j < r)) before += sm->rnsb[j];
        }
        __syncthreads();
      }
      has_rx = has_rx && (before + mine <= S);
    }
    const int want_cnt = has_rx ? rx_nsb : (new_el ? n_max : 0);
    const bool lex = p.retx_priority != 0;
    const float prio = lex ? fm(1e9f, has_rx ? 1.0f : 0.0f) : 0.0f;
    // greedy allocation RBG by RBG (mac.py:322-351)
    uint32_t won = 0u;
    int cnt = 0;
    float left = (float)need;
#pragma unroll
    for (int s = 0; s < SM; ++s) {
      if (s < S) {
        bool want = act && (cnt < want_cnt) && (has_rx || left > 0.0f);
        float mkey = want ? fa(metric[s], prio) : -1.0f;
        bool wr = lex && want && has_rx;
        unsigned long long key = ((unsigned long long)(wr ? 1u : 0u) << 40) |
                                 ((unsigned long long)fkey(mkey) << 8) | (unsigned long long)(255 - r);
        unsigned long long mx = Grp<GW>::max_u64(key, sm, par);
        int wi = 255 - (int)(mx & 0xFFull);
        float best = fkey_inv((uint32_t)((mx >> 8) & 0xFFFFFFFFull));
        bool oh = (wi == r) && (best >= 0.0f);
        if (oh) {
          won |= 1u << s;
          cnt += 1;
        }
        float dec = fm(fm(rate[s], oh ? 1.0f : 0.0f), has_rx ? 0.0f : 1.0f);
        left = fs(left, dec);
      }
    }
    if (!lex) {
      // retransmissions that won fewer RBGs than their TB needs release them to the new-data robots (mac.py:353-379)
      bool short_ = has_rx && (__popc(won) != rx_nsb);
      uint32_t rel_rs = short_ ? won : 0u;
      if (short_) won = 0u;
      cnt = __popc(won);
#pragma unroll
      for (int s = 0; s < SM; ++s) {
        if (s < S) {
          bool want = act && (cnt < want_cnt) && new_el && (left > 0.0f);
          float mkey = want ? metric[s] : -1.0f;
          unsigned long long key = ((unsigned long long)fkey(mkey) << 8) | (unsigned long long)(255 - r);
          unsigned long long mx = Grp<GW>::max_u64(key, sm, par);
          bool av = Grp<GW>::any(((rel_rs >> s) & 1u) != 0u, sm, par);
          int wi = 255 - (int)(mx & 0xFFull);
          float best = fkey_inv((uint32_t)((mx >> 8) & 0xFFFFFFFFull));
          bool oh = (wi == r) && (best >= 0.0f) && av;
          if (oh) {
            won |= 1u << s;
            cnt += 1;
          }
          left = fs(left, fm(rate[s], oh ? 1.0f : 0.0f));
        }
      }
    }
    const int n_sb = __popc(won);
    float n_prb = 0.0f;
#pragma unroll
    for (int s = 0; s < SM; ++s)
      if (s < S && ((won >> s) & 1u)) n_prb = fa(n_prb, s_w[s]);
    const bool tx_rx = has_rx && (n_sb == rx_nsb) && (n_sb > 0);
    const bool tx_new = new_el && (n_sb > 0);
    const bool tx = tx_rx || tx_new;

    // power split over the grant (UlMac._split, mac_ul.py:173-180)
    const float split = fm(10.0f, log10f(clamp_min_t(fm(n_prb, p.inv_ref_prbs), 1e-3f)));
    float negl[SM];  // -10^(clamp(sinr, -30, 60) / 10) of the link-adaptation or decode SINR
    // ---- link adaptation of a new TB (PHY.select_mcs, phy.py:339-350), highest passing MCS scanned downward
    int mcs_new = 0;
    long long tbs_new = 0;
    float lnw = 0.0f;
    if (tx) lnw = lnw_of<SM>(s_lw, won, S);
    if (tx_new) {
      const int np = (int)n_prb;
      const long long trow = (long long)np * p.MCS;
#pragma unroll
      for (int s = 0; s < SM; ++s) {
        negl[s] = 0.0f;
        if (s < S) {
          float est_tx = fa(fs(ref[s], split), csi[s]);
          negl[s] = -powf(10.0f, fm(clampf_t(est_tx, -30.0f, 60.0f), 0.1f));
        }
      }
      const float off = p.olla_on ? olla : 0.0f;
      int chosen = -1;
      for (int m = p.mcs_max; m >= 0; --m) {
        const int tb = A.t.la_tbs[trow + m];
        if (tb <= 0) continue;
        float eff = fa(eesm_db<SM>(negl, s_lw, won, S, s_beta[m], lnw), off);
        float b = bler_lookup(p, A.t.bler, m, eff, A.t.la_i0[trow + m], A.t.la_wi[trow + m]);
        float tbler = fs(1.0f, powf(fs(1.0f, b), A.t.la_ncb[trow + m]));
        if (tbler <= p.target) { chosen = m; break; }
      }
      mcs_new = chosen < 0 ? 0 : chosen;
      tbs_new = A.t.la_tbs[trow + mcs_new];
    }
    long long cap_b = tbs_new / 8 - p.tb_oh;
    cap_b = cap_b < 1 ? 1 : cap_b;
    const long long byt_new = cap_b < unsent ? cap_b : unsent;
    // ---- bind the TB to its HARQ process (mac.py:406-423)
    const int p_tx = tx_rx ? rx_p : p_new;
    const long long hp = eP + p_tx;
    if (tx_new) {
      st.h_lo[hp] = sent;
      st.h_hi[hp] = sent + byt_new;
      st.h_mcs[hp] = mcs_new;
      st.h_tbs[hp] = tbs_new;
      st.h_nsb[hp] = n_sb;
      st.h_ntx[hp] = 0;
      st.h_comb[hp] = 0.0f;
      st.h_state[hp] = 1;
      sent += byt_new;
    }
    // ---- decode on the actual channel, HARQ / OLLA / PF updates (mac.py:424-498)
    bool ok = false, fail = false, exh = false;
    long long served = 0;
    int ntx = 0;
    if (tx) {
      const int mcs = (int)st.h_mcs[hp];
      const long long tbs = st.h_tbs[hp];
      ntx = (int)st.h_ntx[hp] + 1;
#pragma unroll
      for (int s = 0; s < SM; ++s) {
        negl[s] = 0.0f;
        if (s < S) {
          float a_ = fa(fs(ref[s], split), gain[s]);
          negl[s] = -powf(10.0f, fm(clampf_t(a_, -30.0f, 60.0f), 0.1f));
        }
      }
      float eff = eesm_db<SM>(negl, s_lw, won, S, s_beta[mcs], lnw);
      float lin = powf(10.0f, fm(eff, 0.1f));
      float comb = p.comb_cc ? fa(st.h_comb[hp], lin) : lin;
      float eff_used = fm(10.0f, log10f(clamp_min_t(comb, 1e-9f)));
      float cbs, ncb;
      segment(tbs, s_rate[mcs], cbs, ncb);
      int i0;
      float wi;
      cidx(p, cbs, i0, wi);
      float b = bler_lookup(p, A.t.bler, mcs, eff_used, i0, wi);
      float p_err = fs(1.0f, powf(fs(1.0f, b), ncb));
      const uint32_t base_u = key_stream(kenv, (uint32_t)((SITE_BLER_UL << 16) | rel));
      float u = uniform_at(base_u, (uint32_t)r);
      ok = u >= p_err;
      fail = !ok;
      exh = fail && ntx >= p.max_tx;
      if (ok) {
        st.h_state[hp] = 0;
        st.h_ready[hp] = g;
      }
      st.h_ntx[hp] = ntx;
      st.h_comb[hp] = comb;
      if (fail) st.h_ready[hp] = g + p.ul_rtt;
      const long long lo_tx = st.h_lo[hp], hi_tx = st.h_hi[hp];
      if (exh) {
        if (!p.harq_drop) {
          st.h_ntx[hp] = 0;
          st.h_comb[hp] = 0.0f;
          st.h_ready[hp] = g + p.rlc_retx;
        } else {
          st.h_state[hp] = 0;
          for (int f = 0; f < F; ++f) {
            const long long at = eF + f;
            if (st.cap[at] >= 0 && st.start[at] < hi_tx && st.end_[at] > lo_tx) {
              if (!st.lost[at]) ctr.v[9] += 1;
              st.lost[at] = 1;
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
    if (p.olla_on) {
      float up = fm(p.olla_up, ok ? 1.0f : 0.0f), dn = fm(p.olla_dn, fail ? 1.0f : 0.0f);
      olla = clampf_t(fs(fa(olla, up), dn), -10.0f, 10.0f);
    }
    if (tx) bsr = enq - sent;
#pragma unroll
    for (int s = 0; s < SM; ++s) csi[s] = gain[s];
    avg = fmaxf(fa(fm(p.pf_a, avg), fm(p.pf_b, (float)served)), 1e-9f);
    if (p.sched == 2 && tx) last_tx = g;
    if (act) {
      ctr.v[0] += tx_new; ctr.v[1] += tx_rx; ctr.v[2] += ok; ctr.v[3] += fail; ctr.v[4] += exh;
      ctr.v[5] += served; ctr.v[6] += tx_new ? byt_new : 0; ctr.v[7] += (tx_new && pending);
      ctr.v[8] += tx ? (long long)n_prb : 0;
      if (tx) {
        int kx = ntx < p.max_tx ? ntx : p.max_tx;
        kx = kx < 15 ? kx : 15;
        ctr.hist_tx[kx] += 1;
        if (ok) ctr.hist_ok[kx] += 1;
        if (fail) ctr.hist_fail[kx] += 1;
      }
    }
    // ---- RLC in-order delivery (MacLink.ack_ptr, mac.py:194-197, 499-503)
    if (act) {
      long long ack = sent;
      for (int q = 0; q < P; ++q) {
        if (st.h_state[eP + q] == 1) {
          long long hh = st.h_hi[eP + q];
          if (hh > floor_) {
            long long ll = st.h_lo[eP + q];
            ll = ll > floor_ ? ll : floor_;
            ack = ll < ack ? ll : ack;
          }
        }
      }
      const double fin_val = da(da((double)T, ddv((double)(rel + 1), (double)p.N)), p.proc_off);
      int f = f_scan;
      while (f < nvalid) {
        const long long at = eF + f;
        if (st.end_[at] > ack) break;
        if (!st.lost[at] && isinf(st.fin[at])) st.fin[at] = fin_val;
        ++f;
      }
      while (f_scan < nvalid && (st.lost[eF + f_scan] != 0 || !isinf(st.fin[eF + f_scan]))) ++f_scan;
    }
  }

  // ======================================================================= finish (nr_engine.py:843-888)
  if (M > 0) enq = full_enq;
  long long ack_end = sent;
  if (act) {
    for (int q = 0; q < P; ++q) {
      if (st.h_state[eP + q] == 1) {
        long long hh = st.h_hi[eP + q];
        if (hh > floor_) {
          long long ll = st.h_lo[eP + q];
          ll = ll > floor_ ? ll : floor_;
          ack_end = ll < ack_end ? ll : ack_end;
        }
      }
    }
  }
  const double lim = da((double)(T + 1), 1e-9);
  long long newest = -1;
  bool det_hit = false;
  // compaction order: surviving frames first (stable), then the freed slots in index order (queues.py:105-110)
  int order[INB_MAX_F];
  int n_keep = 0, n_gone = 0;
  uint64_t gone_mask = 0ull;
  if (act) {
    const InbOutputs& o = A.o;
    for (int f = 0; f < F; ++f) {
      const long long at = eF + f;
      const long long cap = st.cap[at];
      const bool valid = cap >= 0;
      const double fin = st.fin[at];
      const bool delivered = valid && fin <= lim;
      const bool timed = p.purge && valid && isinf(fin) && ((T + 1 - cap) >= p.timeout);
      const bool dropped = valid && st.lost[at] && (st.end_[at] <= ack_end) && !timed;
      if (delivered && cap > newest) newest = cap;
      if (delivered && st.det[at] && st.hid[at] == last_hid) det_hit = true;
      const double off = st.off[at];
      o.delivered[at] = delivered;
      o.timed_out[at] = timed;
      o.dropped[at] = dropped;
      o.cap[at] = valid ? cap - epoch : -1;
      o.cls[at] = valid ? st.cls[at] : 0;
      const float delay = (float)dsb(dsb(fin, (double)cap), off);
      o.delay[at] = delivered ? delay : NAN;
      o.arrival[at] = valid ? da((double)(cap - epoch), off) : NAN;
      o.arrival_slot[at] = valid ? (long long)rint(dm(off, (double)p.N)) : -1;
      o.tag[at] = valid ? st.tag[at] : 0;
      o.priority[at] = valid ? st.prio[at] : 0;
      o.bytes[at] = valid ? st.end_[at] - st.start[at] : 0;
      const double dl = st.dline[at];
      const bool late = delivered && (dm((double)delay, p.ctl_ms) > dl);
      o.deadline_miss[at] = late || ((timed || dropped) && isfinite(dl));
      const bool gone = delivered || timed || dropped;
      if (gone || !valid) gone_mask |= 1ull << f;
    }
    for (int f = 0; f < F; ++f)
      if (!((gone_mask >> f) & 1ull)) order[n_keep++] = f;
    for (int f = 0; f < F; ++f)
      if ((gone_mask >> f) & 1ull) order[n_keep + n_gone++] = f;
    // permute every frame field in place through registers, one field at a time
    auto perm_i64 = [&](int64_t* a) {
      long long tmp[INB_MAX_F];
      for (int f = 0; f < F; ++f) tmp[f] = a[eF + order[f]];
      for (int f = 0; f < F; ++f) a[eF + f] = tmp[f];
    };
    auto perm_f64 = [&](double* a) {
      double tmp[INB_MAX_F];
      for (int f = 0; f < F; ++f) tmp[f] = a[eF + order[f]];
      for (int f = 0; f < F; ++f) a[eF + f] = tmp[f];
    };
    auto perm_u8 = [&](uint8_t* a) {
      uint8_t tmp[INB_MAX_F];
      for (int f = 0; f < F; ++f) tmp[f] = a[eF + order[f]];
      for (int f = 0; f < F; ++f) a[eF + f] = tmp[f];
    };
    {
      long long tmp[INB_MAX_F];
      for (int f = 0; f < F; ++f) tmp[f] = ((gone_mask >> order[f]) & 1ull) ? -1 : st.cap[eF + order[f]];
      for (int f = 0; f < F; ++f) st.cap[eF + f] = tmp[f];
    }
    perm_i64(st.start); perm_i64(st.end_); perm_i64(st.cls); perm_i64(st.hid); perm_i64(st.tag); perm_i64(st.prio);
    perm_u8(st.lost); perm_u8(st.det);
    perm_f64(st.fin); perm_f64(st.off); perm_f64(st.dline);
    // stream floor, send pointer, HARQ processes holding only purged bytes (MacLink.compact, mac.py:598-616)
    floor_ = n_keep > 0 ? st.start[eF] : enq;
    sent = sent > floor_ ? sent : floor_;
    for (int q = 0; q < P; ++q) {
      const long long at = eP + q;
      if (st.h_state[at] == 1 && st.h_hi[at] <= floor_ && st.h_hi[at] > st.h_lo[at]) {
        st.h_state[at] = 0; st.h_ready[at] = 0; st.h_ntx[at] = 0; st.h_comb[at] = 0.0f;
      }
    }
    bsr = bsr < enq - sent ? bsr : enq - sent;
    long long ackq = sent;
    for (int q = 0; q < P; ++q) {
      if (st.h_state[eP + q] == 1) {
        long long hh = st.h_hi[eP + q];
        if (hh > floor_) {
          long long ll = st.h_lo[eP + q];
          ll = ll > floor_ ? ll : floor_;
          ackq = ll < ackq ? ll : ackq;
        }
      }
    }
    o.newest[er] = newest >= 0 ? newest - epoch : -1;
    o.queue_len[er] = n_keep;
    long long qb = enq - ackq;
    o.queue_bytes[er] = (float)(qb > 0 ? qb : 0);
    o.sinr_db[er] = sinr_obs;
    if (o.pathgain) o.pathgain[er] = pg;
    o.gen_accepted[er] = n_acc;
    o.gen_bytes[er] = full_enq - n0;
    // ---- state back to memory
    st.sent[er] = sent; st.floor_[er] = floor_; st.bsr[er] = bsr; st.sr_t[er] = sr_t; st.last_tx[er] = last_tx;
    st.enq[er] = enq; st.olla[er] = olla; st.avg[er] = avg;
#pragma unroll
    for (int s = 0; s < SM; ++s) {
      if (s < S) {
        st.csi[eS + s] = csi[s];
        st.h[(eS + s) * 2] = hr[s];
        st.h[(eS + s) * 2 + 1] = hi[s];
      }
    }
  }
  // det_env and counters: group reductions, then one writer per group
  bool det_any = Grp<GW>::any(det_hit, sm, par);
  if (env_ok && r == 0) A.o.det_env[e] = det_any ? 1 : 0;
  if (act) {
    int64_t* c = A.ctr + e * INB_NCTR;
#pragma unroll
    for (int i = 0; i < 10; ++i)
      if (ctr.v[i]) atomicAdd((unsigned long long*)&c[i], (unsigned long long)ctr.v[i]);
    for (int i = 0; i < 16; ++i) {
      if (ctr.hist_ok[i]) atomicAdd((unsigned long long*)&c[INB_CTR_NTX_HIST + i], (unsigned long long)ctr.hist_ok[i]);
      if (ctr.hist_tx[i]) atomicAdd((unsigned long long*)&c[INB_CTR_RV_TX + i], (unsigned long long)ctr.hist_tx[i]);
      if (ctr.hist_fail[i]) atomicAdd((unsigned long long*)&c[INB_CTR_RV_FAIL + i], (unsigned long long)ctr.hist_fail[i]);
    }
  }
  if (env_ok && r == 0) A.rng_ctr[e] += 1;
}


}  // namespace inb
