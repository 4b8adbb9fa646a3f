// AR(1) small-scale fading of one control step, ahead of the MAC kernel (NRNet._evolve / _gain,
// isaac_net/core/nr_engine.py:570-611).
//
// The fading of a (robot, RBG) depends only on its own state, the counter-RNG keys and the schedule of the step, not
// on any MAC decision, so it runs as its own launch with one thread per (robot, RBG): few registers, full occupancy,
// and the 2 Box-Muller normals per row (hash elements (r S + s) 2 + {0, 1} of the row's FADING stream) that bitwise
// parity requires are the bulk of its work.  For the u-th UL row of the step it writes the row's gain (dB) to
// gain[u + 1][e R + r][s] and copies the CSI of the previous step into gain[0]; so the MAC kernel finds the CSI of
// its u-th UL row in gain[u] and the row's fading gain in gain[u + 1], a robot's RBGs contiguous.  The new fading
// state h [E,R,S,2] and the CSI state (the gain of the last UL row, the CSI report rule of MacLink, mac.py:485) are
// written back in place.  With C > 1 cells every link (robot, cell) fades on its own (h [E,R,C,S,2], hash elements
// ((r C + c) S + s) 2 + {0, 1}) and gain row u is the u-th UL row's gain of every link, [E R][C][S]; the CSI then
// depends on the serving cell and its handovers, so the MAC kernel keeps it.  With the downlink (p.dl_on, one cell) the
// gain of every row that carries DL data or a CQI report also goes to gain row n_ul_rows + 1 + rows_dl[k][3].
#include <cmath>
#include <cstdint>

#include "nr_common.cuh"

namespace inb {

// The (robot, cell, RBG) element t of the step (RBGs fastest): its AR(1) rows, gain rows and CSI
__device__ __forceinline__ void fade_element(const InbStepArgs& A, const uint32_t* s_salt, long long t) {
  const InbParams& p = A.p;
  const long long NER = (long long)p.E * p.R;
  const int S = p.S;
  const int C = p.C > 1 ? p.C : 1;
  const long long plane = NER * C * S;
  const long long ec = t / S;                  // link (robot, cell)
  const int s = (int)(t - ec * S);
  const long long er = ec / C;
  const int c = (int)(ec - er * C);
  const long long e = er / p.R;
  const int r = (int)(er - e * p.R);
  const InbState& st = A.s;
  const float2 h0 = reinterpret_cast<const float2*>(st.h)[t];
  float hr = h0.x, hi = h0.y;
  float* __restrict__ gout = A.gain + t;
  float last = 0.0f;
  if (C == 1) {
    last = st.csi[t];
    gout[0] = last;
  }
  float ar_ = 0.0f, ai_ = 0.0f, kb = 1.0f;
  if (p.rician) {
    // |sqrt(K/(K+1)) e^{j phi} + sqrt(1/(K+1)) h|^2 (NRNet._gain, nr_engine.py:602-611)
    const float k_lin = st.k_lin[ec];
    const float kinv = fdv(1.0f, fa(k_lin, 1.0f));
    const float ka = sqrtf(fm(k_lin, kinv));
    kb = sqrtf(kinv);
    ar_ = fm(ka, st.spec[ec * 2]);
    ai_ = fm(ka, st.spec[ec * 2 + 1]);
  }
  const uint32_t kenv = key_env(p.s0, A.env_id[e], A.episode[e], CH_STEP, A.rng_ctr[e]);
  const float two_pi = 6.28318548202514648438f;
  const uint32_t j = (uint32_t)(((r * C + c) * S + s) * 2);
  int u = 0;
  for (int k = 0; k < p.K_rows; ++k) {
    const int rel = p.rows[k][0], uls = p.rows[k][1], fad = p.rows[k][3];
    if (p.fading && fad) {
      const uint32_t base_f = mix32(kenv ^ s_salt[k]);   // key_stream(kenv, (SITE_FADING << 16) | rel)
      const float rho = p.rowf[k][0], c1 = p.rowf[k][1];
      const float zr = normal_at(base_f, j, two_pi);
      const float zi = normal_at(base_f, j + 1u, two_pi);
      hr = fa(fm(rho, hr), fm(fm(c1, zr), p.inv_sqrt2));
      hi = fa(fm(rho, hi), fm(fm(c1, zi), p.inv_sqrt2));
    }
    const int dlr = p.dl_on ? p.rows_dl[k][3] : -1;
    if (uls || dlr >= 0) {
      float g = 0.0f;
      if (p.fading) {
        float pw;
        if (p.rician) {
          const float xr = fa(ar_, fm(kb, hr)), xi = fa(ai_, fm(kb, hi));
          pw = fa(fm(xr, xr), fm(xi, xi));
        } else {
          pw = fa(fm(hr, hr), fm(hi, hi));
        }
        g = fm(10.0f, log10f(clamp_min_t(pw, 1e-6f)));
      }
      if (dlr >= 0) gout[(long long)(p.n_ul_rows + 1 + dlr) * plane] = g;
      if (uls) {
        if (C == 1) ++u;
        gout[(long long)u * plane] = g;
        if (C > 1) ++u;
        last = g;
      }
    }
  }
  if (p.fading) reinterpret_cast<float2*>(st.h)[t] = make_float2(hr, hi);
  if (C == 1) st.csi[t] = last;
}

// Elements [t_begin, t_end) (whole envs), one per thread
__global__ void __launch_bounds__(256) nr_fading_kernel(const InbStepArgs A, long long t_begin, long long t_end) {
  const InbParams& p = A.p;
  // the stream salt of each row's FADING draws (the same for every thread): computed once per block
  __shared__ uint32_t s_salt[INB_MAX_ROWS];
  for (int k = threadIdx.x; k < p.K_rows; k += blockDim.x)
    s_salt[k] = salt((uint32_t)((SITE_FADING << 16) | p.rows[k][0]));
  __syncthreads();
  const long long t = t_begin + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < t_end) fade_element(A, s_salt, t);
}

cudaError_t launch_fading(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  const long long per_env = (long long)a.p.R * (a.p.C > 1 ? a.p.C : 1) * a.p.S;
  const long long t0 = (long long)rg.e0 * per_env, t1 = (long long)rg.e1 * per_env;
  const int block = 256;
  const long long grid = (t1 - t0 + block - 1) / block;
  if (grid <= 0) return cudaSuccess;
  nr_fading_kernel<<<(unsigned)grid, block, 0, stream>>>(a, t0, t1);
  return cudaGetLastError();
}

}  // namespace inb
