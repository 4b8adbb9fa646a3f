// Episode resets and counter-RNG draws of the B200 NR engine.
//
// inb_nr_reset: for the envs of a mask, the device side of NRNet.reset(env_ids) (isaac_net/core/nr_engine.py:250-320):
// new episode (episode += 1, STEP counter = 0, nr_rng.py:45-52), MAC and queue state back to the initial values
// (MacLink.STATE, mac.py:67-81; FrameQueue.INIT / EXTRAS, queues.py:374-376), the initial fading state from the
// RESET channel (site H0: h = N(0, 1) / sqrt(2), element (r S + s) 2 + c) and the Rician phasor (site KPHI:
// phi = 2 pi u, one uniform per robot) with K = rician_k_db in linear units.
// inb_rng_draw: uniforms or normals [E, n] of one (channel, stream) for every env row (CounterRNG._draw,
// isaac_net/core/proto/rng.py:137-161).
#include <cmath>
#include <cstdint>

#include "nr_common.cuh"

namespace inb {

__global__ void nr_reset_kernel(const InbResetArgs A) {
  const long long er = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)A.E * A.R;
  if (er >= total) return;
  const long long e = er / A.R;
  const int r = (int)(er % A.R);
  if (A.mask != nullptr && A.mask[e] == 0) return;
  const int S = A.S, P = A.P, F = A.F;
  const InbState& st = A.s;
  // the episode advances for every reset env; each robot thread reads the old value and derives the new one
  const long long ep = A.episode[e] + 1;
  const uint32_t kenv = key_env(A.s0, A.env_id[e], ep, CH_RESET, 0);
  st.sent[er] = 0; st.floor_[er] = 0; st.bsr[er] = 0; st.sr_t[er] = -1; st.last_tx[er] = -1; st.enq[er] = 0;
  st.olla[er] = 0.0f; st.avg[er] = 100.0f;
  if (st.last_nprb != nullptr) st.last_nprb[er] = 0.0f;
  if (st.bsr_est != nullptr) {   // BSR_STATE initial values (mac_ul.py:45-50)
    st.bsr_est[er] = 0; st.bsr_hid[er] = 0; st.bsr_hid_until[er] = -1; st.bsr_enq_seen[er] = 0;
    st.bsr_boot[er] = 0; st.bsr_armed[er] = 0;
    for (int j = 0; j < INB_BSR_DEPTH; ++j) {
      st.bsr_rep_v[er * INB_BSR_DEPTH + j] = 0;
      st.bsr_rep_g[er * INB_BSR_DEPTH + j] = -BIGI;
    }
  }
  const uint32_t base_h = key_stream(kenv, (uint32_t)(SITE_H0 << 16));
  const int C = A.C > 1 ? A.C : 1;
  for (int s = 0; s < S; ++s) st.csi[er * S + s] = 0.0f;
  for (int c = 0; c < C; ++c) {
    const long long ec = er * C + c;            // link (robot, cell)
    for (int s = 0; s < S; ++s) {
      for (int q = 0; q < 2; ++q) {
        const uint32_t j = (uint32_t)(((r * C + c) * S + s) * 2 + q);
        st.h[(ec * S + s) * 2 + q] = fm(normal_at(base_h, j, A.two_pi), A.inv_sqrt2);
      }
    }
  }
  if (A.rician) {
    const uint32_t base_k = key_stream(kenv, (uint32_t)(SITE_KPHI << 16));
    for (int c = 0; c < C; ++c) {
      const long long ec = er * C + c;
      float phi = fm(A.two_pi, uniform_at(base_k, (uint32_t)(r * C + c)));
      st.spec[ec * 2] = cosf(phi);
      st.spec[ec * 2 + 1] = sinf(phi);
      st.k_lin[ec] = A.k_lin0;
    }
  }
  if (A.C > 1) {   // CellAssociation.reset (radio.py:391-396), NRNet._reset_cells (nr_engine.py:424-438)
    st.serv[er] = 0; st.a3_cand[er] = -1; st.a3_cnt[er] = 0; st.ho_end[er] = 0; st.n_ho[er] = 0;
    if (r == 0) {
      st.pending[e] = 1;
      for (int i = 0; i < A.C * S; ++i) st.ni_ul[e * A.C * S + i] = A.noise_mw;
    }
  }
  for (int q = 0; q < P; ++q) {
    const long long at = er * P + q;
    st.h_state[at] = 0; st.h_lo[at] = 0; st.h_hi[at] = 0; st.h_ready[at] = 0; st.h_ntx[at] = 0; st.h_mcs[at] = 0;
    st.h_tbs[at] = 0; st.h_nsb[at] = 0; st.h_comb[at] = 0.0f;
  }
  for (int f = 0; f < F; ++f) {
    const long long at = er * F + f;
    st.cap[at] = -1; st.start[at] = 0; st.end_[at] = 0; st.cls[at] = 0; st.hid[at] = 0; st.tag[at] = 0;
    st.prio[at] = 0; st.lost[at] = 0; st.det[at] = 0; st.fin[at] = INFINITY; st.off[at] = 0.0; st.dline[at] = INFINITY;
  }
}

// second pass: episode / counter update, after every robot thread read the old episode
__global__ void nr_reset_rows_kernel(int E, const uint8_t* mask, int64_t* episode, int64_t* ctr) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  if (mask != nullptr && mask[e] == 0) return;
  episode[e] += 1;
  ctr[e] = 0;
}

__global__ void rng_draw_kernel(int E, int n, uint32_t s0, uint32_t channel, uint32_t stream, const int64_t* env_id,
                                const int64_t* episode, const int64_t* ctr, int normal, float* out, float two_pi) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)E * n) return;
  const long long e = i / n;
  const uint32_t j = (uint32_t)(i % n);
  const uint32_t base = key_stream(key_env(s0, env_id[e], episode[e], channel, ctr != nullptr ? ctr[e] : 0), stream);
  out[i] = normal ? normal_at(base, j, two_pi) : uniform_at(base, j);
}

}  // namespace inb

extern "C" int inb_nr_reset(const InbResetArgs* args, void* cuda_stream) {
  if (args == nullptr) return -1;
  const InbResetArgs& a = *args;
  if (a.E <= 0) return 0;
  if (a.R < 1 || a.S < 1 || a.S > INB_MAX_S || a.P < 1 || a.P > INB_MAX_P || a.F < 1 || a.F > INB_MAX_F) return -2;
  if (a.rician && (a.s.spec == nullptr || a.s.k_lin == nullptr)) return -3;
  cudaStream_t s = (cudaStream_t)cuda_stream;
  const long long total = (long long)a.E * a.R;
  inb::nr_reset_kernel<<<(unsigned)((total + 127) / 128), 128, 0, s>>>(a);
  inb::nr_reset_rows_kernel<<<(a.E + 127) / 128, 128, 0, s>>>(a.E, a.mask, a.episode, a.rng_ctr);
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? 0 : -100 - (int)err;
}

extern "C" int inb_rng_draw(int32_t E, int32_t n, uint32_t s0, uint32_t channel, uint32_t stream,
                            const int64_t* env_id, const int64_t* episode, const int64_t* ctr, int32_t normal,
                            float* out, void* cuda_stream) {
  if (E <= 0 || n <= 0) return 0;
  if (env_id == nullptr || episode == nullptr || out == nullptr) return -1;
  const long long total = (long long)E * n;
  inb::rng_draw_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)cuda_stream>>>(
      E, n, s0, channel, stream, env_id, episode, ctr, normal, out, 6.28318548202514648438f);
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? 0 : -100 - (int)err;
}
