// Radio launch of the NR step (InbStepArgs.rm): the path gain of every robot-cell link from a precomputed radio map
// or the tr38901 / log-distance formula, minus TR 38.901 blockage model A, into rm.pg [E,R,C], with the blocked bits
// of every link into rm.blk [E,R].  The MAC kernel reads both in place of its own channel evaluation.
//
// One thread per robot; a block holds whole envs (epb = floor(256 / R) envs of R robots), so the per-env blockage
// clock can be advanced by one thread after every robot of the env has read it.
//
// Reference: RadioMC.rx_dbm (isaac_net/core/radio.py:238-263), RadioMap._bilinear (channels/radio_map.py:101-115),
// BlockageA.loss_db / advance (channels/blockage.py:190-221), PlaneWaveField / eval_plane_waves and
// uniform_from_field (channels/fields.py:61-64, 103-106).  Every tensor op of the reference is one rounded operation
// here, in its order; the transcendentals are CUDA's (cosf, atan2f, atanf, log10f), which torch's CUDA kernels call.
#include "nr_common.cuh"

namespace inb {

constexpr float RAD2DEG = 57.295779513082320876798154814105f;   // float32(180 / pi): torch.rad2deg's factor
constexpr float DEG2RAD = 0.017453292519943295769236907684886f;  // float32(pi / 180): torch.deg2rad's factor
constexpr float PI_F = 3.14159265358979323846f;                  // float32(math.pi)
constexpr float HALF_PI_F = 1.57079632679489661923f;             // float32(math.pi / 2)
constexpr int NREG = INB_BLK_REGIONS;
constexpr int MAX_COARSE = 1024;
constexpr int RADIO_BLOCK = 256;

// F of eq. 7.6-23 with the sign of Table 7.6.4.1-3 (channels/blockage.py:128-133):
// atan(+-(pi/2) sqrt((pi/lambda) r (1/cos(delta) - 1))) / pi, delta clamped at 89.9 deg
__device__ __forceinline__ float angle_f(float delta, bool inside, float ck) {
  const float c = cosf(fm(fminf(fabsf(delta), 89.9f), DEG2RAD));
  const float q = fmaxf(fs(__frcp_rn(c), 1.0f), 0.0f);
  const float a = fm(HALF_PI_F, sqrtf(fm(ck, q)));
  return fdv(atanf(inside ? a : -a), PI_F);
}

// torch.remainder(x, 360) for float: fmod, then + 360 when the remainder is negative
__device__ __forceinline__ float remainder360(float x) {
  float m = fmodf(x, 360.0f);
  if (m != 0.0f && m < 0.0f) m = fa(m, 360.0f);
  return m;
}

__global__ void __launch_bounds__(RADIO_BLOCK) nr_radio_kernel(const InbStepArgs a, int epb) {
  const InbParams& p = a.p;
  const InbRadio& rm = a.rm;
  __shared__ float s_coarse[MAX_COARSE];
  const int R = p.R, C = p.C;
  const int le = threadIdx.x / R, r = threadIdx.x - le * R;
  const long long e = (long long)blockIdx.x * epb + le;
  const bool live = le < epb && e < p.E;
  const int nc = rm.n_table / INB_CDF_STRIDE;
  if (rm.blockage) {   // every INB_CDF_STRIDE-th CDF entry: the first level of the search
    for (int i = threadIdx.x; i < nc; i += blockDim.x) s_coarse[i] = rm.table[(long long)i * INB_CDF_STRIDE];
    __syncthreads();
  }
  float tn = 0.0f;
  if (live) {
    const long long er = e * R + r;
    const float px = a.pos[er * 2], py = a.pos[er * 2 + 1];
    float rx[INB_MAX_C];
#pragma unroll
    for (int cc = 0; cc < INB_MAX_C; ++cc) {
      rx[cc] = 0.0f;
      if (cc >= C) continue;
      if (rm.map_on) {
        // bilinear in dB on the cell's grid, clamped at the border
        const float fx = clampf_t(fm(fs(px, rm.x0), rm.sx), 0.0f, rm.wm1);
        const float fy = clampf_t(fm(fs(py, rm.y0), rm.sy), 0.0f, rm.hm1);
        const float ix = fminf(floorf(fx), rm.wm2), iy = fminf(floorf(fy), rm.hm2);
        const float tx = fs(fx, ix), ty = fs(fy, iy);
        // a NaN pose samples cell (0, 0) (its gain is NaN through tx / ty all the same)
        const int jx = isnan(ix) ? 0 : (int)ix, jy = isnan(iy) ? 0 : (int)iy;
        const float* g = rm.map + (long long)cc * rm.H * rm.W + (long long)jy * rm.W + jx;
        const float v00 = __ldg(g), v01 = __ldg(g + 1), v10 = __ldg(g + rm.W), v11 = __ldg(g + rm.W + 1);
        const float omx = fs(1.0f, tx), omy = fs(1.0f, ty);
        const float out = fa(fm(fa(fm(v00, omx), fm(v01, tx)), omy), fm(fa(fm(v10, omx), fm(v11, tx)), ty));
        rx[cc] = fa(p.ue_tx, out);
      } else {
        const float dx = fs(px, a.t.gnb[cc * 2]), dy = fs(py, a.t.gnb[cc * 2 + 1]);
        const float d2 = fmaxf(sqrtf(fa(fm(dx, dx), fm(dy, dy))), 1.0f);
        const float* fk = a.t.fk + ((long long)cc * p.E + e) * p.Kf * 2;
        const float* fp = a.t.fphi + ((long long)cc * p.E + e) * p.Kf;
        float cs = 0.0f;
        for (int k = 0; k < p.Kf; ++k) {
          const float cv = cosf(fa(wave_phase(px, py, __ldg(fk + 2 * k), __ldg(fk + 2 * k + 1), p.field_fma != 0),
                                   __ldg(fp + k)));
          cs = k == 0 ? cv : fa(cs, cv);
        }
        rx[cc] = formula_rx(p, d2, fm(p.amp, cs));
      }
    }
    if (rm.blockage) {
      // the env clock advances one control step before the loss is evaluated (radio.py:171)
      tn = fa(rm.t[e], rm.dt);
      const float bx = fa(px, fm(rm.vel[e * 2], tn)), by = fa(py, fm(rm.vel[e * 2 + 1], tn));
      // region centre azimuths: 360 u, u = (#{table < z} + 0.5) / (n + 1) of the unit field z at the drifted point
      float z[NREG];
#pragma unroll
      for (int k = 0; k < NREG; ++k) {
        const float* bk = rm.bk + ((long long)k * p.E + e) * rm.Kb * 2;
        const float* bp = rm.bphi + ((long long)k * p.E + e) * rm.Kb;
        float cs = 0.0f;
        for (int m = 0; m < rm.Kb; ++m) {
          const float cv = cosf(fa(wave_phase(bx, by, __ldg(bk + 2 * m), __ldg(bk + 2 * m + 1), rm.fma_b != 0),
                                   __ldg(bp + m)));
          cs = m == 0 ? cv : fa(cs, cv);
        }
        z[k] = fm(rm.amp_b, cs);
      }
      // searchsorted (left): coarse buckets in shared memory, then the bucket's entries, the regions interleaved
      int lo[NREG], hi[NREG];
#pragma unroll
      for (int k = 0; k < NREG; ++k) {
        int l = 0, h = nc;
        while (l < h) {
          const int mid = (l + h) >> 1;
          if (s_coarse[mid] < z[k]) l = mid + 1; else h = mid;
        }
        // l buckets start below z: the answer is in (start of bucket l-1, start of bucket l]
        lo[k] = l == 0 ? 0 : (l - 1) * INB_CDF_STRIDE + 1;
        hi[k] = l == 0 ? 0 : l * INB_CDF_STRIDE;
      }
#pragma unroll
      for (int it = 0; it < 6; ++it) {        // log2(INB_CDF_STRIDE) halvings
#pragma unroll
        for (int k = 0; k < NREG; ++k) {
          if (lo[k] < hi[k]) {
            const int mid = (lo[k] + hi[k]) >> 1;
            if (__ldg(rm.table + mid) < z[k]) lo[k] = mid + 1; else hi[k] = mid;
          }
        }
      }
      float phik[NREG], xk[NREG], yk[NREG];
#pragma unroll
      for (int k = 0; k < NREG; ++k) {
        phik[k] = fm(360.0f, fdv(fa((float)lo[k], 0.5f), rm.u_den));
        xk[k] = rm.xk[e * NREG + k];
        yk[k] = rm.yk[e * NREG + k];
      }
      unsigned bits = 0;
      const float dz = fs(rm.h_bs, rm.h_ut);
#pragma unroll
      for (int cc = 0; cc < INB_MAX_C; ++cc) {
        if (cc >= C) continue;
        // direct path robot -> gNB: azimuth and zenith (deg)
        const float dx = fs(a.t.gnb[cc * 2], px), dy = fs(a.t.gnb[cc * 2 + 1], py);
        const float az = fm(atan2f(dy, dx), RAD2DEG);
        const float hxy = sqrtf(fa(fm(dx, dx), fm(dy, dy)));
        const float zen = fs(90.0f, fm(atan2f(dz, hxy), RAD2DEG));
        const float zr = fs(zen, 90.0f);
        float loss = 0.0f;
        bool hit = false;
#pragma unroll
        for (int k = 0; k < NREG; ++k) {
          const float da = fs(remainder360(fa(fs(az, phik[k]), 180.0f)), 180.0f);
          const float xh = fm(xk[k], 0.5f), yh = fm(yk[k], 0.5f);
          const float a1 = fs(da, xh), a2 = fa(da, xh);
          const float z1 = fs(zen, fa(90.0f, yh)), z2 = fs(zen, fs(90.0f, yh));
          hit = hit || (a1 < 0.0f && a2 > 0.0f && z1 < 0.0f && z2 > 0.0f);
          if (fabsf(da) < xk[k] && fabsf(zr) < yk[k]) {     // eq. 7.6-22 applies inside this window only
            const float f = fm(fa(angle_f(a1, a1 < 0.0f, rm.ck), angle_f(a2, a2 > 0.0f, rm.ck)),
                               fa(angle_f(z1, z1 < 0.0f, rm.ck), angle_f(z2, z2 > 0.0f, rm.ck)));
            const float arg = fmaxf(fs(1.0f, f), 1e-6f);
            loss = fa(loss, fmaxf(fm(-20.0f, log10f(arg)), 0.0f));
          }
        }
        rx[cc] = fs(rx[cc], fminf(loss, rm.max_db));
        bits |= (hit ? 1u : 0u) << cc;
      }
      rm.blk[er] = (uint8_t)bits;
    }
#pragma unroll
    for (int cc = 0; cc < INB_MAX_C; ++cc)
      if (cc < C) rm.pg[er * C + cc] = fs(rx[cc], p.ue_tx);
  }
  if (rm.blockage) {   // every robot of the env has read the clock
    __syncthreads();
    if (live && r == 0) rm.t[e] = tn;
  }
}

int radio_epb(int R) { return R >= RADIO_BLOCK ? 1 : RADIO_BLOCK / R; }

cudaError_t launch_radio(const InbStepArgs& a, cudaStream_t stream) {
  const int epb = radio_epb(a.p.R);
  const long long blocks = ((long long)a.p.E + epb - 1) / epb;
  nr_radio_kernel<<<(unsigned)blocks, epb * a.p.R, 0, stream>>>(a, epb);
  return cudaGetLastError();
}

}  // namespace inb
