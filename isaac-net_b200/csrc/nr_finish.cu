// End of a control step (NRNet._finish, isaac_net/core/nr_engine.py:843-888; MacLink.end_step / compact, mac.py:585-616;
// FrameQueue.remove / floor, queues.py:105-143; the step-dict outputs of NREngine.step, engine.py:575-594, 918-960),
// after the slot loop of the MAC kernel.
//
// One block per env; each robot is served by FW lanes with one frame per lane (FPL = 2 or 4 when F > FW, up to 128
// frames), so every load and store of the [E,R,F] frame arrays is coalesced.  Per frame: delivered / timed-out / dropped masks and the frame
// outputs.  Per robot (segmented shuffles): the in-order pointer, the newest delivered capture, the FIFO compaction
// (kept frames first in order, then the freed slots in index order, each lane fetching its source frame from the
// owning lane's registers), the stream floor, the send pointer, HARQ processes that only hold purged bytes, BSR and the
// queue outputs.  Per env: det_env.
#include <cmath>
#include <cstdint>

#include "nr_common.cuh"

namespace inb {

template <int FW>
struct Seg {  // the FW lanes of one robot inside a warp
  static __device__ __forceinline__ unsigned mask_bits(bool v) {
    const unsigned b = __ballot_sync(0xFFFFFFFFu, v);
    if constexpr (FW == 32) {
      return b;
    } else {
      return (b >> ((threadIdx.x & 31) / FW * FW)) & ((1u << FW) - 1u);
    }
  }
  static __device__ __forceinline__ long long min_ll(long long x) {
#pragma unroll
    for (int o = FW / 2; o > 0; o >>= 1) {
      const long long y = __shfl_xor_sync(0xFFFFFFFFu, x, o, FW);
      x = y < x ? y : x;
    }
    return x;
  }
  static __device__ __forceinline__ long long max_ll(long long x) {
#pragma unroll
    for (int o = FW / 2; o > 0; o >>= 1) {
      const long long y = __shfl_xor_sync(0xFFFFFFFFu, x, o, FW);
      x = y > x ? y : x;
    }
    return x;
  }
  template <typename V>
  static __device__ __forceinline__ V from(V v, int src_lane) {   // lane index within the segment
    return __shfl_sync(0xFFFFFFFFu, v, src_lane, FW);
  }
};

// index of the n-th set bit (0-based; n < popcount(m)) of a 64-bit mask, by halving with population counts
__device__ __forceinline__ int nth_set64(unsigned long long m, int n) {
  unsigned w = (unsigned)m;
  int pos = 0;
  const int c32 = __popc(w);
  if (n >= c32) { n -= c32; w = (unsigned)(m >> 32); pos = 32; }
  const int c16 = __popc(w & 0xFFFFu);
  if (n >= c16) { n -= c16; w >>= 16; pos += 16; }
  const int c8 = __popc(w & 0xFFu);
  if (n >= c8) { n -= c8; w >>= 8; pos += 8; }
  const int c4 = __popc(w & 0xFu);
  if (n >= c4) { n -= c4; w >>= 4; pos += 4; }
  const int c2 = __popc(w & 0x3u);
  if (n >= c2) { n -= c2; w >>= 2; pos += 2; }
  if (n >= (int)(w & 1u)) pos += 1;
  return pos;
}

// bit `i` of a 128-bit frame mask held as two words (the high word stays 0 with 64 frames or fewer)
__device__ __forceinline__ bool bit128(unsigned long long lo, unsigned long long hi, int i) {
  return ((i < 64 ? lo >> i : hi >> (i - 64)) & 1ull) != 0ull;
}
// index of the n-th set bit (0-based) of a 128-bit mask
__device__ __forceinline__ int nth_set128(unsigned long long lo, unsigned long long hi, int n) {
  const int c = __popcll(lo);
  return n < c ? nth_set64(lo, n) : 64 + nth_set64(hi, n - c);
}

template <int FW, int FPL>                     // lanes per robot, frames per lane (F <= FW * FPL)
__global__ void __launch_bounds__(512, 2) nr_finish_kernel(const InbStepArgs A, const int e_begin) {
  const InbParams& p = A.p;
  const InbState& st = A.s;
  const long long ob = A.o_base != nullptr ? *A.o_base : 0;
  InbOutputs o;   // the output pointers of this step (NULL: not produced, e.g. the downlink call's UL-only outputs)
  auto op = [ob](auto* x) { return x != nullptr ? out_ptr(x, ob) : x; };
  o.delivered = op(A.o.delivered); o.timed_out = op(A.o.timed_out);
  o.dropped = op(A.o.dropped); o.deadline_miss = op(A.o.deadline_miss);
  o.cap = op(A.o.cap); o.cls = op(A.o.cls); o.arrival_slot = op(A.o.arrival_slot);
  o.tag = op(A.o.tag); o.priority = op(A.o.priority); o.bytes = op(A.o.bytes);
  o.delay = op(A.o.delay); o.arrival = op(A.o.arrival); o.newest = op(A.o.newest);
  o.queue_len = op(A.o.queue_len); o.queue_bytes = op(A.o.queue_bytes);
  o.det_env = op(A.o.det_env);
  o.lost_any = op(A.o.lost_any); o.generated = op(A.o.generated);
  const int R = p.R, F = p.F, P = p.P;
  const long long e = (long long)e_begin + blockIdx.x;   // one block per env of the launch's range
  const int seg = threadIdx.x / FW, l = threadIdx.x % FW;
  const int segs = blockDim.x / FW;
  const long long T = (A.T_dev != nullptr) ? *A.T_dev : p.T;
  const long long epoch = A.epoch[e], last_hid = A.det_hid != nullptr ? A.det_hid[e] : A.last_hid[e];
  const double lim = da((double)(T + 1), 1e-9);
  bool det_hit = false;
  const int passes = (R + segs - 1) / segs;
  for (int ps = 0; ps < passes; ++ps) {        // same trip count in every lane of the block
    const int r = ps * segs + seg;
    const bool act = r < R;
    const long long er = act ? e * R + r : 0;
    const long long eP = er * P, eF = er * F;
    long long sent = 0, floor_ = 0, enq = 0, bsr = 0;
    if (act) {
      sent = st.sent[er]; floor_ = st.floor_[er]; enq = st.enq[er]; bsr = st.bsr[er];
    }
    // ---- HARQ processes: lane q holds process q (P <= FW)
    const bool hq = act && l < P;
    long long h_hi = 0, h_lo = 0;
    bool pend = false;
    if (hq) {
      pend = st.h_state[eP + l] == 1;
      h_hi = st.h_hi[eP + l];
      h_lo = st.h_lo[eP + l];
    }
    // in-order pointer (MacLink.ack_ptr, mac.py:194-197)
    auto ack_of = [&](bool pd, long long fl, long long sn) {
      long long v = (pd && h_hi > fl) ? (h_lo > fl ? h_lo : fl) : sn;
      v = Seg<FW>::min_ll(v);
      return v < sn ? v : sn;
    };
    const long long ack_end = ack_of(pend, floor_, sent);
    // ---- frames: lane l holds frames l and l + FW
    long long cap[FPL], start[FPL], end_[FPL], cls[FPL], hid[FPL], tag[FPL], prio[FPL];
    double fin[FPL], off[FPL], dline[FPL];
    uint8_t lost[FPL], det[FPL];
    constexpr bool W2 = FW * FPL > 64;   // frame masks need a second word
    unsigned long long gone = 0ull, gone_hi = 0ull;
    long long newest = -1;
#pragma unroll
    for (int j = 0; j < FPL; ++j) {
      const int f = l + j * FW;
      const bool fv = act && f < F;
      const long long at = eF + f;
      cap[j] = fv ? st.cap[at] : -1;
      start[j] = fv ? st.start[at] : 0;
      end_[j] = fv ? st.end_[at] : 0;
      cls[j] = fv ? st.cls[at] : 0;
      hid[j] = fv ? st.hid[at] : 0;
      tag[j] = fv ? st.tag[at] : 0;
      prio[j] = fv ? st.prio[at] : 0;
      lost[j] = fv ? st.lost[at] : 0;
      det[j] = fv ? st.det[at] : 0;
      fin[j] = fv ? st.fin[at] : INFINITY;
      off[j] = fv ? st.off[at] : 0.0;
      dline[j] = fv ? st.dline[at] : INFINITY;
      const bool valid = cap[j] >= 0;
      const bool delivered = valid && fin[j] <= lim;
      const bool timed = p.purge && valid && isinf(fin[j]) && ((T + 1 - cap[j]) >= p.timeout);
      const bool dropped = valid && lost[j] && (end_[j] <= ack_end) && !timed;
      if (delivered && cap[j] > newest) newest = cap[j];
      if (delivered && det[j] && hid[j] == last_hid) det_hit = true;
      if (fv) {
        if (o.delivered) o.delivered[at] = delivered;
        if (o.timed_out) o.timed_out[at] = timed;
        if (o.dropped) o.dropped[at] = dropped;
        if (o.lost_any) o.lost_any[at] = timed || dropped;            // the DL's dl_lost (engine.py:691)
        if (o.generated) o.generated[at] = valid && cls[j] < 0;      // dl_generated (engine.py:694)
        if (o.cap) o.cap[at] = valid ? cap[j] - epoch : -1;
        if (o.cls) o.cls[at] = valid ? cls[j] : 0;
        const float delay = (float)dsb(dsb(fin[j], (double)cap[j]), off[j]);
        if (o.delay) o.delay[at] = delivered ? delay : NAN;
        if (o.arrival) o.arrival[at] = valid ? da((double)(cap[j] - epoch), off[j]) : NAN;
        if (o.arrival_slot) o.arrival_slot[at] = valid ? (long long)rint(dm(off[j], (double)p.N)) : -1;
        if (o.tag) o.tag[at] = valid ? tag[j] : 0;
        if (o.priority) o.priority[at] = valid ? prio[j] : 0;
        if (o.bytes) o.bytes[at] = valid ? end_[j] - start[j] : 0;
        const bool late = delivered && (dm((double)delay, p.ctl_ms) > dline[j]);
        if (o.deadline_miss) o.deadline_miss[at] = late || ((timed || dropped) && isfinite(dline[j]));
      }
      const bool g_ = !fv || delivered || timed || dropped || !valid;
      const unsigned long long gb = (unsigned long long)Seg<FW>::mask_bits(g_);
      if (!W2 || j * FW < 64) gone |= gb << (j * FW);
      else gone_hi |= gb << (j * FW - 64);
    }
    newest = Seg<FW>::max_ll(newest);
    // ---- compaction: surviving frames first (stable), then the freed slots in index order (queues.py:105-110)
    const unsigned long long all = F >= 64 ? ~0ull : ((1ull << F) - 1ull);
    const unsigned long long all_hi = !W2 || F <= 64 ? 0ull : (F >= 128 ? ~0ull : ((1ull << (F - 64)) - 1ull));
    gone &= all;
    gone_hi &= all_hi;
    const unsigned long long keep = ~gone & all, keep_hi = ~gone_hi & all_hi;
    const int n_keep = __popcll(keep) + (W2 ? __popcll(keep_hi) : 0);
    long long floor_new = enq;
#pragma unroll
    for (int j = 0; j < FPL; ++j) {
      const int f = l + j * FW;
      int src = 0;
      if (f < F) {
        if constexpr (W2) src = f < n_keep ? nth_set128(keep, keep_hi, f) : nth_set128(gone, gone_hi, f - n_keep);
        else src = f < n_keep ? nth_set64(keep, f) : nth_set64(gone, f - n_keep);
      }
      const int sl = src % FW, sj = src / FW;
      // every lane takes part in each shuffle; the value comes from register sj of lane sl
      auto pick64 = [&](const long long* v) {
        long long a = Seg<FW>::from(v[0], sl);
#pragma unroll
        for (int jj = 1; jj < FPL; ++jj) {
          const long long b = Seg<FW>::from(v[jj], sl);
          a = sj == jj ? b : a;
        }
        return a;
      };
      auto pickd = [&](const double* v) {
        double a = Seg<FW>::from(v[0], sl);
#pragma unroll
        for (int jj = 1; jj < FPL; ++jj) {
          const double b = Seg<FW>::from(v[jj], sl);
          a = sj == jj ? b : a;
        }
        return a;
      };
      auto pick8 = [&](const uint8_t* v) {
        int a = Seg<FW>::from((int)v[0], sl);
#pragma unroll
        for (int jj = 1; jj < FPL; ++jj) {
          const int b = Seg<FW>::from((int)v[jj], sl);
          a = sj == jj ? b : a;
        }
        return (uint8_t)a;
      };
      const long long c_src = pick64(cap);   // every lane shuffles; the freed slots get cap -1
      const long long n_cap = (W2 ? bit128(gone, gone_hi, src) : ((gone >> src) & 1ull) != 0ull) ? -1 : c_src;
      const long long n_start = pick64(start), n_end = pick64(end_), n_cls = pick64(cls), n_hid = pick64(hid);
      const long long n_tag = pick64(tag), n_prio = pick64(prio);
      const uint8_t n_lost = pick8(lost), n_det = pick8(det);
      const double n_fin = pickd(fin), n_off = pickd(off), n_dline = pickd(dline);
      if (j == 0) {
        const long long s0 = Seg<FW>::from(n_start, 0);
        if (n_keep > 0) floor_new = s0;
      }
      if (act && f < F) {
        const long long at = eF + f;
        st.cap[at] = n_cap; st.start[at] = n_start; st.end_[at] = n_end; st.cls[at] = n_cls; st.hid[at] = n_hid;
        st.tag[at] = n_tag; st.prio[at] = n_prio; st.lost[at] = n_lost; st.det[at] = n_det;
        st.fin[at] = n_fin; st.off[at] = n_off; st.dline[at] = n_dline;
      }
    }
    // ---- stream floor, send pointer, HARQ processes holding only purged bytes (MacLink.compact, mac.py:598-616)
    floor_ = floor_new;
    sent = sent > floor_ ? sent : floor_;
    if (hq && pend && h_hi <= floor_ && h_hi > h_lo) {
      st.h_state[eP + l] = 0; st.h_ready[eP + l] = 0; st.h_ntx[eP + l] = 0; st.h_comb[eP + l] = 0.0f;
      pend = false;
    }
    bsr = bsr < enq - sent ? bsr : enq - sent;
    if (p.bsr_on && act && l == 0) {   // UlMac.compact (mac_ul.py:255-260): the residue never exceeds the unsent bytes
      const long long h = st.bsr_hid[er];
      st.bsr_hid[er] = h < enq - sent ? h : enq - sent;
    }
    const long long qb = enq - ack_of(pend, floor_, sent);
    if (act && l == 0) {
      if (o.newest) o.newest[er] = newest >= 0 ? newest - epoch : -1;
      if (o.queue_len) o.queue_len[er] = n_keep;
      if (o.queue_bytes) o.queue_bytes[er] = (float)(qb > 0 ? qb : 0);
      st.sent[er] = sent;
      st.floor_[er] = floor_;
      st.bsr[er] = bsr;
    }
  }
  const int any = __syncthreads_or(det_hit ? 1 : 0);
  if (threadIdx.x == 0 && o.det_env) o.det_env[e] = any ? 1 : 0;
}

cudaError_t launch_finish(const InbStepArgs& a, cudaStream_t stream, const Range& rg) {
  const InbParams& p = a.p;
  const int FW = (p.P > 16 || p.F > 32) ? 32 : 16;   // lanes per robot: P <= FW, F <= 2 FW
  const int FPL = p.F > 2 * FW ? 4 : (p.F > FW ? 2 : 1);
  int rp = 1;
  while (rp < p.R) rp <<= 1;
  int threads = rp * FW;
  threads = threads < 32 ? 32 : (threads > 512 ? 512 : threads);
  const int n = rg.e1 - rg.e0;
  if (n <= 0) return cudaSuccess;
  if (FW == 16 && FPL == 1)
    nr_finish_kernel<16, 1><<<n, threads, 0, stream>>>(a, rg.e0);
  else if (FW == 16)
    nr_finish_kernel<16, 2><<<n, threads, 0, stream>>>(a, rg.e0);
  else if (FPL == 1)
    nr_finish_kernel<32, 1><<<n, threads, 0, stream>>>(a, rg.e0);
  else if (FPL == 2)
    nr_finish_kernel<32, 2><<<n, threads, 0, stream>>>(a, rg.e0);
  else
    nr_finish_kernel<32, 4><<<n, threads, 0, stream>>>(a, rg.e0);
  return cudaGetLastError();
}

}  // namespace inb
