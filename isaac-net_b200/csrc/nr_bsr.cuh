// The 5G-LENA SR / BSR grant pipeline of the uplink MAC (ul_grant_model = "bsr"; UlMac, isaac_net/core/mac_ul.py:
// 262-329), one robot per thread.  Instead of the lumped SR grant, the gNB schedules from its estimate of the robot's
// buffer: an SR earns a bootstrap grant of sr_boot_bytes after sr_boot_slots, every PUSCH carries a buffer-status
// report that reaches the gNB bsr_delay slots later (at most INB_BSR_DEPTH in flight; the latest matured one sets the
// estimate, quantized to the short-BSR levels plus a header), each new TB lowers the estimate by its size, and a TB
// that drains the buffer leaves an RLC header residue hidden from the reports until new data arrives or the RLC timer
// reports it.
//
// The state lives in global memory ([E,R] and [E,R,INB_BSR_DEPTH], InbState.bsr_*), read and written at the SR
// opportunities and UL slots only, so the MAC kernel's register budget does not carry it across the slot loop.
#pragma once
#include <cstdint>

#include "nr_common.cuh"

namespace inb {

// Upper bounds (bytes) of the 64 short-BSR buffer-size levels of 3GPP TS 38.321 Table 6.1.3.1-1 as
// isaac_net/core/mac_ul.py:38-42 lists them (the last level repeated): the quantized reports decide the grants.
static __constant__ int32_t kBsrLevels[64] = {
    0,     10,    12,    14,    17,    19,    22,    26,    31,    36,    42,    49,    57,    67,     78,     91,
    107,   125,   146,   171,   200,   234,   274,   321,   376,   440,   515,   603,   706,   826,    967,    1132,
    1326,  1552,  1817,  2127,  2490,  2915,  3413,  3995,  4677,  5476,  6411,  7505,  8787,  10287,  12043,  14099,
    16507, 19325, 22624, 26487, 31009, 36304, 42502, 49759, 58255, 68201, 79846, 93749, 109439, 128125, 150000, 150000};

// UlMac._quant (mac_ul.py:266-270): the first level bound >= min(n, 150000) (torch.searchsorted, left side); 0 for
// n <= 0
__device__ __forceinline__ long long bsr_quant(long long n) {
  const long long x = n < 150000 ? n : 150000;
  int lo = 0, hi = 63;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((long long)kBsrLevels[mid] >= x) hi = mid; else lo = mid + 1;
  }
  return kBsrLevels[lo];
}

// bytes the robot's MAC knows it has: unsent bytes minus the hidden RLC residue, at least 0 (UlMac._visible,
// mac_ul.py:262-264)
__device__ __forceinline__ long long bsr_visible(const InbState& st, long long er, long long enq, long long sent) {
  const long long v = enq - sent - st.bsr_hid[er];
  return v > 0 ? v : 0;
}

// UlMac._arrivals (mac_ul.py:272-278): new data since the last look reveals the residue and re-arms the drain rule
__device__ __forceinline__ void bsr_arrivals(const InbState& st, long long er, long long enq) {
  if (enq > st.bsr_enq_seen[er]) {
    st.bsr_hid[er] = 0;
    st.bsr_hid_until[er] = -1;
    st.bsr_armed[er] = 1;
  }
  st.bsr_enq_seen[er] = enq;
}

// SR opportunity (UlMac._sr_step_bsr, mac_ul.py:280-287): the RLC timer reports an expired residue; an SR goes out
// when the robot has visible data, no estimate, no owed bootstrap grant, no report in flight and no SR pending
__device__ __forceinline__ void bsr_sr_step(const InbState& st, long long er, long long enq, long long sent,
                                            long long g, long long& sr_t) {
  bsr_arrivals(st, er, enq);
  const long long hid = st.bsr_hid[er], hu = st.bsr_hid_until[er];
  if (hid > 0 && hu >= 0 && g >= hu) {
    st.bsr_hid[er] = 0;
    st.bsr_hid_until[er] = -1;
  }
  bool inflight = false;
#pragma unroll
  for (int j = 0; j < INB_BSR_DEPTH; ++j) inflight |= st.bsr_rep_g[er * INB_BSR_DEPTH + j] > -BIGI;
  if (bsr_visible(st, er, enq, sent) > 0 && st.bsr_est[er] <= 0 && !st.bsr_boot[er] && !inflight && sr_t < 0)
    sr_t = g;
}

// Before a UL data slot (UlMac._pre_slot_bsr, mac_ul.py:289-303): an SR old enough owes the bootstrap grant; the
// latest matured report overwrites the estimate (and cancels the owed bootstrap grant); matured reports leave the
// pipeline.  Returns the bytes the scheduler may grant: the estimate plus the owed bootstrap bytes.
__device__ __forceinline__ long long bsr_pre_slot(const InbState& st, const InbParams& p, long long er, long long enq,
                                                  long long g, long long& sr_t) {
  bsr_arrivals(st, er, enq);
  bool boot = st.bsr_boot[er] != 0;
  if (sr_t >= 0 && g - sr_t >= p.sr_boot_slots) {
    boot = true;
    sr_t = -1;
  }
  long long best = -BIGI;
  int jb = 0;
#pragma unroll
  for (int j = 0; j < INB_BSR_DEPTH; ++j) {
    const long long rg = st.bsr_rep_g[er * INB_BSR_DEPTH + j];
    if (rg > -BIGI && g - rg >= p.bsr_delay) {
      if (rg > best) { best = rg; jb = j; }   // report slots are distinct: the max is unique
      st.bsr_rep_g[er * INB_BSR_DEPTH + j] = -BIGI;
    }
  }
  long long est = st.bsr_est[er];
  if (best > -BIGI) {
    const long long v = st.bsr_rep_v[er * INB_BSR_DEPTH + jb];
    est = v > 0 ? bsr_quant(v) + p.bsr_est_hdr : 0;
    boot = false;
    st.bsr_est[er] = est;
  }
  st.bsr_boot[er] = boot ? 1 : 0;
  return est + (boot ? (long long)p.sr_boot_bytes : 0);
}

// Bytes of a new TB of capacity cap_b (UlMac._tb_payload, mac_ul.py:305-316): at most the visible bytes; the TB that
// drains the buffer (armed, no residue yet) holds back an RLC header residue of up to rlc_tail_bytes, reported by the
// RLC timer rlc_tail_slots later
__device__ __forceinline__ long long bsr_tb_payload(const InbState& st, const InbParams& p, long long er,
                                                    long long enq, long long sent, long long cap_b, long long g) {
  const long long vis = bsr_visible(st, er, enq, sent);
  const long long byt = cap_b < vis ? cap_b : vis;
  const long long hid = st.bsr_hid[er];
  if (vis > 0 && cap_b >= vis && hid == 0 && st.bsr_armed[er]) {
    const long long vm = vis - 1 > 0 ? vis - 1 : 0;
    const long long hold = (long long)p.rlc_tail_bytes < vm ? (long long)p.rlc_tail_bytes : vm;
    st.bsr_hid[er] = hid + hold;
    st.bsr_armed[er] = 0;
    if (hold > 0) st.bsr_hid_until[er] = g + p.rlc_tail_slots;
    return byt - hold;
  }
  return byt;
}

// After the slot's TBs (UlMac._post_slot_bsr, mac_ul.py:318-329): a new TB lowers the estimate by its size and uses
// up the bootstrap grant; every PUSCH carries a report of the visible bytes (+ header), into the first free entry of
// the pipeline or over the oldest one
__device__ __forceinline__ void bsr_post_slot(const InbState& st, const InbParams& p, long long er, long long enq,
                                              long long sent, long long g, bool tx, bool tx_new, long long tbs_new) {
  if (tx_new) {
    const long long e2 = st.bsr_est[er] - tbs_new / 8;
    st.bsr_est[er] = e2 > 0 ? e2 : 0;
    st.bsr_boot[er] = 0;
  }
  if (!tx) return;
  const long long vis = bsr_visible(st, er, enq, sent);
  const long long rep = vis > 0 ? vis + p.bsr_hdr : 0;
  int k = -1, kmin = 0;
  long long gmin = BIGI;
#pragma unroll
  for (int j = 0; j < INB_BSR_DEPTH; ++j) {
    const long long rg = st.bsr_rep_g[er * INB_BSR_DEPTH + j];
    if (k < 0 && rg == -BIGI) k = j;
    if (rg < gmin) { gmin = rg; kmin = j; }
  }
  if (k < 0) k = kmin;
  st.bsr_rep_v[er * INB_BSR_DEPTH + k] = rep;
  st.bsr_rep_g[er * INB_BSR_DEPTH + k] = g;
}

// Handover (UlMac.handover, mac_ul.py:247-253): the target cell learns the quantized buffer, the bootstrap grant and
// the reports in flight are dropped
__device__ __forceinline__ void bsr_handover(const InbState& st, const InbParams& p, long long er, long long enq,
                                             long long sent) {
  const long long vis = bsr_visible(st, er, enq, sent);
  st.bsr_est[er] = vis > 0 ? bsr_quant(vis + p.bsr_hdr) + p.bsr_est_hdr : 0;
  st.bsr_boot[er] = 0;
#pragma unroll
  for (int j = 0; j < INB_BSR_DEPTH; ++j) st.bsr_rep_g[er * INB_BSR_DEPTH + j] = -BIGI;
}

}  // namespace inb
