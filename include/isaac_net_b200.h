/*
 * isaac_net_b200 C ABI: the B200 (sm_100a) NR uplink control-step engine of isaac-net, level "L2".
 *
 * Plain C types only (device pointers, sizes, a CUDA stream as void*): any host language can bind it (ctypes, cgo,
 * JNI, N-API).  Every buffer is owned by the caller, allocated once, updated in place; the entry points never
 * allocate device memory and never synchronize with the host, so a step can be captured in a CUDA graph.
 *
 * Reference interfaces replaced (isaac-net v0.2.0):
 *   inb_nr_step        the slot loop and finish of one control step: NRNet.step / step_rx (isaac_net/core/nr_engine.py
 *                      :613-668) + NRNet._finish (nr_engine.py:843-888), MacLink.slot (isaac_net/core/mac.py:228-508),
 *                      UlMac hooks (isaac_net/core/mac_ul.py:66-236), the traffic enqueue and arrival gate of
 *                      NREngine._inject / _open_gate (isaac_net/core/engine.py:505-573) and the step-dict outputs of
 *                      NREngine.step (engine.py:575-594, 918-960).  It is the seam the Triton backend's launch_step occupies
 *                      (isaac_net/core/nr_triton.py:1104-1167, nr_fast.py:702-752).
 *   inb_nr_reset       the device side of NRNet.reset(env_ids) (nr_engine.py:250-320) and MacLink / FrameQueue reset
 *                      (mac.py:176-189, queues.py:399-407): new episode, counter-RNG reset draws (initial fading,
 *                      Rician phase) and the per-robot state back to its initial values, for a mask of envs.
 *   inb_rng_draw       CounterRNG reset draws (isaac_net/core/proto/rng.py:116-161, rng_triton.launch_draw): uniforms
 *                      or Box-Muller normals [E, n] keyed by (seed, env, episode, channel, counter, stream).
 *   inb_traffic_step   TrafficGen.step (isaac_net/core/traffic.py:408-430) with _Stream._step (traffic.py:301-365) for
 *                      periodic, video and bursty models: the step's arrivals [E,R,M] from the engine's
 *                      torch.Generator stream (CUDA Philox), reproduced draw for draw.
 *   inb_net_obs        the Isaac-side consumer of the step dict: NetModule.step's post-processing
 *                      (isaac_net/isaac/net_module.py:340-374) and NetObs.update (isaac_net/isaac/obs.py:48-87).
 * Status: 0 = launched; negative = invalid arguments (nothing launched).  Kernel-side faults are reported in the
 * int32 device status word `status` (0 = ok), which the host reads only when it asks for it.
 */
#ifndef ISAAC_NET_B200_H
#define ISAAC_NET_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INB_ABI_VERSION 17
#define INB_MAX_C 3       /* cells (more need an ordered interference sum) */
#define INB_MAX_S 32      /* RBGs per carrier */
#define INB_MAX_P 32      /* HARQ processes */
#define INB_MAX_F 128     /* frame slots per robot (inb_net_obs: 64) */
#define INB_MAX_M 64      /* traffic arrivals per robot per step */
#define INB_MAX_MCS 32
#define INB_MAX_ROWS 128  /* scheduled slots per control step */
#define INB_MAX_KF 32     /* plane waves per shadowing field */
#define INB_BLK_REGIONS 4 /* blockage model A regions per env (TR 38.901 Sec. 7.6.4.1: K = 4) */
#define INB_CDF_STRIDE 64 /* blockage CDF table: entries per coarse bucket of the two-level search */
#define INB_NCTR 64       /* per-env counter words (int64) */
#define INB_BSR_DEPTH 4   /* buffer-status reports in flight per robot (ul_grant_model = "bsr") */

/* counter words of InbStepArgs.ctr (per env, int64), MacLink.ctr / ntx_hist / rv_tx / rv_fail (mac.py:116-126) */
enum {
  INB_CTR_TB_NEW = 0, INB_CTR_TB_RETX, INB_CTR_TB_OK, INB_CTR_TB_FAIL, INB_CTR_EXHAUST, INB_CTR_BYTES_OK,
  INB_CTR_BYTES_NEW, INB_CTR_NEW_WHILE_PENDING, INB_CTR_PRB_USED, INB_CTR_LOST_FRAMES,
  INB_CTR_TB_BYTES = 10, INB_CTR_TB_EMPTY, INB_CTR_RETX_BLOCK,   /* with InbParams.lena_ctr (mac.py:492-493, 299) */
  INB_CTR_NTX_HIST = 16, INB_CTR_RV_TX = 32, INB_CTR_RV_FAIL = 48
};

/* Per-robot state, reference layouts and dtypes ([E,R], [E,R,S], [E,R,P], [E,R,F]); bool = uint8.  With C > 1 cells
 * the fading state and the Rician phasor have a cell axis after R ([E,R,C,S,2], [E,R,C,2], [E,R,C]). */
typedef struct {
  int64_t *sent, *floor_, *bsr, *sr_t, *last_tx, *enq;     /* [E,R] */
  float *olla, *avg;                                       /* [E,R] */
  float *csi;                                              /* [E,R,S] */
  float *h;                                                /* [E,R,(C,)S,2] AR(1) fading state */
  float *spec, *k_lin;                                     /* Rician: [E,R,(C,)2] phasor, [E,R,(C)] K (NULL: Rayleigh) */
  int64_t *h_state, *h_lo, *h_hi, *h_ready, *h_ntx, *h_mcs, *h_tbs, *h_nsb;   /* [E,R,P] */
  float *h_comb;                                           /* [E,R,P] */
  int64_t *cap, *start, *end_, *cls, *hid, *tag, *prio;    /* [E,R,F] */
  uint8_t *lost, *det;                                     /* [E,R,F] */
  double *fin, *off, *dline;                               /* [E,R,F] */
  /* several cells (NULL with one): CellAssociation (serving cell, A3 candidate and its count in slots, end slot of
   * the handover interruption, handovers), initial association pending per env, the gNBs' N+I per PRB (mW) */
  int64_t *serv, *a3_cand, *a3_cnt, *ho_end, *n_ho;        /* [E,R] */
  uint8_t *pending;                                        /* [E] */
  float *ni_ul;                                            /* [E,C,S] */
  float *last_nprb;             /* [E,R] PRBs of the robot's last PUSCH (ul_amc_alloc = "previous"; NULL otherwise) */
  /* ul_grant_model = "bsr" (NULL otherwise), UlMac's BSR_STATE (isaac_net/core/mac_ul.py:45-50): the gNB's buffer
   * estimate, the bootstrap grant owed after an SR, the reports in flight (value, slot sent; -2^62 = empty), the RLC
   * header residue hidden from the reports and the slot its timer reports it, the queue size last seen, and whether
   * new data arrived since the last buffer-draining TB */
  int64_t *bsr_est;                                        /* [E,R] */
  int64_t *bsr_rep_v, *bsr_rep_g;                          /* [E,R,INB_BSR_DEPTH] */
  int64_t *bsr_hid, *bsr_hid_until, *bsr_enq_seen;         /* [E,R] */
  uint8_t *bsr_boot, *bsr_armed;                           /* [E,R] */
} InbState;

/* Step outputs (the step dict of NREngine.step), [E,R,F] unless noted. */
typedef struct {
  uint8_t *delivered, *timed_out, *dropped, *deadline_miss;
  int64_t *cap, *cls, *arrival_slot, *tag, *priority, *bytes;
  float *delay;
  double *arrival;
  int64_t *newest, *queue_len, *gen_accepted, *gen_bytes;  /* [E,R] */
  float *queue_bytes, *sinr_db;                            /* [E,R] */
  float *pathgain;                                         /* [E,R,C] path gain of every link (dB) */
  uint8_t *det_env;                                        /* [E] */
  int64_t *serving_cell;                                   /* [E,R] (0 with one cell; required with C > 1) */
  /* obstacle outputs of the serving link (NULL: not produced; only with blockage and poses through the radio) */
  uint8_t *blocked;                                        /* [E,R] a blockage region is on the direct path */
  uint8_t *los;                                            /* [E,R] LOS state (InbParams.los_const) */
  /* downlink finish (InbStepArgs.dl): timed out or dropped this step, and generated by a DL traffic model (cls < 0),
   * [E,R,F]; every output of a DL call may be NULL (not produced) */
  uint8_t *lost_any, *generated;
} InbOutputs;

/* Traffic arrivals of this step [E,R,M] (TrafficGen.step, sorted by slot), or M = 0. */
typedef struct {
  const uint8_t *valid, *det;
  const float *nbytes;
  const int64_t *slot, *tag, *prio;
  const double *dline;
} InbArrivals;

/* Static tables (built once per engine on the device). */
typedef struct {
  const float *bler;            /* [M, C, G] code-block BLER */
  const float *thr_ref;         /* [M] 10 % BLER SINR of a 10-PRB RBG */
  const float *se, *beta, *rate;/* [M] spectral efficiency, EESM beta, code rate (float32 as the reference) */
  const float *w, *lw, *lw10;   /* [S] PRBs per RBG, log(w), 10 log10(w / snr_ref_prbs) */
  const int32_t *la_tbs;        /* [NPRB+1, M] TBS (bits) of the data-slot symbols */
  const int32_t *la_i0;         /* [NPRB+1, M] BLER-table code-block index */
  const float *la_wi, *la_ncb;  /* [NPRB+1, M] code-block interpolation weight, number of code blocks */
  const float *fk, *fphi;       /* radio shadowing plane waves: [C,E,K,2], [C,E,K] (NULL: pathgain input) */
  const float *gnb;             /* [C,2] gNB positions */
} InbTables;

/* Scalars of the step; float values are already rounded to float32 exactly as torch rounds python scalars. */
typedef struct {
  int32_t E, R, S, P, F, M, MCS, mcs_max, C_axis, G_axis, nprb, N, K_rows, Kf;
  int64_t T;                    /* global control step */
  int32_t rows[INB_MAX_ROWS][4];/* schedule: (rel, UL data symbols, SR opportunity, fading update) */
  float rowf[INB_MAX_ROWS][2];  /* per row: rho^dt, sqrt(1 - rho^2) of the AR(1) fading update (float32) */
  int32_t sched;                /* 0 pf, 1 maxci, 2 rr */
  int32_t thr_mono;             /* thr_ref is non-decreasing: the per-RBG MCS lookup may binary-search */
  int32_t olla_on, phr_cap, retx_priority, comb_cc, harq_drop, purge, fading, rician, radio;  /* flags */
  int32_t sr_delay, ul_rtt, rlc_retx, max_tx, tb_oh, timeout;
  int32_t dmrs, oh, ref_prbs;
  uint32_t s0;                  /* seed key */
  float inv_sqrt2;              /* float32(1) / float32(sqrt(2)): torch's CUDA division by a python scalar */
  float ul_ref0, noise_prb, ue_tx, sub_noise;   /* ul_ref = (ul_ref0 + pg) - noise_prb; sinr = (pg + ue_tx) - sub_noise */
  float phr_min, olla_up, olla_dn, pf_a, pf_b, target, inv_S;
  float s0_snr, inv_ds, c0_cbs, inv_dc;         /* BLER grid: first SNR, 1/step; first CBS, 1/step */
  double proc_off;              /* proc_offset_ms / control_step_ms */
  double ctl_ms;                /* control_step_ms */
  double inv_N_d;               /* 1.0 / slots_per_step (float64) */
  float inv_ref_prbs;           /* float32(1) / float32(snr_ref_prbs) */
  /* radio: tr38901 (0 UMi, 1 UMa, forced LOS) or log_distance (2) */
  int32_t radio_model;
  float h_bs, h_ut, dbp, fc_term, pl_a, pl_n1, pl_b_term, sigma_sf, amp, hh2;
  float pl_const, pl_10n;
  /* several cells (C = 1: unused) */
  int32_t C;                    /* cells */
  int32_t ttt, ho_int;          /* A3 time-to-trigger and handover interruption, slots */
  int32_t has_floor, ho_flush, pc_on;
  float a3_off, a3_hyst, floor_rx;   /* A3: best > (serving + offset) + hysteresis [and best >= floor_rx] */
  float noise_mw;               /* noise per PRB at a gNB (mW, float32) */
  float ue_tx_ref;              /* float32(ue_tx_dbm - 10 log10(snr_ref_prbs)) (float64 on the host, as python) */
  float ref_db;                 /* 10 log10(snr_ref_prbs) */
  float pc_p0, pc_alpha;        /* fractional UL power control: backoff = ue_tx - (P0 + alpha (ue_tx - RSRP)) */
  float li_alpha, li_beta;      /* N+I filter: ni = alpha ni_now + beta ni (beta = float32(1 - alpha)) */
  int32_t los_const;            /* value of the `los` output (the forced tr38901 LOS state) */
  int32_t pf_rbg;               /* pf_update = "rbg": the PF metric of RBG s uses the average moved by the bytes granted so
                                   far in the slot, and the average update uses the new TBs' bytes (mac.py:326-330,
                                   526-555) */
  int32_t pf_freeze;            /* pf_avg_idle = "freeze": only robots with new data to schedule update their average */
  int32_t field_fma;            /* plane-wave phase k . x as fma(y, k_y, x k_x) (1) or x k_x + y k_y rounded twice (0):
                                   the rounding of the reference's CPU einsum, which takes its BLAS path (fused) when
                                   2 R C K >= 400 (C fields of K waves) and its plain loop (two roundings) below */
  int32_t tdma;                 /* ul_retx_sched = "tdma": one retransmission per slot and cell, the oldest NACK first
                                   (lowest robot on ties), and no new data in a cell that has one (mac.py:279-299) */
  int32_t amc_prev;             /* ul_amc_alloc = "previous": the new TB's MCS is chosen for the PRB count of the
                                   robot's last PUSCH (s.last_nprb, this grant's when 0), its TBS for this grant
                                   (mac.py:393-400, 484) */
  int32_t lena_ctr;             /* 5G-LENA MAC switches on: also count tb_bytes, tb_empty, retx_block (mac.py:119-121) */
  /* ul_grant_model = "bsr": the SR / BSR grant pipeline (mac_ul.py:262-329) replaces the lumped SR grant; slots after
   * an SR until the bootstrap grant, its bytes, the report delay, the RLC timer; header bytes of a report, of the
   * gNB's estimate, and the RLC residue a buffer-draining TB leaves behind */
  int32_t bsr_on, sr_boot_slots, sr_boot_bytes, bsr_delay, rlc_tail_slots, bsr_hdr, bsr_est_hdr, rlc_tail_bytes;
  /* downlink (dl = True, one cell; InbStepArgs.dl): the fading launch also writes the gain of every row that carries
   * DL data or a CQI report, as gain row n_ul_rows + 1 + j (j = rows_dl[k][3], the row's index among those rows);
   * per row: DL data symbols (0 = none), CQI report, HARQ-ACK slot + gnb_proc_slots relative to the step's first slot,
   * DL gain-row index or -1 */
  int32_t dl_on, n_ul_rows, n_dl_rows;
  int32_t rows_dl[INB_MAX_ROWS][4];
  /* the DL call's link-adaptation tables: la_sets stacked [NPRB+1, M] sets (one per DL data-symbol count: a D slot's
   * and, with special_dl_data, an S slot's), dl_nsym_tab[nsym] = the set of a slot with nsym DL data symbols */
  int32_t la_sets;
  int32_t dl_nsym_tab[16];
  /* ul_power = "whole_band" (UlMac._sched_estimate / _split, mac_ul.py:154-180; MacLink's AMC, mac.py:393-400): a
   * fixed PSD over the carrier, so the power split of every grant is wb_db = float32(10 log10(nprb / snr_ref_prbs))
   * (raised to the power-control backoff where that is larger); the scheduler estimate uses the same split (InbTables.
   * lw10 holds wb_db on every RBG, and there is no PHR cap); with amc_prev the MCS is chosen over the whole band. */
  int32_t whole_band;
  float wb_db;
} InbParams;

/* Radio launch (channel "radio_map" and / or blockage model A): ahead of the fading, one thread per robot computes
 * the path gain of every link into `pg` and the blocked bits into `blk`, and the MAC reads them in place of its own
 * tr38901 / log-distance evaluation.  RadioMap._bilinear (isaac_net/core/channels/radio_map.py:101-115) and
 * BlockageA.loss_db (isaac_net/core/channels/blockage.py:195-221), with the clock advance of RadioMC._blockage_db
 * (isaac_net/core/radio.py:168-174). */
typedef struct {
  int32_t on;                   /* 0: no radio launch (the MAC evaluates the channel itself, or reads pathgain_in) */
  int32_t map_on;               /* path gain from the radio map (else the tr38901 / log-distance formula of InbParams
                                   with the shadowing fields of InbTables) */
  int32_t H, W;                 /* map grid */
  float x0, y0, sx, sy;         /* float32(x0), float32(y0), float32((W-1)/(x1-x0)), float32((H-1)/(y1-y0)) */
  float wm1, hm1, wm2, hm2;     /* W-1, H-1, W-2, H-2 */
  const float *map;             /* [C, H*W] path gain (dB) */
  int32_t blockage;             /* blockage model A on */
  int32_t Kb;                   /* plane waves per region field (<= INB_MAX_KF) */
  int32_t n_table;              /* CDF entries: a multiple of INB_CDF_STRIDE, at most 1024 * INB_CDF_STRIDE */
  float amp_b;                  /* float32(sqrt(2 / Kb)) */
  float ck;                     /* float32(pi / lambda * r) of eq. 7.6-23 */
  float max_db;                 /* cap of the summed loss (blockage_max_db) */
  float h_ut, h_bs;             /* antenna heights (m) */
  float dt;                     /* float32(control_step_ms * 1e-3): clock advance per step (s) */
  float u_den;                  /* float32(n_table + 1) */
  int32_t fma_b;                /* region-field phase rounding, as InbParams.field_fma: fused when 2 R 4 Kb >= 400 */
  const float *bk, *bphi;       /* region fields [4, E, Kb, 2] (rad/m), [4, E, Kb] */
  const float *xk, *yk;         /* [E, 4] azimuth / elevation spans (deg) */
  const float *vel;             /* [E, 2] blocker drift velocity (m/s) */
  float *t;                     /* [E] blockage clock (s), advanced by dt in every step */
  const float *table;           /* [n_table] sorted samples of the unit sum-of-cosines marginal */
  float *pg;                    /* [E, R, C] out: path gain of every link (dB) */
  uint8_t *blk;                 /* [E, R] out: bit c = a region is on the direct path to cell c */
} InbRadio;

typedef struct InbStepArgs_ {
  InbParams p;
  InbState s;
  InbOutputs o;
  InbArrivals a;
  InbTables t;
  const float *pos;             /* [E,R,2] poses (radio) or NULL */
  const float *pathgain_in;     /* [E,R] dB path gain (teacher forcing / SNR input) or NULL */
  const float *ul_ref_in;       /* [E,R,S] per-RBG reference SINR input (snr_db=) or NULL */
  const int64_t *env_id, *episode;   /* [E] counter-RNG keys */
  int64_t *rng_ctr;             /* [E] STEP call counter (incremented at the end of the step) */
  const int64_t *epoch;         /* [E] */
  const int64_t *last_hid;      /* [E] */
  int64_t *ctr;                 /* [E, INB_NCTR] counters, accumulated */
  int32_t *status;              /* device status word */
  const int64_t *T_dev;         /* if set, the global control step is read from device memory (CUDA-graph replay) */
  int64_t *trace;               /* optional per-slot trace [K_rows, E, R, 8] (NULL = off): bsr after the SR grant,
                                   need, won RBG mask, new-TB MCS, flags (has_rx | new_el << 1 | tx_rx << 2 |
                                   tx_new << 3 | ok << 4), send pointer after the slot, PHR cap, bits of `left` */
  float *gain;                  /* scratch float32 (n_ul = UL rows of the step): one cell [n_ul + 1, E*R, S], row 0 =
                                   the CSI before the step, row u + 1 = the fading gain (dB) of the u-th UL row;
                                   C > 1 cells [n_ul, E*R, C, S], row u = the gain of every link in UL row u */
  int64_t gain_cap;             /* elements available at `gain` */
  const int64_t *o_base;        /* if set, every pointer in `o` is a byte offset from the address stored here (so a
                                   captured CUDA graph can write each step's outputs into a new block) */
  InbRadio rm;                  /* radio launch (rm.on = 0: none) */
  const int64_t *det_hid;       /* [E] hypothesis id that det_env checks this step, or NULL = last_hid (the legacy
                                   step(t, snr, cur_hid) checks cur_hid without making it the enqueue's last_hid) */
  int32_t phases;               /* 0: the whole step; else a bit mask of the launches of this call: 1 = radio,
                                   2 = fading, 4 = MAC and finish.  Radio and fading need no arrivals and not each
                                   other, so a caller may run them on two streams beside the step's traffic arrivals
                                   and the MAC phase after all of them. */
  /* the downlink link of the step (p.dl_on; NULL = uplink only): a host-memory InbStepArgs for the DL MAC and finish
   * launches, which run after the fading and before the uplink MAC (the uplink MAC advances rng_ctr): its p carries
   * the DL MCS cap, the DL reference SINR constants (ul_ref0 = float32(gnb_tx_dbm - 10 log10(nprb)), noise_prb = the
   * UE's noise per PRB), no PHR cap, TDMA, previous-PRB AMC or BSR; s the DL link's state (csi = the CQI estimate), o
   * the DL outputs (newest, queue_len and the dl_* frame outputs; gen_accepted / gen_bytes = gen_dl_*), a the DL
   * arrivals, ctr the DL counters; the rest as this struct (DlMac, isaac_net/core/mac_dl.py:1-49) */
  const struct InbStepArgs_ *dl;
} InbStepArgs;

/* One control step of the NR uplink engine: the radio (rm.on), fading, MAC and finish launches, on `cuda_stream`.
 * Replaces the slot loop and finish of NRNet.step / step_cells (isaac_net/core/nr_engine.py:634-668, 718-835,
 * 843-888) with MacLink.slot (mac.py:228-508), the traffic enqueue and gate of NREngine.step (engine.py:505-573) and
 * the seam of the Triton backend's launch_step (nr_triton.py:1104-1167).  With rm.on and pathgain_in NULL the radio launch evaluates the poses and the MAC reads rm.pg; a pathgain_in
 * skips it.  -11: a radio pointer or size is missing or out of range, or o.blocked is set without the launch.
 * -12: p.bsr_on without the InbState.bsr_* buffers (or a negative pipeline delay).
 * -13: p.dl_on with several cells, without InbStepArgs.dl, or with DL args / DL rows that do not fit the step. */
int inb_nr_step(const InbStepArgs *args, void *cuda_stream);

/* inb_nr_step whose MAC launches also wait for `mac_wait_event` (a cudaEvent_t recorded by the caller, or NULL),
 * while the radio and fading launches do not: a caller that produces the step's arrivals on another stream
 * (NREngine's traffic generation, engine.py:505-573) lets them run beside the fading, in one call.  No counterpart in
 * the reference (its step is one sequence of torch ops on one stream). */
int inb_nr_step_after(const InbStepArgs *args, void *cuda_stream, void *mac_wait_event);

/* inb_nr_step for callers that cannot hand the library a scratch buffer: the gain rows live in a fixed device array
 * inside the library (INB_NOALLOC_GAIN_MAX float32 elements per device), so `gain` / `gain_cap` are ignored and
 * nothing is allocated at call time.  No counterpart in the reference (its torch backends allocate per call).
 * The array is 128 MiB of device memory on each device where this entry point has been called, held until exit; it
 * sits in a module of its own, so processes that never call this entry point do not load it.
 *   -10: the step's gain rows exceed INB_NOALLOC_GAIN_MAX: (UL rows + 1) x S x E x R with one cell, UL rows x C x S x
 *        E x R with C > 1 cells (use inb_nr_step with a caller buffer); checked only when the call's phases run
 *        the fading or the MAC launch;
 *   -8 / -9: no current CUDA device / the array's device address could not be resolved.
 * The array's address is resolved on the first call on each device: make that call before capturing a CUDA graph.
 * The array needs no initial value (each step writes every row it reads), but all calls on one device share it, so
 * calls on one device must not overlap: issue them on one stream (or order the streams). */
#define INB_NOALLOC_GAIN_MAX (1 << 25)
int inb_nr_step_noalloc(const InbStepArgs *args, void *cuda_stream);

/* Replaces the device work of NRNet.reset(env_ids) (nr_engine.py:250-320), MacLink.reset and FrameQueue.reset
 * (mac.py:176-189, queues.py:70-80).
 * Reset the envs of mask [E] (uint8; NULL = all): episode += 1, STEP counter = 0, per-robot state to its initial
 * values, fading state h = N(0,1)/sqrt(2) draws (site H0, element ((r C + c) S + s) 2 + re/im), Rician phasor (site
 * KPHI, element r C + c) and K; with C > 1 cells also the association (pending for the next step) and N+I. */
typedef struct {
  int32_t E, R, S, P, F;
  uint32_t s0;
  int32_t rician;
  float k_lin0, inv_sqrt2, two_pi;
  const uint8_t *mask;
  const int64_t *env_id;
  int64_t *episode, *rng_ctr;
  InbState s;
  int32_t C;                    /* cells: the fading / Rician state has a cell axis when C > 1 */
  float noise_mw;               /* initial N+I per PRB at each gNB (C > 1) */
} InbResetArgs;
int inb_nr_reset(const InbResetArgs *args, void *cuda_stream);

/* Counter-RNG draws out[E, n] (float32) for every env row: uniforms (normal = 0) or normals (normal = 1), channel
 * RESET or STEP with the given counters.  Replaces CounterRNG._draw (isaac_net/core/proto/rng.py:137-161) and the
 * Triton backend's rng_triton.launch_draw. */
int inb_rng_draw(int32_t E, int32_t n, uint32_t s0, uint32_t channel, uint32_t stream, const int64_t *env_id,
                 const int64_t *episode, const int64_t *ctr, int32_t normal, float *out, void *cuda_stream);

/* One generating traffic model (TrafficModel of kind periodic, video or bursty) and its per-robot state [E,R]. */
#define INB_MAX_SRC 8
typedef struct {
  int32_t kind;                 /* 0 periodic, 1 video, 2 bursty */
  int32_t width;                /* arrival columns of this model (max_per_step) */
  int32_t col;                  /* its first column in the [E,R,M] arrivals */
  int32_t nb, loops, burst;     /* bursty: bursts per step, event-loop iterations, messages per burst */
  int32_t gop_n;                /* video: GOP length (0: constant frame size) */
  int32_t det;                  /* the model's det flag */
  int64_t tag, prio;
  double dline;                 /* deadline_ms (inf: none) */
  double size, gop_i, gop_p;    /* message bytes; video I / P frame bytes */
  double period, jitter;        /* periodic / video, ms */
  double on_ms, off_ms, iat;    /* bursty: mean ON / OFF durations, mean inter-burst time, ms */
  const uint8_t *mask;          /* [R] robots the model runs on */
  double *nom, *nxt;            /* periodic / video state: nominal and jittered next emission (ms from step start) */
  int64_t *cnt;                 /*   frames emitted */
  uint8_t *on;                  /* bursty state: ON period, */
  double *t_tog, *t_bur;        /*   next ON/OFF toggle, next burst (ms from step start) */
  int64_t *deferred;            /* scalar: emissions due inside the step that did not fit its columns (accumulated) */
} InbTrafficSource;

/* Arrivals of one control step for E envs x R robots from the engine's traffic torch.Generator (CUDA Philox
 * stream of seed `seed`, offset `off0` before the first step): uniform draw d of step n is element (e R + r) of the
 * float64 torch.rand([E, R]) call at Philox offset off0 + (n ndraws + d) inc, as torch's grid-stride launch of
 * `stride` threads lays it out. */
typedef struct {
  int32_t E, R, M, N, n_src;
  uint64_t seed, off0;
  int64_t stride;               /* threads of torch's uniform launch over E*R elements */
  int64_t inc;                  /* Philox offset advance of one [E,R] draw */
  int64_t ndraws;               /* [E,R] draws per step, all models */
  double step_ms, inv_slot_ms;  /* control step; float64 1 / slot duration (torch's CUDA division by a scalar) */
  int64_t *calls;               /* [E,R] steps generated so far (read, then incremented) */
  InbTrafficSource src[INB_MAX_SRC];
  uint8_t *valid, *det;         /* out [E,R,M], sorted by (slot, column); invalid entries last */
  float *nbytes;
  int64_t *slot, *tag, *prio;
  double *dline;
  /* counter = 1: the opt-in counter-keyed stream instead of the torch.Generator one (no counterpart in the
   * reference, whose arrivals depend on how the envs are split over engines): uniform d of a robot's step is
   * ((h0 >> 5) 2^26 + (h1 >> 6)) 2^-53 with h0, h1 the counter-RNG element hashes 2r, 2r + 1 of stream d under the
   * key (s0, env_id[e], episode[e], channel 0x54, calls[e,r]), so it depends on the global env id, not on the shard */
  int32_t counter;
  uint32_t s0;
  const int64_t *env_id, *episode;   /* [E] */
} InbTrafficArgs;
int inb_traffic_step(const InbTrafficArgs *args, void *cuda_stream);

/* Store two int64 values at dst[0], dst[1] in stream order (e.g. the control step and the output block address that
 * a captured step reads through T_dev / o_base).  No counterpart in the reference (its graph backend captures
 * torch ops around static tensors, cuda_graph.py:19-30). */
int inb_store2(int64_t *dst, int64_t v0, int64_t v1, void *cuda_stream);

/* Network observation packing of one control step: what isaac-net's Isaac-side module does with the engine's step
 * dict on the engine's own radio.  Replaces NetModule.step's post-processing (isaac_net/isaac/net_module.py:340-374:
 * last_cap = max(last_cap, newest), aoi_s = (t + 1 - last_cap).float() * step_dt, delay_s = delay * step_dt,
 * rsrp_dbm = sinr_db + noise, blocked / los defaults, tag_delivered) and NetObs.update (isaac_net/isaac/obs.py:48-87:
 * the delay history and the selected features, normalised, into x [E,R,dim]).  Inputs are the step dict's device
 * tensors; last_cap [E,R] and hist [E,R,K] are the caller's persistent state, updated in place.  Outputs left NULL
 * are not written.  The float inputs of the normalisation are the float32 values torch uses on a CUDA device:
 * step_dt and noise_db rounded to float32, inv_* = 1.0f / float32(divisor).  -2: sizes out of range; -3: a required
 * pointer is NULL; -4: a feature column beyond dim. */
typedef struct {
  int32_t E, R, F, G, K, dim;   /* envs, robots, frame slots, gNBs (one-hot width), delay-history length, x width */
  int32_t off_mask, off_delay, off_aoi, off_qlen, off_qbytes, off_sinr, off_rsrp, off_serv, off_last, off_hist,
          off_blocked, off_los;   /* first column of each feature in x (isaac/config.py OBS_FEATURES), -1 = off */
  float step_dt, inv_ts, inv_F, inv_qbytes, inv_db, noise_db;
  const int64_t *newest, *t, *queue_len, *serving;   /* [E,R], [E], [E,R], [E,R] */
  const float *queue_bytes, *sinr_db, *delay;        /* [E,R], [E,R], [E,R,F] (control steps, NaN = none) */
  const uint8_t *delivered, *blocked, *los, *det_env; /* [E,R,F]; [E,R] or NULL (defaults); [E,R] or NULL; [E] */
  const int64_t *cap, *cur_tag;                      /* [E,R,F]; [E] or NULL (no tag_delivered) */
  int64_t *last_cap;            /* [E,R] state: newest capture step delivered this episode */
  float *hist;                  /* [E,R,K] state: delay history, newest first */
  int64_t *last_cap_out;        /* [E,R] */
  float *aoi_s, *delay_s, *rsrp_dbm, *x;             /* [E,R], [E,R,F], [E,R], [E,R,dim] */
  uint8_t *delivered_any, *blocked_out, *los_out, *tag_delivered;   /* [E,R], [E,R], [E,R], [E] */
} InbObsArgs;
int inb_net_obs(const InbObsArgs *args, void *cuda_stream);

/* ABI version of the loaded library (INB_ABI_VERSION).  No counterpart in the reference. */
int inb_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* ISAAC_NET_B200_H */
