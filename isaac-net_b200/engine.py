"""NRB200Engine: isaac-net's NR uplink engine (level "L2") with the control step on B200 CUDA kernels.

Drop-in for ``isaac_net.make_engine("L2", E, R, device, config, backend=...)`` on the uplink path: the same contract
API as ``NREngine`` (isaac_net/core/engine.py:319-960): ``reset(env_ids)``, ``submit(t, requests, snr_db=None, *,
tag, priority, deadline_ms)``, ``step(t, x, cur_hid=None, *, snr_db, triggers)`` -> the step dict, ``clock``,
``counters()``, ``output_schema()``, ``reference_state()`` / ``load_reference_state()`` and the legacy
``add_frames`` / ``step(t, snr, hid)`` forms.

What runs where:
  * host (Python / torch plumbing): config checks, the schedule table of each control step, the traffic models'
    generator draws (TrafficGen, torch.Generator by design), the clocks, and building the argument block;
  * device (libisaac_net_b200.so, sm_100a): one fused launch per control step (inb_nr_step: enqueue + arrival gate,
    radio path gain, every scheduled slot, finish and compaction, all outputs) and one per reset (inb_nr_reset).
There is no CPU path: the engine refuses any device but CUDA, and raises if the shared library is missing.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _native as nat
from .config import NRConfig
from .phy import PhyTables
from . import invariants as inv
from .radio_map import cdf_table, load_radio_map
from .downlink import REF as DL_REF, Downlink
from .traffic import CounterDraws, DeviceTrafficGen, Requests, TrafficGen, generates

# counter-RNG constants (isaac_net/core/proto/rng.py:33-38, nr_rng.py:34, radio.py:53-56)
M32 = 0xFFFFFFFF
GOLD = 0x9E3779B9
CH_RESET = 3
RADIO_STREAM = 0x52 << 16
LOG_DISTANCE_STREAM = 10
BLOCKAGE_STREAM = RADIO_STREAM + 48
# blockage model A per scenario family (TR 38.901 Tables 7.6.4.1-2 / -4; channels/blockage.py:100-112): azimuth span
# range (deg), elevation span range (deg), distance r (m), correlation distance (m); 3 km/h blocker drift
MODEL_A = {"indoor": ((15.0, 45.0), (5.0, 15.0), 2.0, 5.0), "outdoor": ((5.0, 15.0), (5.0, 5.0), 10.0, 10.0)}
BLOCKER_SPEED_MPS = 3.0 / 3.6
C_LIGHT_38901 = 3.0e8
# TR 38.901: (default BS height, SF correlation LOS, SF correlation NLOS, sigma_SF LOS, sigma_SF NLOS, PL a, n1, b)
SCN = {"UMi": (10.0, 10.0, 13.0, 4.0, 7.82, 32.4, 21.0, 9.5), "UMa": (25.0, 37.0, 50.0, 4.0, 6.0, 28.0, 22.0, 9.0)}


class B200Unsupported(NotImplementedError, ValueError):
    """The config asks for a feature the B200 engine does not implement (see NRConfig.refusals)."""


def _mix32(x):
    x ^= x >> 16
    x = (x * 0x21F0AAAD) & M32
    x ^= x >> 15
    x = (x * 0x735A2D97) & M32
    return x ^ (x >> 15)


def _salt(v):
    return (_mix32(v & M32) + GOLD) & M32


def seed_key(seed):
    """Key of an engine seed (CounterRNG.s0, proto/rng.py:60)."""
    seed = int(seed)
    return _mix32(_mix32(seed & M32) ^ _salt((seed >> 32) & M32))


def einsum_fused(R, CK):
    """Whether the reference's CPU einsum of a plane-wave field ("erx,cekx->cerk", evaluated as a batch over envs of
    [R,2] x [2, C K] products, CK = fields x waves) takes its BLAS path, which rounds k . x as one fused multiply-add,
    rather than its plain loop for small products (ATen bmm: 2 R C K < 400), which rounds both products and their
    sum."""
    return 2 * R * CK >= 400


def _f32(x):
    return float(np.float32(x))


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def make_engine(level, E, R, device="cuda", config=None, backend="b200", *, sizes=None, seed=None, strict=False,
                traffic_rng="generator"):
    """The B200 NR engine for E envs x R robots (isaac_net/core/engine.py:232-293)."""
    if level != "L2":
        raise ValueError(f"the B200 backend implements level 'L2' (the NR engine), not {level!r}")
    if backend not in ("b200", "auto"):
        raise ValueError(f"unknown backend {backend!r}; this package provides 'b200'")
    cfg = config if config is not None else NRConfig()
    if sizes is not None:
        cfg = cfg.with_(msg_sizes=tuple(float(s) for s in sizes))
    if seed is None:
        seed = cfg.seed
    return NRB200Engine(E, R, device, cfg, seed=seed, traffic_rng=traffic_rng)


class NRB200Engine:
    """Contract API of NREngine over the fused B200 kernels (one cell, uplink)."""

    level = "L2"
    backend = "b200"

    def __init__(self, E, R, device, cfg: NRConfig, seed=None, graphs=True, traffic_rng="generator"):
        """traffic_rng: "generator" (the reference's arrival stream: the traffic models draw from a torch.Generator
        seeded per engine, so the arrivals depend on how a batch is split over engines) or "counter" (an opt-in
        stream with no counterpart in the reference: every uniform is keyed by the seed, the global env id, the
        episode and the step, so an env's arrivals are the same in any shard, traffic.CounterDraws)."""
        if traffic_rng not in ("generator", "counter"):
            raise ValueError(f"traffic_rng must be 'generator' or 'counter', not {traffic_rng!r}")
        self.traffic_rng = traffic_rng
        no = cfg.refusals()
        if no:
            raise B200Unsupported("the B200 engine does not implement " + "; ".join(f"{f}: {w}" for f, w in no))
        dev = torch.device(device)
        if dev.type != "cuda":
            raise B200Unsupported(f"the B200 engine runs on CUDA devices only (got {dev}); it has no CPU path")
        if not 1 <= R <= 128:
            raise B200Unsupported(f"R={R}: the B200 engine handles 1..128 robots per env")
        if cfg.special_ul_data and "S" in cfg.tdd_pattern:
            raise B200Unsupported("UL data in special slots (a second UL symbol count) is not built")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.L = nat.lib()
        self.E, self.R, self.dev, self.config = E, R, dev, cfg
        if seed is None:
            seed = int(torch.randint(0, 2 ** 62, ()).item())
        self.seed = int(seed)
        self.S, self.P, self.F, self.N = cfg.n_subbands, cfg.n_harq, cfg.frame_buffer, cfg.slots_per_step
        self.C = cfg.n_cells
        self.tab = PhyTables(cfg, cfg.subband_prbs, dev)
        self.rician = cfg.rician_mode == "fixed"
        self._alloc_state()
        self.s0 = seed_key(self.seed)
        self.env_id = torch.arange(E, dtype=torch.long, device=dev)
        self.env_offset = 0
        self.episode = torch.full((E,), -1, dtype=torch.long, device=dev)
        self.rng_ctr = torch.zeros(E, dtype=torch.long, device=dev)
        self.ctr = torch.zeros(E, nat.NCTR, dtype=torch.long, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.T = 0
        self.epoch = torch.zeros(E, dtype=torch.long, device=dev)
        self._uniform_epoch = 0
        self._last_snr = torch.zeros(E, R, device=dev)
        self._last_hid = torch.zeros(E, dtype=torch.long, device=dev)
        self.last_g = None
        self.prb_avail = 0.0
        self.traffic = None
        self._extras = False
        if generates(cfg.traffic):
            tseed = (int(self.seed) * 6364136223846793005 + 1442695040888963407) % 2 ** 62
            cd = CounterDraws(self.s0, self.env_id, self.episode, R) if traffic_rng == "counter" else None
            self.traffic = TrafficGen(cfg.traffic, E, R, dev, cfg.control_step_ms, self.N, seed=tseed, counter=cd)
            self._extras = True
        # the arrivals of periodic / video / bursty models come from one kernel that replays the torch.Generator
        # stream; event models (host triggers) keep the torch path
        self.dtraffic = DeviceTrafficGen(self.traffic, self.L) if DeviceTrafficGen.supports(self.traffic) else None
        # the downlink (dl=True, one cell): its state, counters and DL traffic models (downlink.py)
        self.dl = None
        if cfg.dl:
            if traffic_rng != "generator" and generates(cfg.traffic, "dl"):
                raise B200Unsupported("traffic_rng='counter' with downlink traffic models is not built")
            self.dl = Downlink(self)
        self._fields = None
        self._radio_ready = False          # the radio's draws exist (made at the first step with poses)
        self._gnb = torch.tensor(cfg.gnb_xy(), dtype=torch.float32, device=dev).contiguous()
        self._sched = {}
        # CUDA graphs: one captured step (traffic draws + the fused launch) per schedule key, replayed with the poses
        # copied into a static buffer and the control step read from device memory
        self.graphs = bool(graphs) and not any(m.kind == "event" for m in (cfg.traffic or ()))
        self._graphs = {}
        self._pool = None
        # a captured step reads its control step and the address of its output block from here (inb_store2)
        self._ctl = torch.zeros(2, dtype=torch.long, device=dev)
        self._T_dev = self._ctl[0]
        self._pos_buf = None
        self._steps_done = 0
        # debug / test mode: check the state and the step's message conservation after every step (synchronizes)
        self.debug_invariants = False
        self.nvtx = False          # an NVTX range around every step (for nsys / ncu timelines)
        self.concurrent_traffic = True   # graph steps run traffic and radio beside the fading launch
        self._args = nat.InbStepArgs()
        self._fill_static()
        self._setup_radio()
        if self.C > 1:
            self.pathgain = torch.zeros(E, R, self.C, device=dev)     # every link's path gain of the last step
        self._kernel_reset(None)

    # ------------------------------------------------------------------ buffers
    def _alloc_state(self):
        E, R, S, P, F, d = self.E, self.R, self.S, self.P, self.F, self.dev
        full = lambda shape, dt, v: torch.full(shape, v, dtype=dt, device=d)
        L, f32, b = torch.long, torch.float32, torch.bool
        st = {}
        for n, v in (("sent", 0), ("floor_", 0), ("bsr", 0), ("sr_t", -1), ("last_tx", -1), ("enq", 0)):
            st[n] = full((E, R), L, v)
        st["olla"], st["avg"] = full((E, R), f32, 0.0), full((E, R), f32, 100.0)
        st["csi"] = full((E, R, S), f32, 0.0)
        cd = (self.C,) if self.C > 1 else ()
        st["h"] = full((E, R, *cd, S, 2), f32, 0.0)
        if self.rician:
            st["spec"], st["k_lin"] = full((E, R, *cd, 2), f32, 0.0), full((E, R, *cd), f32, 0.0)
        if self.C > 1:   # CellAssociation state, the gNBs' N+I per PRB (mW)
            for n, v in (("serv", 0), ("a3_cand", -1), ("a3_cnt", 0), ("ho_end", 0), ("n_ho", 0)):
                st[n] = full((E, R), L, v)
            st["pending"] = full((E,), b, True)
            st["ni_ul"] = full((E, self.C, S), f32, 0.0)
        for n in ("h_state", "h_lo", "h_hi", "h_ready", "h_ntx", "h_mcs", "h_tbs", "h_nsb"):
            st[n] = full((E, R, P), L, 0)
        st["h_comb"] = full((E, R, P), f32, 0.0)
        st["cap"] = full((E, R, F), L, -1)
        for n in ("start", "end_", "cls", "hid", "tag", "prio"):
            st[n] = full((E, R, F), L, 0)
        st["lost"], st["det"] = full((E, R, F), b, False), full((E, R, F), b, False)
        st["fin"] = full((E, R, F), torch.float64, math.inf)
        st["off"] = full((E, R, F), torch.float64, 0.0)
        st["dline"] = full((E, R, F), torch.float64, math.inf)
        if self.config.ul_amc_alloc == "previous":   # AMC_STATE (mac_ul.py:51)
            st["last_nprb"] = full((E, R), f32, 0.0)
        if self.config.ul_grant_model == "bsr":      # BSR_STATE (mac_ul.py:45-50)
            st["bsr_est"] = full((E, R), L, 0)
            st["bsr_rep_v"] = full((E, R, nat.BSR_DEPTH), L, 0)
            st["bsr_rep_g"] = full((E, R, nat.BSR_DEPTH), L, -(2 ** 62))
            st["bsr_hid"], st["bsr_hid_until"] = full((E, R), L, 0), full((E, R), L, -1)
            st["bsr_enq_seen"] = full((E, R), L, 0)
            st["bsr_boot"], st["bsr_armed"] = full((E, R), b, False), full((E, R), b, False)
        self.st = st

    def _state_struct(self):
        s = nat.InbState()
        for n in nat.STATE_FIELDS:
            t = self.st.get(n)
            setattr(s, n, t.data_ptr() if t is not None else None)
        return s

    def _fill_static(self):
        cfg, a, tab = self.config, self._args, self.tab
        p = a.p
        p.E, p.R, p.S, p.P, p.F = self.E, self.R, self.S, self.P, self.F
        p.MCS, p.mcs_max, p.C_axis, p.G_axis = tab.M, tab.mcs_max, tab.C, tab.G
        p.nprb, p.N = cfg.nprb, self.N
        p.sched = {"pf": 0, "maxci": 1, "rr": 2}[cfg.scheduler]
        thr = tab.thr_ref[: tab.mcs_max + 1].cpu()
        p.thr_mono = int(bool((thr[1:] >= thr[:-1]).all()))
        p.olla_on, p.phr_cap, p.retx_priority = int(cfg.olla), int(cfg.phr_cap), int(cfg.retx_priority)
        # ul_power="whole_band": a fixed PSD over the carrier, the same split for every grant and no PHR cap
        # (mac_ul.py:154-180); the scheduler estimate reads the split from the per-RBG table
        p.whole_band = int(cfg.ul_power == "whole_band")
        p.wb_db = _f32(10 * math.log10(cfg.nprb / cfg.snr_ref_prbs))
        if p.whole_band:
            p.phr_cap = 0
            tab.lw10.fill_(p.wb_db)
        p.comb_cc, p.harq_drop = int(cfg.harq_combining == "cc"), int(cfg.harq_fail == "drop")
        p.purge, p.fading, p.rician = int(cfg.discard == "purge"), int(cfg.fading), int(self.rician)
        p.sr_delay, p.ul_rtt, p.rlc_retx = cfg.sr_delay, cfg.ul_rtt, cfg.rlc_retx_slots
        p.max_tx, p.tb_oh, p.timeout = cfg.max_harq_tx, cfg.tb_overhead_bytes, cfg.timeout_steps
        p.dmrs, p.oh, p.ref_prbs = cfg.dmrs_re_per_prb, cfg.overhead_re_per_prb, cfg.snr_ref_prbs
        p.s0 = 0
        p.inv_sqrt2 = _f32(np.float32(1.0) / np.float32(math.sqrt(2)))
        p.ul_ref0 = _f32(cfg.ue_tx_dbm - 10 * math.log10(cfg.snr_ref_prbs))
        p.noise_prb = _f32(cfg.noise_dbm_per_prb("gnb"))
        p.ue_tx = _f32(cfg.ue_tx_dbm)
        p.sub_noise = _f32(cfg.subband_noise_dbm)
        p.phr_min = _f32(cfg.phr_min_db)
        p.olla_up = _f32(cfg.olla_up_db)
        p.olla_dn = _f32(cfg.olla_up_db * (1 - cfg.bler_target) / cfg.bler_target)
        p.pf_a = _f32(1 - 1 / cfg.pf_window)
        p.pf_b = _f32(1 / cfg.pf_window)
        p.pf_rbg, p.pf_freeze = int(cfg.pf_update == "rbg"), int(cfg.pf_avg_idle == "freeze")
        p.tdma, p.amc_prev = int(cfg.ul_retx_sched == "tdma"), int(cfg.ul_amc_alloc == "previous")
        p.lena_ctr = int(bool(cfg.lena_mac_switches()))
        p.dl_on = int(bool(cfg.dl))
        p.bsr_on = int(cfg.ul_grant_model == "bsr")
        if p.bsr_on:   # the SR / BSR pipeline's timing and header sizes (config.py:588-594, 1088-1090)
            p.sr_boot_slots, p.sr_boot_bytes = int(cfg.sr_boot_slots), int(cfg.sr_boot_bytes)
            p.bsr_delay, p.rlc_tail_slots = int(cfg.bsr_delay_slots), int(cfg.rlc_tail_timer_slots)
            p.bsr_hdr, p.bsr_est_hdr = int(cfg.bsr_hdr_bytes), int(cfg.bsr_est_hdr_bytes)
            p.rlc_tail_bytes = int(cfg.rlc_tail_bytes)
        p.target = _f32(cfg.bler_target)
        p.inv_S = _f32(1.0 / self.S)
        p.s0_snr, p.c0_cbs = _f32(tab.s0), _f32(tab.c0)
        p.inv_ds = _f32(np.float32(1.0) / np.float32(tab.ds))
        p.inv_dc = _f32(np.float32(1.0) / np.float32(tab.dc))
        p.proc_off = cfg.proc_offset_ms / cfg.control_step_ms
        p.ctl_ms = float(cfg.control_step_ms)
        p.inv_N_d = 1.0 / self.N
        p.inv_ref_prbs = _f32(np.float32(1.0) / np.float32(cfg.snr_ref_prbs))
        K = cfg.shadow_modes
        p.Kf = K
        p.field_fma = int(einsum_fused(self.R, self.C * K))
        if cfg.channel == "tr38901":
            hbs, _, _, sl, _, pa, n1, bb = SCN[cfg.tr38901_scenario]
            h_bs = float(cfg.gnb_height_m) if cfg.gnb_height_m is not None else hbs
            h_ut = float(cfg.ue_height_m)
            fc = cfg.carrier_ghz * 1e9
            dbp = 4 * (h_bs - 1.0) * (h_ut - 1.0) * fc / 3.0e8
            p.radio_model = 0 if cfg.tr38901_scenario == "UMi" else 1
            p.h_bs, p.h_ut, p.dbp = _f32(h_bs), _f32(h_ut), _f32(dbp)
            p.pl_a, p.pl_n1 = _f32(pa), _f32(n1)
            p.fc_term = _f32(20 * math.log10(cfg.carrier_ghz))
            p.pl_b_term = _f32(bb * math.log10(dbp ** 2 + (h_bs - h_ut) ** 2))
            p.sigma_sf = _f32(sl)
            p.amp = _f32(math.sqrt(2 / K))
            p.hh2 = _f32((h_bs - h_ut) ** 2)
            if cfg.tr38901_los != "los":
                raise B200Unsupported("tr38901 with an NLOS state is not built (forced LOS only)")
        elif cfg.channel == "log_distance":
            p.radio_model = 2
            p.pl_const, p.pl_10n = _f32(cfg.pl_const_db), _f32(10 * cfg.pathloss_exp)
            p.amp = _f32(cfg.shadow_sigma_db * math.sqrt(2 / K))
        p.C = self.C
        if self.C > 1:   # CellAssociation (radio.py:348-359) with the NR slot clock; nr_engine.py:221-222, 671-675
            slot_ms = cfg.control_step_ms / self.N
            p.ttt = int(round(cfg.a3_ttt_ms / slot_ms))
            p.ho_int = int(round(cfg.ho_interruption_ms / slot_ms))
            p.a3_off, p.a3_hyst = _f32(cfg.a3_offset_db), _f32(cfg.a3_hyst_db)
            floor = cfg.a3_min_target_rsrp_dbm
            p.has_floor = int(floor is not None)
            p.floor_rx = _f32(floor - (cfg.gnb_tx_dbm - 10 * math.log10(12 * cfg.nprb) - cfg.ue_tx_dbm)) \
                if floor is not None else 0.0
            p.ho_flush = int(cfg.ho_rlc == "flush")
            p.pc_on = int(cfg.ul_pc_on)
            self.noise_mw = 10 ** (cfg.noise_dbm_per_prb("gnb") / 10)
            p.noise_mw = _f32(self.noise_mw)
            p.ref_db = _f32(10 * math.log10(cfg.snr_ref_prbs))
            p.ue_tx_ref = _f32(cfg.ue_tx_dbm - 10 * math.log10(cfg.snr_ref_prbs))
            p.pc_p0, p.pc_alpha = _f32(cfg.ul_pc_p0_dbm), _f32(cfg.ul_pc_alpha)
            p.li_alpha, p.li_beta = _f32(cfg.li_alpha), _f32(1 - cfg.li_alpha)
        a.s = self._state_struct()
        t = a.t
        t.bler, t.thr_ref, t.se, t.beta, t.rate = (tab.bler.data_ptr(), tab.thr_ref.data_ptr(), tab.se.data_ptr(),
                                                   tab.beta.data_ptr(), tab.rate.data_ptr())
        t.w, t.lw, t.lw10 = tab.w.data_ptr(), tab.lw.data_ptr(), tab.lw10.data_ptr()
        t.la_tbs, t.la_i0, t.la_wi, t.la_ncb = (tab.la_tbs.data_ptr(), tab.la_i0.data_ptr(), tab.la_wi.data_ptr(),
                                                tab.la_ncb.data_ptr())
        t.gnb = self._gnb.data_ptr()
        a.env_id, a.episode, a.rng_ctr = self.env_id.data_ptr(), self.episode.data_ptr(), self.rng_ctr.data_ptr()
        a.epoch, a.last_hid, a.ctr, a.status = (self.epoch.data_ptr(), self._last_hid.data_ptr(),
                                                self.ctr.data_ptr(), self.status.data_ptr())
        # fading-gain rows of one step: the CSI before the step + one row per UL slot (at most slots_per_step); with
        # several cells one row per UL slot holds every link's gain
        rows = self.N * self.C if self.C > 1 else self.N + 1 + (self.N if cfg.dl else 0)   # + the DL gain rows
        self._gain = torch.empty(rows * self.S * self.E * self.R, dtype=torch.float32, device=self.dev)
        a.gain, a.gain_cap = self._gain.data_ptr(), self._gain.numel()

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)

    # ------------------------------------------------------------------ radio fields (channels/fields.py:38-91)
    def _uniforms(self, stream, n):
        out = torch.empty(self.E, n, dtype=torch.float32, device=self.dev)
        rc = self.L.inb_rng_draw(self.E, n, self.s0, CH_RESET, stream, self.env_id.data_ptr(), self.episode.data_ptr(),
                                 None, 0, out.data_ptr(), self._stream())
        nat.check(rc, "inb_rng_draw")
        return out

    def _plane_waves(self, stream, spectrum, dcorr, C=None):
        C, K = (self.C if C is None else C), self.config.shadow_modes
        rand = lambda i: self._uniforms(stream + i, C * K).view(self.E, C, K)
        ang = rand(0) * 2 * math.pi
        if spectrum == "sos":
            wl = 20 + 40 * rand(1)
            if dcorr != 10.3:
                wl = wl * (dcorr / 10.3)
            k = torch.stack([torch.cos(ang), torch.sin(ang)], -1) * (2 * math.pi / wl)[..., None]
        else:
            u = rand(1).clamp(max=1 - 1e-6)
            kmag = torch.sqrt((1 - u) ** -2 - 1) / dcorr
            k = torch.stack([torch.cos(ang), torch.sin(ang)], -1) * kmag[..., None]
        phi = rand(2) * 2 * math.pi
        return k.permute(1, 0, 2, 3).contiguous(), phi.permute(1, 0, 2).contiguous()

    def _draw_fields(self):
        cfg = self.config
        if cfg.channel == "tr38901":
            return self._plane_waves(RADIO_STREAM + 16, "exp", SCN[cfg.tr38901_scenario][1])
        return self._plane_waves(LOG_DISTANCE_STREAM, cfg.shadow_acf, cfg.shadow_dcorr_m)

    # ------------------------------------------------------------------ radio map and blockage (radio launch)
    def _setup_radio(self):
        """Static part of the radio launch: the radio map on the device (RadioMapChannel, channels/models.py:179-199)
        and the blockage model A constants and CDF table (BlockageA.__init__, channels/blockage.py:157-170)."""
        cfg, rm = self.config, self._args.rm
        self._map = self._blk = None
        self._obstacles = bool(cfg.blockage)
        rm.on = int(cfg.channel == "radio_map" or cfg.blockage)
        self._rpg = self._rblk = None
        if not rm.on:
            return
        E, R, C, dev = self.E, self.R, self.C, self.dev
        self._rpg = torch.zeros(E, R, C, dtype=torch.float32, device=dev)
        self._rblk = torch.zeros(E, R, dtype=torch.uint8, device=dev)
        rm.pg, rm.blk = self._rpg.data_ptr(), self._rblk.data_ptr()
        if cfg.channel == "radio_map":
            gain, H, W, bounds, meta = load_radio_map(cfg.radio_map_path)
            if gain.shape[0] != C:
                raise ValueError(f"the radio map has {gain.shape[0]} cells but the config has n_cells={C}")
            want = meta.get("gnb_xy")
            if want is not None:
                want = np.asarray(want, dtype=np.float32).reshape(-1, 2)
                have = np.asarray(cfg.gnb_xy(), dtype=np.float32)
                if want.shape != have.shape or not np.allclose(want, have, atol=0.5, rtol=1e-5):
                    raise ValueError(f"the radio map was made for gNBs at {want.tolist()}; set cell_positions_m to "
                                     "match")
            self._map = gain.to(dev)
            x0, y0, x1, y1 = bounds
            rm.map_on, rm.H, rm.W, rm.map = 1, H, W, self._map.data_ptr()
            rm.x0, rm.y0 = _f32(x0), _f32(y0)
            rm.sx, rm.sy = _f32((W - 1) / (x1 - x0)), _f32((H - 1) / (y1 - y0))
            rm.wm1, rm.hm1, rm.wm2, rm.hm2 = float(W - 1), float(H - 1), float(W - 2), float(H - 2)
        if cfg.blockage:
            family = "outdoor" if cfg.channel == "tr38901" and cfg.tr38901_scenario in ("UMi", "UMa") else "indoor"
            self._blk_family = MODEL_A[family]
            r = self._blk_family[2]
            lam = C_LIGHT_38901 / (cfg.carrier_ghz * 1e9)
            K = cfg.shadow_modes
            self._cdf = cdf_table(K).to(dev)
            rm.blockage, rm.Kb, rm.n_table = 1, K, self._cdf.numel()
            rm.amp_b, rm.ck, rm.max_db = _f32(math.sqrt(2 / K)), _f32(math.pi / lam * r), _f32(cfg.blockage_max_db)
            h_ut = float(cfg.ue_height_m)
            if cfg.channel == "tr38901":
                h_bs = float(cfg.gnb_height_m) if cfg.gnb_height_m is not None else SCN[cfg.tr38901_scenario][0]
            else:
                h_bs = float(cfg.gnb_height_m) if cfg.gnb_height_m is not None else h_ut
            rm.h_ut, rm.h_bs = _f32(h_ut), _f32(h_bs)
            rm.dt, rm.u_den = _f32(cfg.control_step_ms * 1e-3), float(self._cdf.numel() + 1)
            rm.table = self._cdf.data_ptr()
            rm.fma_b = int(einsum_fused(self.R, nat.BLK_REGIONS * K))
            self._blk_t = torch.zeros(E, dtype=torch.float32, device=dev)
            rm.t = self._blk_t.data_ptr()
            self._args.p.los_const = int(cfg.channel == "tr38901" and cfg.tr38901_los == "los")

    def _draw_blockage(self):
        """Model-A draws of every env (BlockageA._draw, channels/blockage.py:172-186): region fields (RESET streams
        BLOCKAGE_STREAM + 0..2), azimuth / elevation spans (+ 3, + 4), drift direction (+ 5)."""
        xr, yr, _, dcorr = self._blk_family
        K = nat.BLK_REGIONS
        k, phi = self._plane_waves(BLOCKAGE_STREAM, "exp", dcorr, C=K)
        ux = self._uniforms(BLOCKAGE_STREAM + 3, K)
        uy = self._uniforms(BLOCKAGE_STREAM + 4, K)
        ua = self._uniforms(BLOCKAGE_STREAM + 5, 1).view(self.E)
        xk = xr[0] + (xr[1] - xr[0]) * ux
        yk = yr[0] + (yr[1] - yr[0]) * uy
        ang = 2 * math.pi * ua
        vel = BLOCKER_SPEED_MPS * torch.stack([torch.cos(ang), torch.sin(ang)], -1)
        return {"k": k, "phi": phi, "xk": xk.contiguous(), "yk": yk.contiguous(), "vel": vel.contiguous()}

    def _make_radio(self):
        cfg = self.config
        if cfg.channel != "radio_map":
            self._fields = self._draw_fields()
            self._bind_fields()
        if cfg.blockage:
            self._blk = self._draw_blockage()
            rm = self._args.rm
            b = self._blk
            rm.bk, rm.bphi, rm.xk, rm.yk, rm.vel = (b["k"].data_ptr(), b["phi"].data_ptr(), b["xk"].data_ptr(),
                                                    b["yk"].data_ptr(), b["vel"].data_ptr())
            self._blk_t.zero_()
        self._radio_ready = True
        self._graphs.clear()

    def _bind_fields(self):
        k, phi = self._fields
        self._args.t.fk, self._args.t.fphi = k.data_ptr(), phi.data_ptr()

    def _reset_radio(self, m):
        if not self._radio_ready:
            return
        if self._fields is not None:
            k, phi = self._draw_fields()
            k0, p0 = self._fields
            k0.copy_(torch.where(m.view(1, -1, 1, 1), k, k0))
            p0.copy_(torch.where(m.view(1, -1, 1), phi, p0))
        if self._blk is not None:       # BlockageA.reset (channels/blockage.py:183-189)
            new = self._draw_blockage()
            for n, v in new.items():
                mv = m.view(1, -1, *([1] * (v.dim() - 2))) if n in ("k", "phi") else m.view(-1, *([1] * (v.dim() - 1)))
                self._blk[n].copy_(torch.where(mv, v, self._blk[n]))
            self._blk_t.masked_fill_(m, 0.0)

    # ------------------------------------------------------------------ resets
    def _kernel_reset(self, mask):
        a = nat.InbResetArgs()
        a.E, a.R, a.S, a.P, a.F = self.E, self.R, self.S, self.P, self.F
        a.s0, a.rician = self.s0, int(self.rician)
        a.k_lin0 = _f32(10 ** (self.config.rician_k_db / 10)) if self.rician else 0.0
        a.inv_sqrt2 = self._args.p.inv_sqrt2
        a.two_pi = _f32(2 * math.pi)
        a.mask = mask.data_ptr() if mask is not None else None
        a.env_id, a.episode, a.rng_ctr = self.env_id.data_ptr(), self.episode.data_ptr(), self.rng_ctr.data_ptr()
        a.s = self._state_struct()
        a.C = self.C
        a.noise_mw = self._args.p.noise_mw
        nat.check(self.L.inb_nr_reset(ctypes.byref(a), self._stream()), "inb_nr_reset")

    def _ids(self, env_ids):
        if env_ids is None or (isinstance(env_ids, slice) and env_ids == slice(None)):
            return None
        if isinstance(env_ids, torch.Tensor):
            if env_ids.dtype == torch.bool:
                return env_ids.to(self.dev).nonzero(as_tuple=True)[0]
            return env_ids.to(device=self.dev, dtype=torch.long).reshape(-1)
        return torch.as_tensor(list(env_ids), dtype=torch.long, device=self.dev)

    def reset(self, env_ids=None):
        """Re-initialize env_ids (None = all): queues, HARQ, SR/BSR, OLLA, PF, CSI, fading, radio and clock."""
        ids = self._ids(env_ids)
        if ids is not None and ids.numel() == 0:
            return
        if ids is None:
            if self.traffic is not None:
                self.traffic.reset(None)
            if self.dl is not None:
                self.dl.reset(None)
            self._kernel_reset(None)
            self.ctr.zero_()
            if self.C > 1:
                self.pathgain = torch.zeros_like(self.pathgain)
            self.prb_avail = 0.0
            self.T = 0
            self.epoch.zero_()
            self._uniform_epoch = 0
            self._last_snr = torch.zeros_like(self._last_snr)   # the last step's output tensor stays the caller's
            self._last_hid.zero_()
            self.last_g = None
            self._reset_radio(torch.ones(self.E, dtype=torch.bool, device=self.dev))
            return
        m = torch.zeros(self.E, dtype=torch.bool, device=self.dev)
        m[ids] = True
        if self.traffic is not None:
            self.traffic.reset(m)
        if self.dl is not None:
            self.dl.reset(m)
        self._kernel_reset(m)
        self.epoch.index_fill_(0, ids, self.T)
        self._uniform_epoch = None
        self._last_snr = self._last_snr.index_fill(0, ids, 0.0)
        self._last_hid.index_fill_(0, ids, 0)
        self._reset_radio(m)

    def set_env_offset(self, offset, redo_reset=True):
        """Make this engine a shard of a larger batch: key the counter-RNG rows by global env id offset + i and redo
        the initial reset under those keys with the episode counters rewound first, so every env stays in its first
        episode and draws what it would draw in one unsharded engine (isaac_net/core/sharded.py:61-77;
        CounterRNG.set_env_offset, proto/rng.py:103-109).  redo_reset=False only re-keys the rows."""
        offset = int(offset)
        if offset == self.env_offset:
            return
        self.env_id.add_(offset - self.env_offset)
        self.env_offset = offset
        if redo_reset:
            self.episode.sub_(1)
            self.reset(None)

    # ------------------------------------------------------------------ clocks
    @property
    def clock(self):
        return self.T - self.epoch

    def _now(self, t):
        if t is None:
            return self.T
        if isinstance(t, torch.Tensor):
            if t.dim() == 0:
                t = int(t)
            else:
                if not torch.equal(t.to(self.dev, torch.long), self.clock):
                    raise ValueError("t must equal the engine clock (the NR engine cannot jump in time); pass t=None")
                return self.T
        t = int(t)
        if self._uniform_epoch is None:
            raise ValueError("after a partial reset the envs have different clocks: pass t=None")
        if t + self._uniform_epoch != self.T:
            raise ValueError(f"t={t} but the engine clock is {self.T - self._uniform_epoch}: pass t=None")
        return self.T

    # ------------------------------------------------------------------ policy messages (engine.py:796-819)
    def submit(self, t, requests, snr_db=None, *, tag=None, priority=None, deadline_ms=None):
        """Enqueue the policy's messages at capture step t: Requests or send [E,R]; returns accepted [E,R]."""
        T = self._now(t)
        req = requests if isinstance(requests, Requests) else Requests(send=requests)
        send = req.send.to(self.dev, torch.long)
        det = req.det.to(self.dev, torch.bool) if req.det is not None else torch.zeros_like(send, dtype=torch.bool)
        hid = req.hid.to(self.dev, torch.long) if req.hid is not None else torch.zeros(self.E, dtype=torch.long,
                                                                                          device=self.dev)
        self._last_hid.copy_(hid)
        if tag is not None or priority is not None or deadline_ms is not None:
            self._extras = True
        st, F = self.st, self.F
        sizes = torch.tensor(self.config.msg_sizes, dtype=torch.float32, device=self.dev)
        nbytes = sizes[(send - 1).clamp(min=0)]
        cnt = (st["cap"] >= 0).sum(-1)
        acc = (send > 0) & (cnt < F) & (nbytes > 0)
        i = cnt.clamp(max=F - 1)
        oh = (i[..., None] == torch.arange(F, device=self.dev)) & acc[..., None]
        nb = nbytes.round().long()
        put = lambda n, v: st[n].copy_(torch.where(oh, v[..., None].to(st[n].dtype) if torch.is_tensor(v)
                                                   else torch.full_like(st[n], v), st[n]))
        put("cap", T)
        put("start", st["enq"])
        put("end_", st["enq"] + nb)
        put("lost", False)
        put("fin", math.inf)
        put("off", 0.0)
        put("cls", send)
        put("det", det)
        put("hid", hid[:, None].expand(-1, self.R))
        for n, v, dflt in (("tag", tag, 0), ("prio", priority, 0), ("dline", deadline_ms, math.inf)):
            if v is None:
                put(n, dflt)
            else:
                put(n, torch.as_tensor(v, dtype=st[n].dtype, device=self.dev).expand(self.E, self.R))
        st["enq"].add_(nb * acc)
        return acc

    def add_dl_frames(self, t, nbytes, cls=None):
        """One downlink frame of nbytes [E,R] application bytes per robot (0 = none) at capture step t, cls [E,R]
        tagging it (NREngine.add_dl_frames, engine.py:825-827); returns accepted [E,R]."""
        if self.dl is None:
            raise ValueError("add_dl_frames needs config.dl = True")
        return self.dl.add_frames(self._now(t), nbytes, cls)

    def add_frames(self, t, send, det, hid, snr_db):
        """Legacy wrapper (NetSlot API)."""
        self.submit(t, Requests(send, det, hid), snr_db)

    # ------------------------------------------------------------------ one control step
    def _rows(self, g0):
        """Schedule rows of the step at slot g0 with the fading coefficients of each row (advances last_g)."""
        cfg = self.config
        sched = cfg.schedule(g0)
        dt0 = 0 if not sched else (1 if self.last_g is None else g0 + sched[0][0] - self.last_g)
        key = (g0 % cfg.schedule_period(), dt0 if cfg.fading else 0)
        ent = self._sched.get(key)
        if ent is None:
            rows, rowf, rows_dl = [], [], []
            prev = None
            j = 0
            for rel, dls, uls, sr, cqi, ack in sched:
                dt = dt0 if prev is None else rel - prev
                prev = rel
                rho = cfg.fading_rho_per_ms ** (dt * cfg.slot_ms)
                rows.append((rel, uls, int(sr), int(dt > 0)))
                rowf.append((_f32(rho), _f32(math.sqrt(1 - rho ** 2))))
                # the downlink's view of the row: DL symbols, CQI report, HARQ-ACK slot + gNB processing (relative to
                # g0, mac_dl.py:47-49), index of its DL gain row (rows with DL data or a CQI report) or -1
                need = bool(dls or cqi)
                rows_dl.append((dls, int(cqi), ack + cfg.gnb_proc_slots, j if need else -1))
                j += int(need)
            if len(rows) > nat.MAX_ROWS:
                raise B200Unsupported(f"{len(rows)} scheduled slots per control step (at most {nat.MAX_ROWS})")
            ent = (rows, rowf, sum(1 for r in rows if r[1]), rows_dl, j, sum(1 for r in rows_dl if r[0]))
            self._sched[key] = ent
        if sched and cfg.fading:
            self.last_g = g0 + sched[-1][0]
        self._rows_key = key
        return ent

    def _out_layout(self, M, dl=False):
        """(name, dtype, shape, byte offset, bytes) of every step output in one block, and the block's size; dl: with
        the downlink's outputs (the CUDA-graph step's block; an eager step's DL outputs are the DL call's own)."""
        E, R, F = self.E, self.R, self.F
        spec = [("delivered", torch.bool, (E, R, F)), ("timed_out", torch.bool, (E, R, F)),
                ("dropped", torch.bool, (E, R, F)), ("deadline_miss", torch.bool, (E, R, F)),
                ("cap", torch.long, (E, R, F)), ("cls", torch.long, (E, R, F)),
                ("arrival_slot", torch.long, (E, R, F)), ("tag", torch.long, (E, R, F)),
                ("priority", torch.long, (E, R, F)), ("bytes", torch.long, (E, R, F)),
                ("delay", torch.float32, (E, R, F)), ("arrival", torch.float64, (E, R, F)),
                ("newest", torch.long, (E, R)), ("queue_len", torch.long, (E, R)),
                ("gen_accepted", torch.long, (E, R)), ("gen_bytes", torch.long, (E, R)),
                ("queue_bytes", torch.float32, (E, R)), ("sinr_db", torch.float32, (E, R)),
                ("pathgain", torch.float32, (E, R, self.C) if self.C > 1 else (E, R)), ("det_env", torch.bool, (E,))]
        spec.append(("serving_cell", torch.long, (E, R)))      # 0 with one cell, written by the MAC kernel
        if self._obstacles:       # obstacle outputs of the serving link (engine.py:437-448)
            spec.append(("blocked", torch.bool, (E, R)))
            if self.config.channel == "tr38901":
                spec.append(("los", torch.bool, (E, R)))
        if dl and self.dl is not None:
            spec += [(n, dt, shape) for n, dt, shape, f in self.dl.out_spec()]
        off, lay = 0, []
        for n, dt, shape in spec:
            nb = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            lay.append((n, dt, shape, off, nb))
            off += (nb + 255) // 256 * 256
        return lay, off

    def _alloc_outputs(self):
        lay = getattr(self, "_lay", None)
        if lay is None:
            self._lay = lay = self._out_layout(0)
        spec, total = lay
        blob = torch.empty(total, dtype=torch.uint8, device=self.dev)
        out = {}
        o = nat.InbOutputs()
        for n, dt, shape, off, nb in spec:
            v = blob[off:off + nb].view(dt).view(shape)
            out[n] = v
            setattr(o, n, v.data_ptr())
        return out, o

    def step(self, t=None, x=None, cur_hid=None, *, snr_db=None, dl_snr_db=None, pathgain_db=None, vel=None,
             triggers=None, blockers=None, fetch=None, _pathgain=None, _arrivals=None, _dl_arrivals=None):
        """Advance [t, t+1). x: poses [E,R,2|3] (through the engine's radio) or SNR [E,R] dB; snr_db= [E,R] or
        [E,R,S]; triggers= feeds event traffic models.  Returns the step dict (or (newest, det_env) in the legacy
        form step(t, snr, cur_hid)).

        Host memory: poses x may live on the host (pinned, for an asynchronous copy); they are copied to the device on
        the engine's input stream, which overlaps the copy with the kernels of the previous step.  fetch= {key: host
        tensor} fills those host tensors with this step's outputs on the engine's output stream, overlapping the copy
        with the kernels of the next step; the CUDA event `fetch_done` marks the copies complete (`sync_fetch()` waits
        for it on the host)."""
        if self.nvtx:
            torch.cuda.nvtx.range_push(f"inb.step T={self.T}")
        staged = None
        if x is not None and torch.is_tensor(x) and x.device.type == "cpu" and x.dim() == 3:
            x, staged = self._stage_poses(x)
        q_before = self.queued().clone() if self.debug_invariants else None
        res = self._step(t, x, cur_hid, snr_db=snr_db, dl_snr_db=dl_snr_db, pathgain_db=pathgain_db, vel=vel,
                         triggers=triggers, blockers=blockers, _pathgain=_pathgain, _arrivals=_arrivals,
                         _dl_arrivals=_dl_arrivals)
        if q_before is not None and isinstance(res, dict):
            # submitted messages are queued already when the step starts; the step adds the traffic models' ones
            acc = res["gen_accepted"] if "gen_accepted" in res else torch.zeros_like(q_before)
            bad = inv.state_violations(self) + inv.step_violations(q_before, acc, res)
            if bad or int(self.status.item()) != 0:
                raise RuntimeError(f"engine invariants violated at T={self.T - 1}: {bad}, status "
                                   f"{int(self.status.item()):#x}")
        if staged is not None:
            staged.record(torch.cuda.current_stream(self.dev))     # the staging buffer has been read
        if fetch:
            if not isinstance(res, dict):
                raise ValueError("fetch= needs the dict form of step (no cur_hid)")
            self._fetch(res, fetch)
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        return res

    # ------------------------------------------------------------------ host <-> device copies off the compute stream
    def _stage_poses(self, x):
        """Copy host poses into one of two device staging buffers on the input stream; the current stream waits for
        the copy.  Returns the buffer and the event to record once the step has read it."""
        if getattr(self, "_h2d", None) is None:
            self._h2d = torch.cuda.Stream(self.dev)
            self._stage = [torch.empty(self.E, self.R, 2, dtype=torch.float32, device=self.dev) for _ in range(2)]
            self._stage_free = [None, None]
            self._stage_i = 0
        i = self._stage_i
        self._stage_i ^= 1
        buf = self._stage[i]
        if self._stage_free[i] is not None:
            self._h2d.wait_event(self._stage_free[i])          # the step two calls ago has read this buffer
        with torch.cuda.stream(self._h2d):
            buf.copy_(x[..., :2], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(self._h2d)
        torch.cuda.current_stream(self.dev).wait_event(ready)
        self._stage_free[i] = torch.cuda.Event()
        return buf, self._stage_free[i]

    def _fetch(self, res, fetch):
        if getattr(self, "_d2h", None) is None:
            self._d2h = torch.cuda.Stream(self.dev)
            self._fetch_hold = []
        cur = torch.cuda.current_stream(self.dev)
        done = torch.cuda.Event()
        done.record(cur)
        self._d2h.wait_event(done)
        with torch.cuda.stream(self._d2h):
            for k, dst in fetch.items():
                dst.copy_(res[k], non_blocking=True)
            self.fetch_done = torch.cuda.Event()
            self.fetch_done.record(self._d2h)
        # The copied outputs stay referenced until a later step's fetch, and the compute stream waits for their
        # copies before the reference is dropped, so their memory is reused only after the copies (cheaper on the
        # host than per-tensor record_stream bookkeeping).
        self._fetch_hold.append(([res[k] for k in fetch], self.fetch_done))
        if len(self._fetch_hold) > 2:
            _, ev = self._fetch_hold.pop(0)
            cur.wait_event(ev)

    def sync_fetch(self):
        """Block the host until the last step's fetch= copies are complete."""
        ev = getattr(self, "fetch_done", None)
        if ev is not None:
            ev.synchronize()

    def _step(self, t, x, cur_hid, *, snr_db, dl_snr_db, pathgain_db, vel, triggers, blockers, _pathgain, _arrivals,
              _dl_arrivals=None):
        cfg = self.config
        if dl_snr_db is not None and self.dl is None:
            raise ValueError("dl_snr_db= needs config.dl = True")
        if pathgain_db is not None:
            if self.C == 1:
                raise ValueError("pathgain_db= needs config.n_cells > 1; use x (poses or SNR) with one cell")
            _pathgain = pathgain_db
        if self.C > 1 and _pathgain is None and (snr_db is not None or x is None or x.dim() != 3):
            raise ValueError("several cells: pass poses [E,R,2|3] or pathgain_db=[E,R,C]")
        if blockers is not None:
            raise B200Unsupported("blockers= (screen blockage) is not built")
        T = self._now(t)
        legacy = cur_hid is not None
        det_hid = cur_hid.to(self.dev, torch.long).contiguous() if legacy else None
        E, R, S, a, p = self.E, self.R, self.S, self._args, self._args.p
        if (self.graphs and self._steps_done > 0 and not legacy and _pathgain is None and _arrivals is None
                and _dl_arrivals is None
                and snr_db is None and x is not None and x.dim() == 3 and self._radio_ready
                and getattr(self, "trace_buf", None) is None and getattr(self, "_kernel_events", None) is None):
            return self._graph_step(T, x)
        self._steps_done += 1
        keep = []                                   # tensors whose pointers the launch reads
        a.det_hid = None
        if det_hid is not None:       # this step's det_env checks cur_hid; last_hid stays the submit's (engine.py:894)
            keep.append(det_hid)
            a.det_hid = det_hid.data_ptr()
        # inputs
        a.pos = a.pathgain_in = a.ul_ref_in = None
        snr_out = snr_in = None
        if _pathgain is not None:
            pg = _pathgain.to(self.dev, torch.float32).contiguous()
            keep.append(pg)
            a.pathgain_in = pg.data_ptr()
        elif snr_db is not None or (x is not None and x.dim() == 2):
            s = snr_db if snr_db is not None else x
            s = s.to(self.dev, torch.float32)
            snr_in = s
            ref = (s if s.dim() == 3 else s[..., None].expand(E, R, S)).contiguous()
            zero = torch.zeros(E, R, device=self.dev)
            keep += [ref, zero]
            a.ul_ref_in, a.pathgain_in = ref.data_ptr(), zero.data_ptr()
            snr_out = s if s.dim() == 2 else s.mean(-1)
        elif x is not None and x.dim() == 3:
            pos = x[..., :2].to(self.dev, torch.float32).contiguous()
            keep.append(pos)
            if not self._radio_ready:
                self._make_radio()
            a.pos = pos.data_ptr()
        else:
            raise ValueError("step needs poses [E,R,2|3] or an SNR [E,R] (x= or snr_db=)")
        rows, rowf, n_ul, rows_dl, n_dlg, n_dl = self._rows(T * self.N)
        p.K_rows = len(rows)
        for k, (r4, f2) in enumerate(zip(rows, rowf)):
            p.rows[k][0], p.rows[k][1], p.rows[k][2], p.rows[k][3] = r4
            p.rowf[k][0], p.rowf[k][1] = f2
        if self.dl:
            p.n_ul_rows, p.n_dl_rows = n_ul, n_dlg
            for k, r4 in enumerate(rows_dl):
                p.rows_dl[k][0], p.rows_dl[k][1], p.rows_dl[k][2], p.rows_dl[k][3] = r4
        p.T = T
        p.s0 = self.s0
        out, o = self._alloc_outputs()
        if self._obstacles and a.pos is None:     # no poses through the radio: no obstacle outputs
            o.blocked = o.los = None
            out.pop("blocked", None)
            out.pop("los", None)
        a.o = o
        tr = getattr(self, "trace_buf", None)
        a.trace = tr.data_ptr() if tr is not None else None
        ev = getattr(self, "_kernel_events", None)      # optional (start, end) CUDA events around the launches
        if ev is not None:
            ev[0].record()
        gen = None
        if self.traffic is not None:
            if _arrivals is not None:
                arr = _arrivals
            elif self.dtraffic is not None:
                arr = self.dtraffic.step()
            else:
                arr = self.traffic.step(self.clock, triggers)
            self.last_arrivals = arr
            M = arr.valid.shape[-1]
            if M > 64:
                raise B200Unsupported(f"{M} traffic arrivals per robot per step (at most 64)")
            fields = {"valid": arr.valid, "det": arr.det, "nbytes": arr.nbytes, "slot": arr.slot, "tag": arr.tag,
                      "prio": arr.prio, "dline": arr.dline}
            for n, v in fields.items():
                v = v.contiguous()
                keep.append(v)
                setattr(a.a, n, v.data_ptr())
            p.M = M
            gen = arr
        else:
            p.M = 0
            for n in nat.ARR_FIELDS:
                setattr(a.a, n, None)
        dl_out = None
        a.dl = None
        if self.dl is not None:      # the DL MAC and finish run inside the same call, before the uplink MAC
            d, dl_out = self.dl.launch_args(a, snr=snr_in, dl_snr=dl_snr_db, arrivals=_dl_arrivals)
            a.dl = ctypes.addressof(d)
        nat.check(self.L.inb_nr_step(ctypes.byref(a), self._stream()), "inb_nr_step")
        if ev is not None:
            ev[1].record()
        self.prb_avail += float(cfg.nprb) * E * n_ul * self.C     # every cell's PRBs (mac.py:491)
        if self.dl is not None:
            self.dl.prb_avail += float(cfg.nprb) * E * n_dl
        self.T = T + 1
        sinr = out.pop("sinr_db") if snr_out is None else snr_out.clone()
        self.pathgain = out.pop("pathgain")
        self._last_snr = sinr                   # this step's output tensor (never modified in place)
        if legacy:
            return out["newest"], out["det_env"]
        res = {k: out[k] for k in ("newest", "det_env", "delivered", "timed_out", "dropped", "cap", "cls", "delay",
                                   "queue_len", "queue_bytes")}
        if self._extras:
            for k in ("arrival", "arrival_slot", "tag", "priority", "bytes", "deadline_miss"):
                res[k] = out[k]
        res["sinr_db"] = sinr
        res["serving_cell"] = out["serving_cell"]
        res["t"] = T - self.epoch
        if gen is not None:
            res["gen_accepted"] = out["gen_accepted"]
            res["gen_bytes"] = out["gen_bytes"]
        for k in ("los", "blocked"):
            if k in out:
                res[k] = out[k]
        if dl_out is not None:         # dl_newest, dl_queue_len; with DL traffic models the dl_* frame outputs
            dl_out["dl_newest"] = dl_out["dl_newest"]
            res.update(dl_out)
        self._keep = keep                           # the launch is asynchronous: keep its inputs alive
        return res

    # ------------------------------------------------------------------ CUDA-graph step
    def _capture(self, key, sched):
        """Capture one control step (traffic generation + the fused launch; with the downlink also its traffic and its
        MAC / finish launches) for this schedule key."""
        rows, rowf, n_ul, rows_dl, n_dlg, n_dl = sched
        a = nat.InbStepArgs.from_buffer_copy(self._args)
        p = a.p
        p.K_rows = len(rows)
        for k, (r4, f2) in enumerate(zip(rows, rowf)):
            p.rows[k][0], p.rows[k][1], p.rows[k][2], p.rows[k][3] = r4
            p.rowf[k][0], p.rowf[k][1] = f2
        if self.dl is not None:
            p.n_ul_rows, p.n_dl_rows = n_ul, n_dlg
            for k, r4 in enumerate(rows_dl):
                p.rows_dl[k][0], p.rows_dl[k][1], p.rows_dl[k][2], p.rows_dl[k][3] = r4
        p.T, p.s0 = 0, self.s0
        a.T_dev = self._ctl.data_ptr()
        a.pos, a.pathgain_in, a.ul_ref_in, a.trace = self._pos_buf.data_ptr(), None, None, None
        a.det_hid = None
        # output pointers as offsets from the block address stored at _ctl[1] (never 0: a null pointer means "absent")
        if getattr(self, "_glay", None) is None:
            self._glay = self._out_layout(0, dl=True)
        o = nat.InbOutputs()
        dl_names = {n for n, dt, shape, f in self.dl.out_spec()} if self.dl is not None else set()
        for n, dt, shape, off, nb in self._glay[0]:
            if n not in dl_names:
                setattr(o, n, self._OFF + off)
        a.o = o
        a.o_base = self._ctl.data_ptr() + 8
        a.dl = None
        dl_offsets = {n: off for n, dt, shape, off, nb in self._glay[0] if n in dl_names}
        dl_tr = self.dl.traffic if self.dl is not None else None
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        if self.traffic is not None and self.dtraffic is None:
            g.register_generator_state(self.traffic.gen)
        if dl_tr is not None and self.dl.dtraffic is None:
            g.register_generator_state(dl_tr.gen)
        arr = dl_arr = None

        def dl_arrivals():
            if dl_tr is None:
                return None
            return self.dl.dtraffic.step() if self.dl.dtraffic is not None else \
                dl_tr.step(self._T_dev - self.epoch, None)

        dl_args = []
        with torch.cuda.graph(g, pool=self._pool):
            if self.dtraffic is not None and self.concurrent_traffic:
                # the traffic kernel and the radio launch on a side stream, concurrent with the fading launch (none
                # of them needs another's results); the MAC launch waits for all
                main = torch.cuda.current_stream(self.dev)
                if getattr(self, "_side", None) is None:
                    self._side = torch.cuda.Stream(self.dev)
                fork = torch.cuda.Event()
                fork.record(main)
                self._side.wait_event(fork)
                with torch.cuda.stream(self._side):
                    arr = self.dtraffic.step()
                    for n in nat.ARR_FIELDS:
                        setattr(a.a, n, getattr(arr, n).data_ptr())
                    p.M = arr.valid.shape[-1]
                    dl_arr = dl_arrivals()
                    if a.rm.on:
                        a.phases = 1
                        nat.check(self.L.inb_nr_step(ctypes.byref(a), self._stream()), "inb_nr_step")
                    join = torch.cuda.Event()
                    join.record(self._side)
                # fading and MAC in one call; the MAC launches also wait for the side stream's arrivals and path
                # gains
                if self.dl is not None:
                    dl_args.append(self.dl.graph_args(a, dl_arr, dl_offsets, self._OFF))
                    a.dl = ctypes.addressof(dl_args[-1])
                a.phases = 6
                nat.check(self.L.inb_nr_step_after(ctypes.byref(a), self._stream(), join._as_parameter_),
                          "inb_nr_step_after")
                a.phases = 0
            else:
                if self.traffic is not None:
                    arr = self.dtraffic.step() if self.dtraffic is not None else \
                        self.traffic.step(self._T_dev - self.epoch, None)
                    for n in nat.ARR_FIELDS:
                        setattr(a.a, n, getattr(arr, n).data_ptr())
                    p.M = arr.valid.shape[-1]
                else:
                    p.M = 0
                if self.dl is not None:
                    dl_arr = dl_arrivals()
                    dl_args.append(self.dl.graph_args(a, dl_arr, dl_offsets, self._OFF))
                    a.dl = ctypes.addressof(dl_args[-1])
                nat.check(self.L.inb_nr_step(ctypes.byref(a), self._stream()), "inb_nr_step")
        ent = {"graph": g, "args": a, "arr": arr, "dl_arr": dl_arr, "dl_args": dl_args}
        self._graphs[key] = ent
        return ent

    _OFF = 256   # bias of the offset-form output pointers

    def _graph_step(self, T, x):
        cfg, E, R = self.config, self.E, self.R
        if self._pos_buf is None:
            self._pos_buf = torch.empty(E, R, 2, dtype=torch.float32, device=self.dev)
        sched = self._rows(T * self.N)
        n_ul, n_dl = sched[2], sched[5]
        key = self._rows_key
        ent = self._graphs.get(key)
        if ent is None:
            ent = self._capture(key, sched)
        # a new output block for this step (the caller owns fresh tensors); the graph writes into it through _ctl[1]
        spec, total = self._glay
        blob = torch.empty(total, dtype=torch.uint8, device=self.dev)
        self._pos_buf.copy_(x[..., :2], non_blocking=True)
        nat.check(self.L.inb_store2(self._ctl.data_ptr(), T, blob.data_ptr() - self._OFF, self._stream()),
                  "inb_store2")
        ent["graph"].replay()
        self._steps_done += 1
        self.last_arrivals = ent["arr"]
        out = {n: blob[off:off + nb].view(dt).view(shape) for n, dt, shape, off, nb in spec}
        self.prb_avail += float(cfg.nprb) * E * n_ul * self.C     # every cell's PRBs (mac.py:491)
        self.T = T + 1
        sinr = out.pop("sinr_db")
        self.pathgain = out.pop("pathgain")
        self._last_snr = sinr                   # this step's output tensor (never modified in place)
        res = {k: out[k] for k in ("newest", "det_env", "delivered", "timed_out", "dropped", "cap", "cls", "delay",
                                   "queue_len", "queue_bytes")}
        if self._extras:
            for k in ("arrival", "arrival_slot", "tag", "priority", "bytes", "deadline_miss"):
                res[k] = out[k]
        res["sinr_db"] = sinr
        res["serving_cell"] = out["serving_cell"]
        res["t"] = T - self.epoch
        if self.traffic is not None:
            res["gen_accepted"] = out["gen_accepted"]
            res["gen_bytes"] = out["gen_bytes"]
        for k in ("los", "blocked"):
            if k in out:
                res[k] = out[k]
        if self.dl is not None:       # dl_newest, dl_queue_len; with DL traffic models the dl_* frame outputs
            self.dl.prb_avail += float(cfg.nprb) * E * n_dl
            if self.dl.traffic is not None:
                self.dl.last_arrivals = ent["dl_arr"]
            res.update({n: out[n] for n, dt, shape, f in self.dl.out_spec()})
        return res

    # ------------------------------------------------------------------ observability
    def counters(self):
        """{"ul": counters[, "dl": counters]} as NRNet.counters() (nr_engine.py:916-925), folded from the per-env
        device words."""
        res = self.fold_counters(self.ctr.sum(0), self.prb_avail)
        if self.dl is not None:
            res["dl"] = self.dl.counters()
        return res

    def fold_counters(self, c, prb_avail):
        """counters() from a summed counter vector c [INB_NCTR] and the PRBs offered (also for sums over shards)."""
        c = c.cpu()
        res = {k: float(c[i]) for i, k in enumerate(nat.CTR_NAMES)}
        if self.config.lena_mac_switches():      # grant accounting of the 5G-LENA switches (mac.py:119-121)
            for i, k in enumerate(nat.LENA_CTR_NAMES):
                res[k] = float(c[len(nat.CTR_NAMES) + i])
        res["prb_avail"] = float(prb_avail)
        H = self.config.max_harq_tx + 1
        res["ntx_hist"] = [float(v) for v in c[nat.CTR_NTX_HIST:nat.CTR_NTX_HIST + H]]
        res["rv_tx"] = [float(v) for v in c[nat.CTR_RV_TX:nat.CTR_RV_TX + H]]
        res["rv_fail"] = [float(v) for v in c[nat.CTR_RV_FAIL:nat.CTR_RV_FAIL + H]]
        return {"ul": res}

    def queued(self):
        return (self.st["cap"] >= 0).sum(-1)

    def output_schema(self):
        """{key: {"shape", "dtype"}} of the keys step() returns under this config."""
        E, R, F = self.E, self.R, self.F
        sch = {"newest": ((E, R), "int64"), "det_env": ((E,), "bool"), "delivered": ((E, R, F), "bool"),
               "timed_out": ((E, R, F), "bool"), "dropped": ((E, R, F), "bool"), "cap": ((E, R, F), "int64"),
               "cls": ((E, R, F), "int64"), "delay": ((E, R, F), "float32"), "queue_len": ((E, R), "int64"),
               "queue_bytes": ((E, R), "float32"), "sinr_db": ((E, R), "float32"),
               "serving_cell": ((E, R), "int64"), "t": ((E,), "int64")}
        if self._extras:
            sch.update({"arrival": ((E, R, F), "float64"), "arrival_slot": ((E, R, F), "int64"),
                        "tag": ((E, R, F), "int64"), "priority": ((E, R, F), "int64"),
                        "bytes": ((E, R, F), "int64"), "deadline_miss": ((E, R, F), "bool")})
        if self.traffic is not None:
            sch.update({"gen_accepted": ((E, R), "int64"), "gen_bytes": ((E, R), "int64")})
        if self._obstacles:        # with poses through the radio
            sch["blocked"] = ((E, R), "bool")
            if self.config.channel == "tr38901":
                sch["los"] = ((E, R), "bool")
        return {k: {"shape": s, "dtype": d} for k, (s, d) in sch.items()}

    # ------------------------------------------------------------------ checkpoints (core/checkpoint.py:1-60, 115-160)
    _HOST = ("T", "_uniform_epoch", "last_g", "prb_avail", "env_offset", "_steps_done", "seed")
    _DEV = ("env_id", "episode", "rng_ctr", "ctr", "status", "epoch", "_last_hid", "_last_snr")

    def state_dict(self):
        """Every piece of engine state as a flat dict {key: tensor clone | host value}: the per-robot MAC / HARQ /
        queue / fading / association state, the counter-RNG rows, per-env clocks and counters, the radio's draws
        (made at the first step with poses), the traffic models' state and generator positions, and the host
        clocks.  load_state_dict on an engine of the same config and size continues exactly like this one (bitwise,
        same device), as the reference's engine.state_dict() / load_state_dict() guarantee."""
        sd = {"meta.level": "L2", "meta.backend": "b200", "meta.E": self.E, "meta.R": self.R,
              "meta.config": repr(sorted(self.config.field_dict().items()))}
        for n, t in self.st.items():
            sd["st." + n] = t.clone()
        for n in self._DEV:
            sd["eng." + n] = getattr(self, n).clone()
        for n in self._HOST:
            sd["host." + n] = getattr(self, n)
        if getattr(self, "pathgain", None) is not None:
            sd["eng.pathgain"] = self.pathgain.clone()
        if self.dl is not None:            # the downlink: state, counters, DL traffic models
            for n, t in self.dl.st.items():
                sd["dl.st." + n] = t.clone()
            sd["dl.ctr"], sd["dl.prb_avail"] = self.dl.ctr.clone(), self.dl.prb_avail
            tg = self.dl.traffic
            if tg is not None:
                sd["dl.traffic.gen"], sd["dl.traffic.rgen"] = tg.gen.get_state(), tg.rgen.get_state()
                for i, src in enumerate(tg.sources):
                    for n in src.names:
                        sd[f"dl.traffic.src{i}.{n}"] = getattr(src, n).clone()
                    sd[f"dl.traffic.src{i}.deferred"] = src.deferred.clone()
                if self.dl.dtraffic is not None:
                    sd["dl.traffic.calls"] = self.dl.dtraffic.calls.clone()
        if self._radio_ready:
            sd["radio.ready"] = True
            if self._fields is not None:
                sd["radio.k"], sd["radio.phi"] = self._fields[0].clone(), self._fields[1].clone()
            if self._blk is not None:
                for n, t in self._blk.items():
                    sd["radio.blk." + n] = t.clone()
                sd["radio.blk.t"] = self._blk_t.clone()
        if self.traffic is not None:
            tg = self.traffic
            sd["traffic.gen"], sd["traffic.rgen"] = tg.gen.get_state(), tg.rgen.get_state()
            for i, src in enumerate(tg.sources):
                for n in src.names:
                    sd[f"traffic.src{i}.{n}"] = getattr(src, n).clone()
                sd[f"traffic.src{i}.deferred"] = src.deferred.clone()
            if self.dtraffic is not None:
                sd["traffic.calls"] = self.dtraffic.calls.clone()
            elif tg.counter is not None:     # host steps of the counter stream: its key
                sd["traffic.calls"] = tg.calls.clone()
        return sd

    def load_state_dict(self, sd, strict=True):
        """Restore a state_dict() in place: tensors are copied into the engine's own buffers (so captured CUDA graphs
        keep reading the right memory), generator states and host values are set.  strict: raise on keys that do
        not belong to this engine and on missing ones (else skip them); the size and config must match."""
        if sd.get("meta.level") != "L2" or sd.get("meta.backend") != "b200":
            raise ValueError("not a state_dict of the B200 L2 engine")
        if (sd.get("meta.E"), sd.get("meta.R")) != (self.E, self.R):
            raise ValueError(f"state_dict for E, R = {sd.get('meta.E')}, {sd.get('meta.R')}; this engine has "
                             f"{self.E}, {self.R}")
        if sd.get("meta.config") != repr(sorted(self.config.field_dict().items())):
            raise ValueError("state_dict of an engine with another config")
        mine = set(self.state_dict()) | {"radio.ready", "radio.k", "radio.phi", "radio.blk.k", "radio.blk.phi",
                                         "radio.blk.xk", "radio.blk.yk", "radio.blk.vel", "radio.blk.t",
                                         "eng.pathgain"}
        extra = set(sd) - mine
        missing = {k for k in self.state_dict() if not k.startswith(("radio.", "eng.pathgain"))} - set(sd)
        if strict and (extra or missing):
            raise KeyError(f"state_dict keys not placed: {sorted(extra)}; missing: {sorted(missing)}")
        cp = lambda dst, key: dst.copy_(sd[key].to(dst.device)) if key in sd else None   # noqa: E731
        for n, t in self.st.items():
            cp(t, "st." + n)
        for n in self._DEV:
            key = "eng." + n
            if key not in sd:
                continue
            if n == "_last_snr":
                self._last_snr = sd[key].to(self.dev).clone()
            else:
                cp(getattr(self, n), key)
        old_seed = self.seed
        for n in self._HOST:
            if "host." + n in sd:
                setattr(self, n, sd["host." + n])
        if self.seed != old_seed:            # the seed key is baked into captured steps
            self.s0 = seed_key(self.seed)
            self._args.p.s0 = self.s0
            self._graphs.clear()
        if "eng.pathgain" in sd:
            self.pathgain = sd["eng.pathgain"].to(self.dev).clone()
        if self.dl is not None:
            for n, t in self.dl.st.items():
                cp(t, "dl.st." + n)
            cp(self.dl.ctr, "dl.ctr")
            self.dl.prb_avail = sd.get("dl.prb_avail", self.dl.prb_avail)
            tg = self.dl.traffic
            if tg is not None:
                if "dl.traffic.gen" in sd:
                    tg.gen.set_state(sd["dl.traffic.gen"])
                    tg.rgen.set_state(sd["dl.traffic.rgen"])
                for i, src in enumerate(tg.sources):
                    for n in src.names:
                        cp(getattr(src, n), f"dl.traffic.src{i}.{n}")
                    cp(src.deferred, f"dl.traffic.src{i}.deferred")
                if self.dl.dtraffic is not None:
                    cp(self.dl.dtraffic.calls, "dl.traffic.calls")
        if sd.get("radio.ready"):
            if not self._radio_ready:
                self._make_radio()
            if self._fields is not None:
                cp(self._fields[0], "radio.k")
                cp(self._fields[1], "radio.phi")
            if self._blk is not None:
                for n, t in self._blk.items():
                    cp(t, "radio.blk." + n)
                cp(self._blk_t, "radio.blk.t")
        elif self._radio_ready:              # the source had not made its radio yet: neither has this engine now
            self._radio_ready = False
            self._graphs.clear()
        if self.traffic is not None:
            tg = self.traffic
            if "traffic.gen" in sd:
                tg.gen.set_state(sd["traffic.gen"])
                tg.rgen.set_state(sd["traffic.rgen"])
            for i, src in enumerate(tg.sources):
                for n in src.names:
                    cp(getattr(src, n), f"traffic.src{i}.{n}")
                cp(src.deferred, f"traffic.src{i}.deferred")
            if self.dtraffic is not None:
                cp(self.dtraffic.calls, "traffic.calls")
            elif tg.counter is not None:
                cp(tg.calls, "traffic.calls")

    def reference_checkpoint(self):
        """This engine's state under the keys of the reference engine's state_dict() (isaac_net/core/checkpoint.py:
        MAC, queue, fading, clocks, RNG counters, association, radio fields, traffic-model state, counters; the
        mapping is in isaac-net_b200/checkpoint.py), CPU tensors."""
        from . import checkpoint
        return checkpoint.save(self)

    def load_reference_checkpoint(self, sd, strict=False):
        """Continue from a checkpoint the reference engine wrote (its state_dict(), a flat dict of tensors and host
        values): the state is copied in place; returns the keys not used (constants, scratch and generator states
        of the reference's object graph).  strict: raise when a key naming state could not be placed."""
        from . import checkpoint
        return checkpoint.load(self, sd, strict=strict)

    def save(self, path, extra=None):
        """state_dict() (plus `extra`) to a file (torch.save), as checkpoint.save(net, path, extra=...)."""
        torch.save({"format": 1, "state": self.state_dict(), "extra": extra}, path)

    def load(self, path, strict=True):
        """Restore a file written by save(); returns its `extra`."""
        d = torch.load(path, map_location="cpu", weights_only=False)
        self.load_state_dict(d["state"], strict=strict)
        return d.get("extra")

    # ------------------------------------------------------------------ state exchange (reference names)
    _REF = {"ul.sent": "sent", "ul.floor": "floor_", "ul.olla": "olla", "ul.avg": "avg", "ul.bsr": "bsr",
            "ul.sr_t": "sr_t", "ul.last_tx": "last_tx", "ul.csi": "csi", "ul.h_state": "h_state",
            "ul.h_lo": "h_lo", "ul.h_hi": "h_hi", "ul.h_ready": "h_ready", "ul.h_ntx": "h_ntx",
            "ul.h_mcs": "h_mcs", "ul.h_tbs": "h_tbs", "ul.h_nsb": "h_nsb", "ul.h_comb": "h_comb",
            "q.cap": "cap", "q.start": "start", "q.end": "end_", "q.lost": "lost", "q.fin": "fin", "q.enq": "enq",
            "q.cls": "cls", "q.det": "det", "q.hid": "hid", "q.off": "off", "q.tag": "tag", "q.prio": "prio",
            "q.dline": "dline", "net.h": "h", "net.spec": "spec", "net.k_lin": "k_lin", "assoc.serv": "serv",
            "assoc.a3_cand": "a3_cand", "assoc.a3_cnt": "a3_cnt", "assoc.ho_end": "ho_end", "assoc.n_ho": "n_ho",
            "assoc.pending": "pending", "net.ni_ul": "ni_ul", "ul.last_nprb": "last_nprb",
            "ul.est": "bsr_est", "ul.boot": "bsr_boot", "ul.rep_v": "bsr_rep_v", "ul.rep_g": "bsr_rep_g",
            "ul.hid": "bsr_hid", "ul.hid_until": "bsr_hid_until", "ul.enq_seen": "bsr_enq_seen",
            "ul.armed": "bsr_armed"}

    # the radio field the kernel evaluates, under the reference's names (RadioMC.k / phi for log_distance,
    # TR38901Channel.sf_los for tr38901 with the forced LOS state)
    _FIELD_KEYS = {"log_distance": ("radio.k", "radio.phi"), "tr38901": ("radio.sf_los.k", "radio.sf_los.phi")}

    def reference_state(self):
        """Engine state under the reference's names (ul.*, q.*, net.*, rng.*, eng.*), device tensors (views)."""
        out = {k: self.st[v] for k, v in self._REF.items() if v in self.st}
        out["net.last_g"] = torch.tensor(-1 if self.last_g is None else self.last_g)
        out["rng.episode"], out["rng.ctr_step"] = self.episode, self.rng_ctr
        out["eng.T"], out["eng.epoch"] = torch.tensor(self.T), self.epoch
        out["eng.last_snr"], out["eng.last_hid"] = self._last_snr, self._last_hid
        if self.C > 1 and getattr(self, "pathgain", None) is not None:
            out["net.pg"] = self.pathgain
        if self._blk is not None:
            for n, v in self._blk.items():
                out["radio.blk." + n] = v
            out["radio.blk.t"] = self._blk_t
        if self._fields is not None and self.config.channel in self._FIELD_KEYS:
            kk, pk = self._FIELD_KEYS[self.config.channel]
            out[kk], out[pk] = self._fields
        if self.dl is not None:            # the downlink MacLink and its queue (net.dl.*, net.dl.q.*)
            for k, v in DL_REF.items():
                out[k] = self.dl.st[v]
        return out

    def load_reference_state(self, snap):
        """Copy a state dict keyed by the reference's names into the engine's buffers (in place).  The radio's draws
        are a function of (seed, env id, episode): envs whose episode the snapshot changes get theirs redrawn, and
        the blockage clock and draws (radio.blk.*) are taken from the snapshot when it has them."""
        ep0 = self.episode.clone()
        blk, fld = {}, {}
        for k, v in snap.items():
            t = torch.as_tensor(np.asarray(v) if not torch.is_tensor(v) else v)
            if k.startswith("radio.blk."):
                blk[k[len("radio.blk."):]] = t
            elif k in self._FIELD_KEYS.get(self.config.channel, ()):
                fld[k] = t
            elif k in self._REF and self._REF[k] in self.st:
                self.st[self._REF[k]].copy_(t.to(self.dev))
            elif k in DL_REF and self.dl is not None:
                self.dl.st[DL_REF[k]].copy_(t.to(self.dev))
            elif k == "net.last_g":
                self.last_g = None if int(t) < 0 else int(t)
            elif k == "rng.episode":
                self.episode.copy_(t.to(self.dev))
            elif k == "rng.ctr_step":
                self.rng_ctr.copy_(t.to(self.dev))
            elif k == "eng.T":
                self.T = int(t)
            elif k == "eng.epoch":
                self.epoch.copy_(t.to(self.dev))
            elif k == "eng.last_snr":
                self._last_snr = t.to(self.dev, torch.float32).clone()
            elif k == "eng.last_hid":
                self._last_hid.copy_(t.to(self.dev))
        if self._radio_ready:
            changed = self.episode != ep0
            if bool(changed.any()):
                self._reset_radio(changed)
        if (blk and self.config.blockage) or fld:
            if not self._radio_ready:
                self._make_radio()
        if blk and self.config.blockage:
            for n, t in blk.items():
                (self._blk_t if n == "t" else self._blk[n]).copy_(t.to(self.dev))
        if fld and self._fields is not None:    # the shadowing field the kernel evaluates: wave vectors, phases
            kk, pk = self._FIELD_KEYS[self.config.channel]
            for key, buf in ((kk, self._fields[0]), (pk, self._fields[1])):
                if key in fld:
                    buf.copy_(fld[key].to(self.dev))
        if torch.any(self.epoch != 0):
            self._uniform_epoch = None


__all__ = ["make_engine", "NRB200Engine", "B200Unsupported", "seed_key"]
