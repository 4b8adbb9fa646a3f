"""NRConfig: the configuration dataclass of the NR uplink engine (level "L2").

Field names, defaults and the derived quantities follow isaac_net's ``NRConfig``
(isaac_net/core/config.py:477-1496) for every field the uplink control-step path reads, so a config written for the
reference builds here unchanged.  Fields the B200 engine does not implement are still accepted (same defaults) and
``refusals()`` names the ones set away from their defaults, as ``NRTritonEngine.refusals`` does for the Triton
backend (isaac_net/core/nr_fast.py:539-554).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, fields, replace

# TS 38.101-1 Table 5.3.2-1: N_RB per (SCS kHz, bandwidth MHz), FR1 (isaac_net/core/config.py:24-30)
NRB_FR1 = {
    15: {5: 25, 10: 52, 15: 79, 20: 106, 25: 133, 30: 160, 35: 188, 40: 216, 45: 242, 50: 270},
    30: {5: 11, 10: 24, 15: 38, 20: 51, 25: 65, 30: 78, 35: 92, 40: 106, 45: 119, 50: 133,
         60: 162, 70: 189, 80: 217, 90: 245, 100: 273},
    60: {10: 11, 15: 18, 20: 24, 25: 31, 30: 38, 35: 44, 40: 51, 45: 58, 50: 65,
         60: 79, 70: 93, 80: 107, 90: 121, 100: 135},
}
# TS 38.214 Table 5.1.2.2.1-1: (largest BWP size, RBG size config 1, config 2)
_RBG_ROWS = ((36, 2, 4), (72, 4, 8), (144, 8, 16), (275, 16, 16))


def rbg_size_38214(n_prb, config=1):
    """Nominal RBG size P for a bandwidth part of n_prb PRBs (TS 38.214 Table 5.1.2.2.1-1)."""
    for top, p1, p2 in _RBG_ROWS:
        if n_prb <= top:
            return p1 if config == 1 else p2
    raise ValueError(f"no RBG size for {n_prb} PRBs")


@dataclass
class NRConfig:
    """Configuration of the NR uplink engine; every field has the reference's default."""
    # numerology and carrier
    mu: int = 1
    bandwidth_mhz: int = 20
    n_prb: int | None = None
    rbg_size: int | None = None
    rbg_config: int = 1
    duplex: str = "tdd"
    tdd_pattern: str = "DDDSU"
    special_split: tuple = (10, 2, 2)
    special_dl_data: bool = True
    special_ul_data: bool = False
    dl_ctrl_symbols: int = 1
    ul_data_symbols: int = 12
    ul_mini_slot_symbols: int | None = None
    mini_slot_dl: bool = False
    dl_n_prb: int | None = None
    dl_bandwidth_mhz: int | None = None
    dmrs_re_per_prb: int = 12
    overhead_re_per_prb: int = 0
    # MAC timing (slots)
    k1: int = 2
    k2: int = 2
    gnb_proc_slots: int = 1
    sr_period_slots: int = 5
    sr_grant_delay_slots: int | None = None
    ul_harq_rtt_slots: int | None = None
    cqi_period_slots: int = 10
    proactive_grant: str = "off"
    proc_offset_ms: float = 0.0
    # HARQ / RLC
    n_harq: int = 16
    max_harq_tx: int = 4
    harq_combining: str = "cc"
    harq_fail: str = "rlc_am"
    rlc_retx_slots: int = 50
    discard: str = "purge"
    # PHY abstraction / link adaptation
    mcs_table: int = 1
    eff_sinr: str = "eesm"
    bler_source: str = "pdsch"
    tbs_mode: str = "38214"
    bler_target: float = 0.1
    ul_mcs_max: int | None = None
    dl_mcs_max: int | None = None
    cqi_table: str = "mcs"               # DL CQI quantization: the MCS grid ("mcs") or TS 38.214's 4-bit CQI ("38214")
    dl_snr_offset_db: float = 10.0       # SNR input: default DL per-PRB SNR = UL input SNR + offset
    olla: bool = True
    olla_up_db: float = 0.05
    scheduler: str = "pf"
    pf_metric: str = "subband"
    pf_window: float = 100.0
    retx_priority: bool = True
    n_layers_max: int = 1
    pf_update: str = "slot"
    pf_avg_idle: str = "decay"
    ul_retx_sched: str = "ofdma"
    ul_amc_alloc: str = "current"
    ul_grant_model: str = "lumped"
    # ul_grant_model = "bsr": the 5G-LENA SR / BSR pipeline (isaac_net/core/config.py:588-594)
    sr_boot_slots: int = 6
    sr_boot_bytes: int = 17
    bsr_delay_slots: int = 10
    bsr_hdr_bytes: int = 8
    bsr_est_hdr_bytes: int = 5
    rlc_tail_bytes: int = 16
    rlc_tail_timer_ms: float = 10.0
    # radio model inside the engine
    snr_ref_prbs: int = 10
    ul_power: str = "allocated"
    phr_cap: bool = True
    phr_min_db: float = 3.0
    fading: bool = True
    fading_rho_per_ms: float = 0.93 ** (1 / 2.5)
    ue_speed_mps: float | None = None
    carrier_ghz: float = 3.5
    fading_doppler: str = "global"
    fading_rician: bool = False
    rician_k_db: float | None = None
    rician_k_from_los: bool = True
    rician_k_ramp_slots: int = 4
    fading_freq_corr: bool = False
    # link budget
    noise_model: str = "fixed"
    ni_fixed_dbm: float = -90.0
    gnb_nf_db: float = 5.0
    ue_nf_db: float = 9.0
    ue_tx_dbm: float = 23.0
    gnb_tx_dbm: float = 43.0
    tb_overhead_bytes: int = 0
    pkt_payload_bytes: int = 1400
    pkt_overhead_bytes: int = 0
    # large-scale channel
    pl_const_db: float = 40.0
    pathloss_exp: float = 3.5
    shadow_sigma_db: float = 6.0
    shadow_modes: int = 8
    shadow_dcorr_m: float = 10.3
    shadow_acf: str = "sos"
    shadow_white_frac: float = 0.0
    channel: str = "log_distance"
    tr38901_scenario: str = "InF-SH"
    tr38901_los: str = "stochastic"
    gnb_height_m: float | None = None
    ue_height_m: float = 1.5
    o2i_indoor_frac: float = 0.0
    radio_map_path: str | None = None
    blockage: bool = False
    blockage_model: str = "sphere"
    blockage_max_db: float = 40.0
    los_source: str = "stochastic"
    # cells
    n_cells: int = 1
    cell_layout: str = "custom"
    cell_positions_m: tuple = ((0.0, 0.0),)
    cell_isd_m: float = 100.0
    cell_center_m: tuple = (75.0, 75.0)
    cell_arena_m: float = 150.0
    gnb_antenna: str = "isotropic"
    ul_interference: bool = True
    dl_interference: bool = True
    li_alpha: float = 1.0
    ul_pc: bool | None = None
    ul_pc_p0_dbm: float = -88.0
    ul_pc_alpha: float = 1.0
    ul_tpc: bool = False
    a3_offset_db: float = 0.0
    a3_hyst_db: float = 3.0
    a3_ttt_ms: float = 300.0
    ho_interruption_ms: float = 40.0
    ho_rlc: str = "carry"
    a3_min_target_rsrp_dbm: float | None = None
    rlf: bool = False
    rach: bool = False
    drx: bool = False
    # directions and application
    ul: bool = True
    dl: bool = False
    control_step_ms: float = 100.0
    frame_buffer: int = 16
    timeout_steps: int = 20
    msg_sizes: tuple = (4000.0, 30000.0)
    traffic: tuple | None = None
    # randomness
    seed: int | None = None
    rng: str = "engine"

    def __post_init__(self):
        from .traffic import normalize_traffic
        self.traffic = normalize_traffic(self.traffic)
        self.msg_sizes = tuple(float(s) for s in self.msg_sizes)
        self.cell_positions_m = tuple(tuple(float(v) for v in p) for p in self.cell_positions_m)
        if self.ue_speed_mps is not None:
            raise ValueError("ue_speed_mps (Jakes rho from a speed) is not implemented by the B200 engine; set "
                             "fading_rho_per_ms directly")
        if self.channel.startswith("tr38901_"):
            short = {"tr38901_rma": "RMa", "tr38901_uma": "UMa", "tr38901_umi": "UMi", "tr38901_inh": "InH"}
            if self.channel not in short:
                raise ValueError(f"channel {self.channel!r} is not supported")
            self.channel, self.tr38901_scenario = "tr38901", short[self.channel]
        assert self.mu in (0, 1, 2) and set(self.tdd_pattern) <= set("DSU") and self.tdd_pattern
        assert sum(self.special_split) == 14 and 1 <= self.n_cells <= 7
        assert self.frame_buffer >= 1 and self.timeout_steps >= 1 and self.control_step_ms > 0
        if self.cell_layout == "custom":
            assert len(self.cell_positions_m) == self.n_cells, "custom layout: one position per cell"

    def with_(self, **kw):
        return replace(self, **kw)

    # ------------------------------------------------------------------ derived (config.py:875-1110)
    @property
    def scs_khz(self):
        return 15 * 2 ** self.mu

    @property
    def slot_ms(self):
        return 1.0 / 2 ** self.mu

    @property
    def nprb(self):
        if self.n_prb is not None:
            return self.n_prb
        tab = NRB_FR1[self.scs_khz]
        if self.bandwidth_mhz not in tab:
            raise ValueError(f"{self.bandwidth_mhz} MHz not defined at {self.scs_khz} kHz")
        return tab[self.bandwidth_mhz]

    @property
    def rbg(self):
        return self.rbg_size if self.rbg_size is not None else rbg_size_38214(self.nprb, self.rbg_config)

    @property
    def n_subbands(self):
        return math.ceil(self.nprb / self.rbg)

    @property
    def subband_prbs(self):
        s = [self.rbg] * self.n_subbands
        s[-1] = self.nprb - self.rbg * (self.n_subbands - 1)
        return s

    @property
    def slots_per_step(self):
        n = self.control_step_ms / self.slot_ms
        assert abs(n - round(n)) < 1e-9, "control step must be a whole number of slots"
        return int(round(n))

    def slot_symbols(self, pos):
        """(DL data symbols, UL data symbols) of the slot at pattern position pos."""
        if self.duplex == "fdd":
            return 14 - self.dl_ctrl_symbols, self.ul_data_symbols
        c = self.tdd_pattern[pos % len(self.tdd_pattern)]
        if c == "D":
            return 14 - self.dl_ctrl_symbols, 0
        if c == "U":
            return 0, self.ul_data_symbols
        dl = self.special_split[0] - self.dl_ctrl_symbols if self.special_dl_data else 0
        ul = self.special_split[2] if self.special_ul_data else 0
        return max(dl, 0), ul

    def ul_capable(self, pos):
        if self.duplex == "fdd":
            return True
        c = self.tdd_pattern[pos % len(self.tdd_pattern)]
        return c == "U" or (c == "S" and self.special_split[2] > 0)

    def first_ul_in_window(self, g, period):
        if not self.ul_capable(g):
            return False
        return not any(self.ul_capable(x) for x in range(period * (g // period), g))

    @property
    def sr_delay(self):
        return self.sr_grant_delay_slots if self.sr_grant_delay_slots is not None else self.gnb_proc_slots + self.k2

    @property
    def ul_rtt(self):
        return self.ul_harq_rtt_slots if self.ul_harq_rtt_slots is not None else self.gnb_proc_slots + self.k2

    @property
    def ul_pc_on(self):
        return self.n_cells > 1 if self.ul_pc is None else bool(self.ul_pc)

    @property
    def rician_mode(self):
        if not (self.fading and self.fading_rician):
            return None
        if self.rician_k_db is not None:
            return "fixed"
        return "los" if self.rician_k_from_los else None

    def noise_dbm_per_prb(self, rx="gnb"):
        if self.noise_model == "fixed":
            return self.ni_fixed_dbm - 10 * math.log10(self.snr_ref_prbs)
        nf = self.gnb_nf_db if rx == "gnb" else self.ue_nf_db
        return -174.0 + 10 * math.log10(12 * self.scs_khz * 1e3) + nf

    @property
    def subband_noise_dbm(self):
        return self.noise_dbm_per_prb("gnb") + 10 * math.log10(self.snr_ref_prbs)

    def gnb_xy(self):
        """gNB positions (env-local metres), as NRConfig.gnb_xy (config.py:1417-1434)."""
        n = self.n_cells
        if self.cell_layout == "custom":
            return [tuple(map(float, p)) for p in self.cell_positions_m]
        if self.cell_layout == "hex":
            isd = self.cell_isd_m
            pts = [(0.0, 0.0)] + [(isd * math.cos(math.pi / 3 * j), isd * math.sin(math.pi / 3 * j))
                                  for j in range(6)]
            pts = pts[:n]
            cx, cy = sum(p[0] for p in pts) / n, sum(p[1] for p in pts) / n
            return [(p[0] - cx + self.cell_center_m[0], p[1] - cy + self.cell_center_m[1]) for p in pts]
        cols = math.ceil(math.sqrt(n))
        rows = math.ceil(n / cols)
        a = self.cell_arena_m
        return [((j % cols + 0.5) * a / cols, (j // cols + 0.5) * a / rows) for j in range(n)]

    def next_ul_capable(self, g):
        """Smallest slot index >= g that is UL-capable (config.py:1070-1076)."""
        for d in range(len(self.tdd_pattern)):
            if self.ul_capable(g + d):
                return g + d
        raise ValueError("pattern has no UL-capable slot")

    def schedule(self, g0):
        """Scheduled slots of the control step starting at slot g0, the rows of NRNet._schedule
        (isaac_net/core/nr_engine.py:506-523): [(rel, DL data symbols, UL data symbols, SR opportunity, CQI report,
        HARQ-ACK slot relative to g0)]."""
        out = []
        for rel in range(self.slots_per_step):
            g = g0 + rel
            dls, uls = self.slot_symbols(g)
            dls = dls if self.dl else 0
            uls = uls if self.ul else 0
            sr = self.first_ul_in_window(g, self.sr_period_slots) and self.ul
            cqi = self.first_ul_in_window(g, self.cqi_period_slots) and self.dl
            if dls or uls or cqi or sr:
                ack = self.next_ul_capable(g + self.k1) - g0 if self.dl else 0
                out.append((rel, dls, uls, bool(sr), bool(cqi), ack))
        return out

    def schedule_period(self):
        """Period (in slots) after which the schedule of a control step repeats."""
        return math.lcm(len(self.tdd_pattern), self.sr_period_slots, self.cqi_period_slots)

    @property
    def rlc_tail_timer_slots(self):
        """ul_grant_model="bsr": the RLC buffer-status timer in slots, at least one (config.py:1088-1090)."""
        return max(1, int(round(self.rlc_tail_timer_ms / self.slot_ms)))

    def lena_mac_switches(self):
        """The 5G-LENA MAC switches set away from their defaults, {field: value} (config.py:1092-1094)."""
        d = {"pf_update": "slot", "pf_avg_idle": "decay", "ul_retx_sched": "ofdma", "ul_amc_alloc": "current",
             "ul_grant_model": "lumped"}
        return {k: getattr(self, k) for k, v in d.items() if getattr(self, k) != v}

    def field_dict(self):
        """{field: value} of every field (the plain form the reference's NRConfig(**...) takes, traffic aside)."""
        return {f.name: getattr(self, f.name) for f in fields(self)}

    # ------------------------------------------------------------------ what the B200 engine runs
    def refusals(self):
        """[(feature, why)] of settings the B200 engine does not implement (empty: it runs)."""
        out = []
        d = NRConfig()
        # the SR/BSR pipeline fields (sr_boot_*, bsr_*, rlc_tail_*) are read only under ul_grant_model="bsr"
        # (reference config.py:119, 307), so a lumped config keeps whatever values they hold
        chk = [("ul_mini_slot_symbols", "mini-slot occasions are not built"),
               ("mini_slot_dl", "mini-slot occasions are not built"),
               ("dl_n_prb", "FDD's paired downlink carrier is not built"),
               ("dl_bandwidth_mhz", "FDD's paired downlink carrier is not built"),
               ("n_layers_max", "rank-2 MIMO is not built"),
               ("ul_tpc", "closed-loop power control is not built"),
               ("eff_sinr", "only EESM is built"),
               ("bler_source", "only the shipped Sionna PDSCH tables are built"),
               ("tbs_mode", "only the exact 38.214 TBS is built"),
               ("pf_metric", "only the subband PF metric is built"),
               ("fading_freq_corr", "frequency-correlated fading is not built"),
               ("fading_doppler", "per-robot Doppler is not built"),
               ("proactive_grant", "proactive grants are not built"),
               ("rach", "the access state machine is not built"),
               ("drx", "the access state machine is not built"),
               ("rlf", "radio link failure is not built"),
               ("duplex", "FDD is not built"),
               ("gnb_antenna", "sector antennas are not built"),
               ("o2i_indoor_frac", "O2I penetration is not built"),
               ("shadow_white_frac", "the white shadowing component is not built"),
               ("pkt_overhead_bytes", "per-packet overhead is not built"),
               ("rng", "only the engine counter RNG is built")]
        for name, why in chk:
            if getattr(self, name) != getattr(d, name):
                out.append((f"{name}={getattr(self, name)!r}", why))
        if self.ul_retx_sched not in ("ofdma", "tdma") or self.ul_amc_alloc not in ("current", "previous"):
            out.append((f"ul_retx_sched={self.ul_retx_sched!r} / ul_amc_alloc={self.ul_amc_alloc!r}",
                        "unknown 5G-LENA MAC option"))
        if self.pf_update not in ("slot", "rbg") or self.pf_avg_idle not in ("decay", "freeze"):
            out.append((f"pf_update={self.pf_update!r} / pf_avg_idle={self.pf_avg_idle!r}", "unknown PF option"))
        if self.pf_update == "rbg" and self.scheduler != "pf":
            out.append((f"pf_update='rbg' with scheduler={self.scheduler!r}", "per-RBG PF updates need the pf "
                                                                              "scheduler"))
        if self.scheduler not in ("pf", "rr", "maxci"):
            out.append((f"scheduler={self.scheduler!r}", "schedulers built: pf, rr, maxci"))
        if self.harq_combining not in ("cc", "none"):
            out.append((f"harq_combining={self.harq_combining!r}", "combining built: cc, none"))
        if self.discard == "pdcp_arrival":
            out.append(("discard='pdcp_arrival'", "PDCP arrival discard is not built"))
        if self.rician_mode == "los":
            out.append(("Rician K from the LOS state", "only a fixed rician_k_db is built"))
        if self.n_cells > 3:
            out.append((f"n_cells={self.n_cells}", "at most 3 cells (more need an ordered interference sum)"))
        if self.dl and self.n_cells > 1:
            out.append(("dl with n_cells > 1", "the downlink with several cells (DL interference) is not built"))
        # ho_rlc="flush" under traffic models: the reference keeps the step's later arrivals through a flush (its
        # handover wrapper, engine.py:486-497); the kernels' handover drops them too
        if self.ho_rlc == "flush" and self.n_cells > 1 and any(m.generates and m.direction == "ul"
                                                               for m in (self.traffic or ())):
            out.append(("ho_rlc='flush' with traffic models", "the flush that keeps the step's later arrivals is not "
                                                              "built"))
        # the reference adds same-slot UL interference only with thermal noise and ul_interference on
        # (nr_engine.py:220, 229); the kernels' multi-cell instances always add it
        if self.n_cells > 1 and not (self.noise_model == "thermal" and self.ul_interference):
            out.append((f"n_cells={self.n_cells} with noise_model={self.noise_model!r}, "
                        f"ul_interference={self.ul_interference!r}",
                        "several cells without same-slot UL interference are not built (use noise_model='thermal')"))
        if self.dl and self.cqi_table != "mcs":
            out.append((f"cqi_table={self.cqi_table!r}", "only the MCS-grid CQI report is built"))
        if self.channel not in ("log_distance", "tr38901", "radio_map"):
            out.append((f"channel={self.channel!r}", "channels built: log_distance, tr38901, radio_map"))
        if self.channel == "tr38901" and self.tr38901_los == "stochastic":
            out.append(("tr38901_los='stochastic'", "the spatially consistent LOS state is not built"))
        if self.channel == "tr38901" and self.tr38901_scenario not in ("UMi", "UMa"):
            out.append((f"tr38901_scenario={self.tr38901_scenario!r}", "tr38901 scenarios built: UMi, UMa"))
        if self.blockage and self.blockage_model != "stochastic":
            out.append((f"blockage_model={self.blockage_model!r}", "only blockage model A ('stochastic') is built"))
        if self.los_source != "stochastic":
            out.append((f"los_source={self.los_source!r}", "geometric LOS sources are not built"))
        if self.shadow_modes > 32:
            out.append((f"shadow_modes={self.shadow_modes}", "at most 32 plane waves per shadowing field"))
        if self.ul_power not in ("allocated", "whole_band"):
            out.append((f"ul_power={self.ul_power!r}", "UL power built: allocated, whole_band"))
        if self.ul_power == "whole_band" and self.ul_amc_alloc == "previous" and self.pf_update != "rbg":
            out.append(("ul_power='whole_band' with ul_amc_alloc='previous'", "the MCS choice over the whole band is "
                        "built with pf_update='rbg' (the 5G-LENA switch set)"))
        if self.frame_buffer > 128:
            out.append((f"frame_buffer={self.frame_buffer}", "at most 128 frames per robot"))
        if self.n_harq > 32:
            out.append((f"n_harq={self.n_harq}", "at most 32 HARQ processes"))
        if self.n_subbands > 32:
            out.append((f"{self.n_subbands} RBGs", "at most 32 RBGs"))
        return out


__all__ = ["NRConfig", "NRB_FR1", "rbg_size_38214"]
