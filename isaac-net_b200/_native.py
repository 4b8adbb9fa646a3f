"""ctypes binding of the C ABI in include/isaac_net_b200.h (libisaac_net_b200.so, built in-tree).

The structures below mirror the C structures field by field; tests/test_abi.py checks their sizes and offsets
against the compiled header.  There is no fallback: if the shared library is missing or was built for another ABI
version, loading raises.
"""
from __future__ import annotations

import ctypes
import os

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libisaac_net_b200_check.so" if os.environ.get("INB_CHECK") == "1"
                        else "libisaac_net_b200.so")
ABI_VERSION = 17
MAX_ROWS = 128
NCTR = 64
BLK_REGIONS = 4        # INB_BLK_REGIONS
CDF_STRIDE = 64        # INB_CDF_STRIDE
CTR_NAMES = ("tb_new", "tb_retx", "tb_ok", "tb_fail", "exhaust", "bytes_ok", "bytes_new", "new_while_pending",
             "prb_used", "lost_frames")
LENA_CTR_NAMES = ("tb_bytes", "tb_empty", "retx_block")   # words 10-12 with InbParams.lena_ctr
CTR_NTX_HIST, CTR_RV_TX, CTR_RV_FAIL = 16, 32, 48

P = ctypes.c_void_p
i32, i64, u32, f32, f64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float, ctypes.c_double

STATE_FIELDS = ("sent", "floor_", "bsr", "sr_t", "last_tx", "enq", "olla", "avg", "csi", "h", "spec", "k_lin",
                "h_state", "h_lo", "h_hi", "h_ready", "h_ntx", "h_mcs", "h_tbs", "h_nsb", "h_comb", "cap", "start",
                "end_", "cls", "hid", "tag", "prio", "lost", "det", "fin", "off", "dline", "serv", "a3_cand", "a3_cnt",
                "ho_end", "n_ho", "pending", "ni_ul", "last_nprb", "bsr_est", "bsr_rep_v", "bsr_rep_g", "bsr_hid",
                "bsr_hid_until", "bsr_enq_seen", "bsr_boot", "bsr_armed")
BSR_DEPTH = 4          # INB_BSR_DEPTH
OUT_FIELDS = ("delivered", "timed_out", "dropped", "deadline_miss", "cap", "cls", "arrival_slot", "tag", "priority",
              "bytes", "delay", "arrival", "newest", "queue_len", "gen_accepted", "gen_bytes", "queue_bytes",
              "sinr_db", "pathgain", "det_env", "serving_cell", "blocked", "los", "lost_any", "generated")
ARR_FIELDS = ("valid", "det", "nbytes", "slot", "tag", "prio", "dline")
TAB_FIELDS = ("bler", "thr_ref", "se", "beta", "rate", "w", "lw", "lw10", "la_tbs", "la_i0", "la_wi", "la_ncb", "fk",
              "fphi", "gnb")


class InbState(ctypes.Structure):
    _fields_ = [(n, P) for n in STATE_FIELDS]


class InbOutputs(ctypes.Structure):
    _fields_ = [(n, P) for n in OUT_FIELDS]


class InbArrivals(ctypes.Structure):
    _fields_ = [(n, P) for n in ARR_FIELDS]


class InbTables(ctypes.Structure):
    _fields_ = [(n, P) for n in TAB_FIELDS]


class InbParams(ctypes.Structure):
    _fields_ = ([(n, i32) for n in ("E", "R", "S", "P", "F", "M", "MCS", "mcs_max", "C_axis", "G_axis", "nprb", "N",
                                    "K_rows", "Kf")]
                + [("T", i64), ("rows", (i32 * 4) * MAX_ROWS), ("rowf", (f32 * 2) * MAX_ROWS), ("sched", i32),
                   ("thr_mono", i32)]
                + [(n, i32) for n in ("olla_on", "phr_cap", "retx_priority", "comb_cc", "harq_drop", "purge",
                                      "fading", "rician", "radio")]
                + [(n, i32) for n in ("sr_delay", "ul_rtt", "rlc_retx", "max_tx", "tb_oh", "timeout")]
                + [(n, i32) for n in ("dmrs", "oh", "ref_prbs")]
                + [("s0", u32), ("inv_sqrt2", f32)]
                + [(n, f32) for n in ("ul_ref0", "noise_prb", "ue_tx", "sub_noise")]
                + [(n, f32) for n in ("phr_min", "olla_up", "olla_dn", "pf_a", "pf_b", "target", "inv_S")]
                + [(n, f32) for n in ("s0_snr", "inv_ds", "c0_cbs", "inv_dc")]
                + [("proc_off", f64), ("ctl_ms", f64), ("inv_N_d", f64), ("inv_ref_prbs", f32), ("radio_model", i32)]
                + [(n, f32) for n in ("h_bs", "h_ut", "dbp", "fc_term", "pl_a", "pl_n1", "pl_b_term", "sigma_sf",
                                      "amp", "hh2")]
                + [(n, f32) for n in ("pl_const", "pl_10n")]
                + [(n, i32) for n in ("C", "ttt", "ho_int", "has_floor", "ho_flush", "pc_on")]
                + [(n, f32) for n in ("a3_off", "a3_hyst", "floor_rx", "noise_mw", "ue_tx_ref", "ref_db", "pc_p0",
                                      "pc_alpha", "li_alpha", "li_beta")]
                + [("los_const", i32), ("pf_rbg", i32), ("pf_freeze", i32), ("field_fma", i32), ("tdma", i32),
                   ("amc_prev", i32), ("lena_ctr", i32)]
                + [(n, i32) for n in ("bsr_on", "sr_boot_slots", "sr_boot_bytes", "bsr_delay", "rlc_tail_slots",
                                      "bsr_hdr", "bsr_est_hdr", "rlc_tail_bytes")]
                + [(n, i32) for n in ("dl_on", "n_ul_rows", "n_dl_rows")] + [("rows_dl", (i32 * 4) * MAX_ROWS)]
                + [("la_sets", i32), ("dl_nsym_tab", i32 * 16), ("whole_band", i32), ("wb_db", f32)])


class InbRadio(ctypes.Structure):
    _fields_ = ([(n, i32) for n in ("on", "map_on", "H", "W")]
                + [(n, f32) for n in ("x0", "y0", "sx", "sy", "wm1", "hm1", "wm2", "hm2")]
                + [("map", P)]
                + [(n, i32) for n in ("blockage", "Kb", "n_table")]
                + [(n, f32) for n in ("amp_b", "ck", "max_db", "h_ut", "h_bs", "dt", "u_den")]
                + [("fma_b", i32)]
                + [(n, P) for n in ("bk", "bphi", "xk", "yk", "vel", "t", "table", "pg", "blk")])


class InbStepArgs(ctypes.Structure):
    _fields_ = [("p", InbParams), ("s", InbState), ("o", InbOutputs), ("a", InbArrivals), ("t", InbTables),
                ("pos", P), ("pathgain_in", P), ("ul_ref_in", P), ("env_id", P), ("episode", P), ("rng_ctr", P),
                ("epoch", P), ("last_hid", P), ("ctr", P), ("status", P), ("T_dev", P),
                ("trace", P), ("gain", P), ("gain_cap", i64), ("o_base", P), ("rm", InbRadio), ("det_hid", P), ("phases", i32),
                ("dl", P)]


class InbResetArgs(ctypes.Structure):
    _fields_ = ([(n, i32) for n in ("E", "R", "S", "P", "F")] + [("s0", u32), ("rician", i32)]
                + [(n, f32) for n in ("k_lin0", "inv_sqrt2", "two_pi")]
                + [(n, P) for n in ("mask", "env_id", "episode", "rng_ctr")] + [("s", InbState)]
                + [("C", i32), ("noise_mw", f32)])


MAX_SRC = 8
u64 = ctypes.c_uint64


class InbTrafficSource(ctypes.Structure):
    _fields_ = ([(n, i32) for n in ("kind", "width", "col", "nb", "loops", "burst", "gop_n", "det")]
                + [("tag", i64), ("prio", i64)]
                + [(n, f64) for n in ("dline", "size", "gop_i", "gop_p", "period", "jitter", "on_ms", "off_ms", "iat")]
                + [(n, P) for n in ("mask", "nom", "nxt", "cnt", "on", "t_tog", "t_bur", "deferred")])


TRAFFIC_OUT = ("valid", "det", "nbytes", "slot", "tag", "prio", "dline")


class InbTrafficArgs(ctypes.Structure):
    _fields_ = ([(n, i32) for n in ("E", "R", "M", "N", "n_src")] + [("seed", u64), ("off0", u64)]
                + [(n, i64) for n in ("stride", "inc", "ndraws")] + [("step_ms", f64), ("inv_slot_ms", f64)]
                + [("calls", P), ("src", InbTrafficSource * MAX_SRC)] + [(n, P) for n in TRAFFIC_OUT]
                + [("counter", i32), ("s0", u32), ("env_id", P), ("episode", P)])


OBS_OFFS = ("off_mask", "off_delay", "off_aoi", "off_qlen", "off_qbytes", "off_sinr", "off_rsrp", "off_serv",
            "off_last", "off_hist", "off_blocked", "off_los")   # in the order of isaac/config.py OBS_FEATURES
OBS_IN = ("newest", "t", "queue_len", "serving", "queue_bytes", "sinr_db", "delay", "delivered", "blocked", "los",
          "det_env", "cap", "cur_tag")
OBS_OUT = ("last_cap", "hist", "last_cap_out", "aoi_s", "delay_s", "rsrp_dbm", "x", "delivered_any", "blocked_out",
           "los_out", "tag_delivered")


class InbObsArgs(ctypes.Structure):
    _fields_ = ([(n, i32) for n in ("E", "R", "F", "G", "K", "dim")] + [(n, i32) for n in OBS_OFFS]
                + [(n, f32) for n in ("step_dt", "inv_ts", "inv_F", "inv_qbytes", "inv_db", "noise_db")]
                + [(n, P) for n in OBS_IN + OBS_OUT])


EXPORTS = ("inb_nr_step", "inb_nr_step_after", "inb_nr_step_noalloc", "inb_nr_reset", "inb_rng_draw", "inb_traffic_step",
           "inb_store2", "inb_net_obs", "inb_abi_version")
NOALLOC_GAIN_MAX = 1 << 25
_lib = None


def lib():
    """The loaded shared library (raises if it is missing: build it with __graft_entry__.build())."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: the B200 engine has no fallback path. Build the CUDA library with "
                           "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a).")
    L = ctypes.CDLL(LIB_PATH)
    L.inb_abi_version.restype = ctypes.c_int
    L.inb_abi_version.argtypes = []
    if L.inb_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH} has ABI {L.inb_abi_version()}, expected {ABI_VERSION}: rebuild it")
    L.inb_nr_step.restype = ctypes.c_int
    L.inb_nr_step.argtypes = [ctypes.POINTER(InbStepArgs), P]
    L.inb_nr_step_after.restype = ctypes.c_int
    L.inb_nr_step_after.argtypes = [ctypes.POINTER(InbStepArgs), P, P]
    L.inb_nr_step_noalloc.restype = ctypes.c_int
    L.inb_nr_step_noalloc.argtypes = [ctypes.POINTER(InbStepArgs), P]
    L.inb_nr_reset.restype = ctypes.c_int
    L.inb_nr_reset.argtypes = [ctypes.POINTER(InbResetArgs), P]
    L.inb_rng_draw.restype = ctypes.c_int
    L.inb_rng_draw.argtypes = [i32, i32, u32, u32, u32, P, P, P, i32, P, P]
    L.inb_store2.restype = ctypes.c_int
    L.inb_store2.argtypes = [P, i64, i64, P]
    L.inb_traffic_step.restype = ctypes.c_int
    L.inb_traffic_step.argtypes = [ctypes.POINTER(InbTrafficArgs), P]
    L.inb_net_obs.restype = ctypes.c_int
    L.inb_net_obs.argtypes = [ctypes.POINTER(InbObsArgs), P]
    _lib = L
    return L


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed with status {rc}")


__all__ = ["lib", "check", "InbStepArgs", "InbResetArgs", "InbParams", "InbState", "InbOutputs", "InbArrivals",
           "InbTables", "InbRadio", "InbTrafficArgs", "InbTrafficSource", "InbObsArgs", "EXPORTS", "LIB_PATH"]
