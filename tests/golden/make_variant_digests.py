"""Digests of the reference's step outputs for single-setting variants of the benchmark workloads: the reference
engine (make_engine("L2", E, R, "cpu", cfg)) is stepped with this repository's seeded poses (presets.Motion) and its
own traffic models, one partial reset on the way, and every step's output dict is reduced to a SHA-256 digest.

    python tests/golden/make_variant_digests.py --ref /path/to/isaac-net    # writes tests/golden/variant_digests.json

tests/test_variant_digests.py steps the oracle (aten mode) on the same inputs (the host traffic generator reproduces
the reference's arrivals bitwise) and requires the same digests: a broad, small pin of the oracle over settings the
full fixtures do not hold.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

E, STEPS, RESETS = 2, 8, {5: [1]}
# (workload, config overrides)
VARIANTS = [
    (1, dict(olla=False)), (1, dict(bler_target=0.01)), (1, dict(harq_combining="none")), (1, dict(harq_fail="drop")),
    (1, dict(max_harq_tx=2, ue_tx_dbm=-10.0)), (1, dict(n_harq=2)),
    (1, dict(rlc_retx_slots=3, ue_tx_dbm=-12.0, max_harq_tx=2)), (1, dict(k2=4)), (1, dict(gnb_proc_slots=3)),
    (1, dict(sr_period_slots=1)), (1, dict(sr_grant_delay_slots=7)), (1, dict(ul_harq_rtt_slots=5, ue_tx_dbm=-10.0)),
    (1, dict(phr_cap=False, ue_tx_dbm=-5.0)), (1, dict(phr_min_db=10.0, ue_tx_dbm=-5.0)), (2, dict(pf_window=10.0)),
    (2, dict(retx_priority=False, ue_tx_dbm=-6.0)), (2, dict(scheduler="maxci")), (1, dict(timeout_steps=2)),
    (1, dict(frame_buffer=4)), (1, dict(discard="none", timeout_steps=2)), (1, dict(proc_offset_ms=0.7)),
    (1, dict(ul_mcs_max=10)), (2, dict(mcs_table=2)), (1, dict(dmrs_re_per_prb=24)), (1, dict(overhead_re_per_prb=18)),
    (1, dict(ul_data_symbols=13)), (1, dict(tdd_pattern="DDDSU")),
    (1, dict(tdd_pattern="DSUUU", special_split=(6, 4, 4))),
    (1, dict(fading=False)), (1, dict(fading_rho_per_ms=0.5)), (2, dict(rician_k_db=10.0)), (1, dict(gnb_nf_db=9.0)),
    (1, dict(snr_ref_prbs=20)), (1, dict(rbg_size=4)), (1, dict(rbg_config=2)), (2, dict(n_prb=100)),
    (1, dict(tb_overhead_bytes=12)), (1, dict(carrier_ghz=28.0)), (1, dict(ue_height_m=3.0)),
    (1, dict(gnb_height_m=25.0)), (3, dict(a3_offset_db=2.0)), (3, dict(a3_min_target_rsrp_dbm=-95.0)),
    (3, dict(ul_pc=False)), (3, dict(ul_pc_p0_dbm=-80.0, ul_pc_alpha=0.8)), (3, dict(li_alpha=0.3)),
    (3, dict(shadow_sigma_db=2.0)), (3, dict(cell_isd_m=120.0)), (3, dict(ho_interruption_ms=0.0)),
    (3, dict(harq_fail="drop", a3_ttt_ms=2.0, a3_hyst_db=0.5)), (3, dict(scheduler="rr")), (3, dict(scheduler="maxci")),
    (1, dict(shadow_acf="exp", shadow_dcorr_m=20.0)), (1, dict(shadow_modes=4)),
    (1, dict(pathloss_exp=3.0, pl_const_db=35.0)), (1, dict(msg_sizes=(700.0,))), (2, dict(control_step_ms=2.5)),
    (1, dict(mu=0, control_step_ms=10.0)), (1, dict(mu=2, control_step_ms=2.5, bandwidth_mhz=40)),
    (1, dict(ue_nf_db=5.0)), (1, dict(ni_fixed_dbm=-100.0, noise_model="fixed")), (2, dict(fading_rician=False)),
    (5, dict(blockage_max_db=10.0)), (5, dict(scheduler="pf")),
    (1, dict(channel="tr38901", tr38901_scenario="UMa", tr38901_los="los")),
    (2, dict(tdd_pattern="DDSUU", k1=3)), (2, dict(pf_update="rbg", retx_priority=False)),
    (2, dict(ul_grant_model="bsr", sr_boot_slots=3, bsr_delay_slots=4, rlc_tail_bytes=40)),
    # settings the kernels refuse but the oracle restates: lena_like's switches, no same-slot interference, a flush
    # at handover under traffic models
    (1, dict(pf_metric="wideband")), (2, dict(pf_metric="wideband", scheduler="maxci")),
    (2, dict(discard="pdcp_arrival", timeout_steps=2, ue_tx_dbm=-8.0)), (1, dict(pkt_overhead_bytes=60)),
    (3, dict(pf_metric="wideband", discard="pdcp_arrival", timeout_steps=3)), (3, dict(ul_interference=False)),
    (3, dict(ho_rlc="flush", a3_ttt_ms=2.0, a3_hyst_db=0.5)),
    # radio: blockage model A on the other channels and cell layouts, forced-LOS / NLOS TR 38.901, no blockage on the map
    (5, dict(blockage=False)), (5, dict(a3_hyst_db=1.0, a3_ttt_ms=10.0)),
    (1, dict(blockage=True, blockage_model="stochastic")), (3, dict(blockage=True, blockage_model="stochastic")),
    (1, dict(channel="tr38901", tr38901_scenario="UMi", tr38901_los="los", blockage=True,
             blockage_model="stochastic", gnb_height_m=10.0)),
    (3, dict(channel="tr38901", tr38901_scenario="UMa", tr38901_los="los")),
    (1, dict(channel="tr38901", tr38901_scenario="UMi", tr38901_los="nlos")),
]
# the downlink (one cell, DDDSU, make_golden.dl_traffic's DL models beside the uplink's): (workload, overrides)
DL_BASE = dict(tdd_pattern="DDDSU", dl=True)
DL_VARIANTS = [
    (1, dict()), (1, dict(ul=False)), (1, dict(dl_mcs_max=12)), (1, dict(k1=4)), (1, dict(cqi_period_slots=2)),
    (1, dict(cqi_period_slots=40)), (1, dict(gnb_tx_dbm=20.0)), (1, dict(special_dl_data=False)),
    (1, dict(dl_ctrl_symbols=3)), (1, dict(gnb_proc_slots=3)),
    (1, dict(harq_fail="drop", gnb_tx_dbm=10.0, max_harq_tx=2)),
    (1, dict(harq_combining="none", gnb_tx_dbm=12.0)), (1, dict(tdd_pattern="DDSUU")),
    (1, dict(tdd_pattern="DSUUU", special_split=(6, 4, 4))), (1, dict(ue_nf_db=4.0)), (1, dict(scheduler="rr")),
    (1, dict(scheduler="maxci")), (1, dict(olla=False)), (1, dict(timeout_steps=2, gnb_tx_dbm=8.0)),
    (1, dict(frame_buffer=4)), (2, dict(mcs_table=2)), (2, dict(pf_update="rbg", pf_avg_idle="freeze")),
    (1, dict(mu=0, control_step_ms=10.0)), (1, dict(fading=False)), (2, dict(rician_k_db=8.0)),
    (1, dict(proc_offset_ms=0.4)),
    # several cells (oracle only: the kernels refuse the downlink with several cells)
    (3, dict()), (3, dict(dl_interference=False)), (3, dict(li_alpha=0.5, gnb_tx_dbm=30.0)),
    (3, dict(a3_ttt_ms=2.0, a3_hyst_db=0.5, ho_interruption_ms=1.5)), (3, dict(harq_fail="drop", a3_ttt_ms=2.0)),
    # lena_like's switches on both links (oracle only)
    (1, dict(pf_metric="wideband")), (1, dict(discard="pdcp_arrival", timeout_steps=2, gnb_tx_dbm=8.0)),
    (1, dict(pkt_overhead_bytes=60, pkt_payload_bytes=500)),
]


def robots(i):
    """Robots per env of a variant: config 2's traffic names robots up to 31, the others run 16."""
    return 32 if i == 2 else 16


# the per-robot MAC / HARQ / queue state both sides name alike (the reference's attribute names)
STATE_KEYS = tuple("ul." + n for n in ("sent", "floor", "olla", "avg", "bsr", "sr_t", "last_tx", "csi", "h_state",
                                       "h_lo", "h_hi", "h_ready", "h_ntx", "h_mcs", "h_tbs", "h_nsb", "h_comb")) + \
    tuple("q." + n for n in ("cap", "start", "end", "lost", "fin", "enq"))


def digest(out):
    """SHA-256 (first 16 hex digits) of {key: array}: keys in order, shape, NaN mask and the values widened to
    float64 / int64 (exact, so the digest does not depend on the integer or float width a side stores)."""
    h = hashlib.sha256()
    for k in sorted(out):
        v = np.asarray(out[k])
        h.update(f"{k}:{v.shape}".encode())
        if v.dtype.kind == "f":
            nan = np.isnan(v)
            h.update(np.packbits(nan).tobytes())
            v = np.where(nan, 0, v).astype(np.float64)
        else:
            v = v.astype(np.int64)
        h.update(np.ascontiguousarray(v).tobytes())
    return h.hexdigest()[:16]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ISAAC_NET_REF"),
                    help="source tree of the reference (isaac-net); default $ISAAC_NET_REF, else it must be importable")
    a = ap.parse_args()
    if a.ref:
        sys.path.insert(0, a.ref)
    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    import json
    import torch
    from make_golden import dl_traffic, run_case
    torch.set_num_threads(8)
    res = []
    runs = [(i, over, over) for i, over in VARIANTS]
    runs += [(i, dict(DL_BASE, **over), dict(DL_BASE, **over, traffic=dl_traffic(i, robots(i))))
             for i, over in DL_VARIANTS]
    for i, over, run_over in runs:
        rec = run_case(i, E, robots(i), STEPS, RESETS, STEPS, run_over)
        ds, sd = [], {}
        for s in range(STEPS):
            pre = f"s{s}/out."
            ds.append(digest({k[len(pre):]: v for k, v in rec.items() if k.startswith(pre)}))
            if f"s{s}/st.ul.sent" in rec:
                sd[str(s)] = digest({k: rec[f"s{s}/st.{k}"] for k in STATE_KEYS})
        res.append({"workload": i, "over": repr(over), "dl_traffic": "traffic" in run_over, "digests": ds,
                    "state_digests": sd})
        print(i, over, ds[-1], flush=True)
    path = os.path.join(HERE, "variant_digests.json")
    with open(path, "w") as fh:
        json.dump(res, fh, indent=0)
    print(path, os.path.getsize(path), len(res))


if __name__ == "__main__":
    main()
