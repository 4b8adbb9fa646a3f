"""Generate the golden fixtures of the NR uplink engine from the reference implementation (isaac-net v0.2.0).

Run in a container where the reference is importable (its source tree on PYTHONPATH or given with --ref):

    python tests/golden/make_golden.py --ref /path/to/isaac-net

For each benchmark workload (isaac-net_b200/presets.py) at a small E x R, the reference engine
(make_engine("L2", E, R, "cpu", cfg, backend="reference")) is driven with this repository's seeded pose generator for
a number of control steps, with two partial resets on the way.  The fixture keeps, per step: the poses, the traffic
arrivals the reference generated (captured at TrafficGen.step), the reset schedule, every key of the step dict, and
the engine state after the step (MAC, queue, fading, RNG counters, radio fields, engine clocks) under the reference's
attribute names.  The fixtures are what the oracle (oracle/nr_oracle.py) and the host-side traffic generator are
pinned against; tests read them with numpy only.
"""
from __future__ import annotations

import argparse
import importlib
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# name: (workload id, E, R, steps, resets {step: env ids}, state snapshot every k steps, config overrides
#        [, speed factor of the pose generator]).
# The "s" cases stress the retransmission paths: a weak link (HARQ failures, exhaustion and RLC resends), short
# deadlines (purged frames) and a small frame buffer (refused messages).
CASES = {
    "1": (1, 6, 16, 40, {12: [1], 30: [0, 4]}, 1, {}),
    "2": (2, 3, 32, 32, {15: [2]}, 2, {}),
    "4": (4, 2, 128, 16, {10: [1]}, 4, {}),
    "1s": (1, 4, 16, 40, {20: [2]}, 1, dict(ue_tx_dbm=-12.0, timeout_steps=5, frame_buffer=8, max_harq_tx=2,
                                            rlc_retx_slots=7)),
    "2s": (2, 3, 32, 32, {11: [0]}, 2, dict(ue_tx_dbm=-8.0, n_harq=4, timeout_steps=6, frame_buffer=6)),
    # several cells (config 3: 3 hex cells, log-distance shadowing, A3 handover, UL power control and inter-cell
    # interference); "3s" makes handovers frequent (short TTT, low hysteresis and interruption) on weak links
    "3": (3, 3, 64, 24, {10: [1]}, 2, {}),
    "3s": (3, 3, 64, 24, {9: [2]}, 1, dict(a3_ttt_ms=2.0, a3_hyst_db=0.5, ho_interruption_ms=1.5, ue_tx_dbm=-6.0,
                                            n_harq=4, max_harq_tx=3, frame_buffer=10, timeout_steps=8), 2000.0),
    # a TTT of several control steps: A3 candidates carried across steps and fired inside a later one
    "3t": (3, 2, 64, 24, {14: [0]}, 1, dict(a3_ttt_ms=47.5, a3_hyst_db=1.0, ho_interruption_ms=6.0), 800.0),
    # config 5: two cells on the baked radio map (isaac-net_b200/data/make_radio_map.py) with TR 38.901 blockage
    # model A; "5s" lowers the UE power so that blockage losses move links across MCS and handover thresholds
    "5": (5, 4, 48, 24, {10: [1]}, 2, {}),
    "5s": (5, 3, 48, 24, {12: [0]}, 1, dict(ue_tx_dbm=-20.0, a3_ttt_ms=10.0, a3_hyst_db=1.0, n_harq=4,
                                            timeout_steps=8), 3.0),
    # blockage model A on the single-cell TR 38.901 UMi channel: the "outdoor" family, gNB above the UE (zenith
    # terms active; a 3 m mast puts most links inside the regions' elevation window)
    "1b": (1, 4, 16, 24, {10: [2]}, 2, dict(blockage=True, blockage_model="stochastic", ue_tx_dbm=-10.0,
                                            gnb_height_m=3.0)),
    # 5G-LENA PF switches: the average moves after every RBG (pf_update="rbg") and idle robots keep theirs
    # (pf_avg_idle="freeze"); with retransmission priority off (released RBGs), and with three cells
    "2r": (2, 3, 32, 24, {9: [1]}, 2, dict(pf_update="rbg", pf_avg_idle="freeze", retx_priority=False,
                                           ue_tx_dbm=-6.0)),
    "3r": (3, 2, 64, 16, {9: [1]}, 2, dict(pf_update="rbg", pf_avg_idle="freeze")),
    # the validated 5G-LENA MAC of ul_v2l (lena_validation_v2 without the BSR pipeline): TDMA retransmissions (one per
    # slot and cell, oldest first, no new data beside it) and the MCS chosen for the previous PUSCH's PRB count, on
    # weak links so that retransmissions compete; with PF on one and three cells, and with round robin
    "2v": (2, 3, 32, 24, {9: [1]}, 2, dict(pf_update="rbg", pf_avg_idle="freeze", ul_retx_sched="tdma",
                                           ul_amc_alloc="previous", ue_tx_dbm=-6.0)),
    "3v": (3, 2, 64, 16, {9: [1]}, 2, dict(pf_update="rbg", pf_avg_idle="freeze", ul_retx_sched="tdma",
                                           ul_amc_alloc="previous", ue_tx_dbm=-4.0)),
    "1v": (1, 4, 16, 24, {10: [2]}, 2, dict(ul_retx_sched="tdma", ul_amc_alloc="previous", ue_tx_dbm=-12.0,
                                            max_harq_tx=3)),
    # the 5G-LENA SR / BSR grant pipeline (ul_grant_model="bsr"): bootstrap grants, quantized reports in flight, the
    # RLC tail residue; on one cell, and on three cells with frequent handovers (the target learns the buffer)
    "2g": (2, 3, 32, 24, {9: [1]}, 2, dict(ul_grant_model="bsr", ue_tx_dbm=-6.0)),
    "3g": (3, 2, 64, 16, {9: [1]}, 1, dict(ul_grant_model="bsr", a3_ttt_ms=2.0, a3_hyst_db=0.5,
                                           ho_interruption_ms=1.5), 2000.0),
    # the UE's power over the whole band (ul_power="whole_band": a fixed PSD, no PHR cap): one cell, and three cells
    # where the power-control backoff competes with the whole-band split
    "2w": (2, 3, 32, 24, {9: [1]}, 2, dict(ul_power="whole_band", ue_tx_dbm=-4.0)),
    "3w": (3, 2, 64, 16, {9: [1]}, 2, dict(ul_power="whole_band")),
    # the reference's ul_v2l case (lena_validation_v2: the 5G-LENA MAC switches with the SR / BSR grant pipeline,
    # fading off, the whole-band PSD with its MCS chosen over the whole band for the previous PUSCH's PRBs, a 7 dB
    # noise figure and 128-frame buffers) on config 2's cell
    # the largest per-robot sizes (32 HARQ processes, 128 frame slots) on ragged robot counts: 5 robots in a 16-lane
    # group (11 idle lanes), and one env of 100 robots in a 128-lane block
    "1m": (1, 2, 5, 20, {8: [1]}, 1, dict(n_harq=32, frame_buffer=128, max_harq_tx=6, ue_tx_dbm=-8.0)),
    "2m": (2, 1, 100, 12, {6: [0]}, 2, dict(n_harq=32, frame_buffer=128)),
    # three cells on a weak uplink with long timeouts: the queues fill all 128 frame slots (refused messages, the
    # compaction over the second word of the frame masks)
    "3m": (3, 1, 20, 32, {20: [0]}, 2, dict(n_harq=32, frame_buffer=128, timeout_steps=400, ue_tx_dbm=-24.0)),
    # three cells with the reference's default fixed noise: no same-slot interference (it needs thermal noise), the
    # gNBs' N+I stays the fixed noise (oracle only: the kernels always add the UL interference and refuse this)
    "3f": (3, 2, 64, 16, {9: [1]}, 2, dict(noise_model="fixed")),
    # ho_rlc="flush" with frequent handovers: the queue is flushed at a handover, but messages of the step's traffic
    # that arrive in a later slot are not queued yet and survive it (NREngine's handover wrapper, engine.py:486-497)
    "3h": (3, 2, 64, 16, {9: [1]}, 1, dict(ho_rlc="flush", a3_ttt_ms=2.0, a3_hyst_db=0.5, ho_interruption_ms=1.5),
           2000.0),
    # the rest of the reference's lena_like base (config.py:1685-1701; oracle only, the kernels refuse these): the PF
    # rate from one wideband EESM MCS per robot (pf_metric="wideband"), PDCP discard of arriving frames behind a
    # stale head of line (discard="pdcp_arrival", no purge) and a per-packet overhead on the air
    # (pkt_overhead_bytes per started pkt_payload_bytes); one cell and three cells
    "2L": (2, 3, 32, 24, {9: [1]}, 2, dict(pf_metric="wideband", discard="pdcp_arrival", pkt_overhead_bytes=50,
                                           timeout_steps=4, ue_tx_dbm=-8.0)),
    "3L": (3, 2, 64, 16, {9: [1]}, 2, dict(pf_metric="wideband", discard="pdcp_arrival", pkt_overhead_bytes=50,
                                           pkt_payload_bytes=600, timeout_steps=3)),
    # the reference's ul_v2l benchmark config (lena_validation_v2) with the shipped tables in place of the 5G-LENA
    # extraction (bler_source="pdsch", tbs_mode="38214", harq_combining="cc"), on config 2's traffic
    "2V": (2, 3, 32, 24, {9: [1]}, 2, dict(tdd_pattern="DDDSU", bandwidth_mhz=20, n_prb=50, rbg_size=10,
                                           ul_data_symbols=13, dmrs_re_per_prb=0, n_harq=16, max_harq_tx=4,
                                           harq_fail="drop", discard="pdcp_arrival", olla=False,
                                           pf_metric="wideband", pf_update="rbg", pf_avg_idle="freeze",
                                           ul_retx_sched="tdma", ul_amc_alloc="previous", ul_grant_model="bsr",
                                           ul_power="whole_band", phr_cap=False, fading=False,
                                           noise_model="thermal", gnb_nf_db=6.99697, tb_overhead_bytes=8,
                                           pkt_overhead_bytes=50, frame_buffer=128)),
    "2x": (2, 3, 32, 24, {9: [1]}, 2, dict(pf_update="rbg", pf_avg_idle="freeze", ul_retx_sched="tdma",
                                           ul_amc_alloc="previous", ul_grant_model="bsr", tb_overhead_bytes=8,
                                           fading=False, ul_power="whole_band", gnb_nf_db=6.99697,
                                           frame_buffer=128, ue_tx_dbm=-6.0)),
}


def _ref_traffic(ref_tm, m):
    kw = dict(size_bytes=m.size_bytes, period_ms=m.period_ms, jitter_ms=m.jitter_ms, phase=m.phase,
              rate_hz=m.rate_hz, burst_size=m.burst_size, on_off=m.on_off, gop=m.gop, trigger=m.trigger, det=m.det,
              robots=m.robots, tag=m.tag, priority=m.priority, deadline_ms=m.deadline_ms,
              max_msgs_per_step=m.max_msgs_per_step, direction=m.direction)
    return ref_tm(m.kind, **kw)


def ref_config(wl, **over):
    from isaac_net.core.config import NRConfig as RefCfg
    from isaac_net.core.traffic import TrafficModel as RefTM
    f = {**wl.fields, **over}
    if f.get("traffic") is not None:
        f["traffic"] = tuple(_ref_traffic(RefTM, m) for m in f["traffic"])
    return RefCfg(**f)


def ref_state(eng):
    """Engine state under the reference's names (numpy)."""
    net, ul = eng.net, eng.net.ul
    q = ul.q
    st = {}
    for n in ("sent", "floor", "olla", "avg", "bsr", "sr_t", "last_tx", "csi", "h_state", "h_lo", "h_hi", "h_ready",
              "h_ntx", "h_mcs", "h_tbs", "h_nsb", "h_comb"):
        st["ul." + n] = getattr(ul, n)
    for n in ("cap", "start", "end", "lost", "fin", "enq", "cls", "det", "hid"):
        st["q." + n] = getattr(q, n)
    for n in ("off", "tag", "prio", "dline"):
        if hasattr(q, n):
            st["q." + n] = getattr(q, n)
    if hasattr(ul, "last_nprb"):
        st["ul.last_nprb"] = ul.last_nprb
    if hasattr(ul, "rep_v"):                # BSR_STATE (mac_ul.py:45-50)
        for n in ("est", "boot", "rep_v", "rep_g", "hid", "hid_until", "enq_seen", "armed"):
            st["ul." + n] = getattr(ul, n)
    st["net.h"] = net.h
    if net.rician:
        st["net.spec"] = net.spec
        st["net.k_lin"] = net.k_lin
    st["net.last_g"] = torch.tensor(-1 if net.last_g is None else net.last_g)
    st["rng.episode"] = net.rng.episode
    st["rng.ctr_step"] = net.rng.ctr[2]
    st["eng.T"] = torch.tensor(eng.T)
    st["eng.epoch"] = eng.epoch
    st["eng.last_snr"] = eng._last_snr
    st["eng.last_hid"] = eng._last_hid
    rad = eng.radio
    if rad is not None:
        if rad.k is not None:
            st["radio.k"], st["radio.phi"] = rad.k, rad.phi
        ch = rad.ch
        blk = getattr(rad, "blk_a", None)
        if blk is not None:
            st["radio.blk.k"], st["radio.blk.phi"] = blk.field.k, blk.field.phi
            for n in ("xk", "yk", "vel", "t"):
                st["radio.blk." + n] = getattr(blk, n)
        if ch is not None and hasattr(ch, "sf_los"):
            for nm in ("sf_los", "sf_nlos", "los_field"):
                fld = getattr(ch, nm)
                st[f"radio.{nm}.k"], st[f"radio.{nm}.phi"] = fld.k, fld.phi
    if net.dl is not None:     # the downlink MacLink and its queue
        dl, dq = net.dl, net.dl.q
        for n in ("sent", "floor", "olla", "avg", "bsr", "sr_t", "last_tx", "csi", "h_state", "h_lo", "h_hi",
                  "h_ready", "h_ntx", "h_mcs", "h_tbs", "h_nsb", "h_comb"):
            st["dl." + n] = getattr(dl, n)
        for n in ("cap", "start", "end", "lost", "fin", "enq", "cls", "off", "tag", "prio", "dline"):
            if hasattr(dq, n):
                st["dq." + n] = getattr(dq, n)
        for k, v in dl.ctr.items():
            st["dctr." + k] = v
    if net.C > 1:
        for n in ("serv", "pending", "a3_cand", "a3_cnt", "ho_end", "n_ho"):
            st["assoc." + n] = getattr(net.assoc, n)
        st["net.ni_ul"] = net.ni_ul
        st["net.pg"] = net._pg
        if net.dl is not None:
            st["net.ni_dl"] = net.ni_dl
    for k, v in ul.ctr.items():
        st["ctr." + k] = v
    st["ctr.ntx_hist"], st["ctr.rv_tx"], st["ctr.rv_fail"] = ul.ntx_hist, ul.rv_tx, ul.rv_fail
    st["ctr.prb_used_env"] = ul.prb_used_env
    return {k: v.detach().cpu().clone().numpy() for k, v in st.items()}


# Downlink cases (dl=True): a TDD pattern with D, S and U slots, DL traffic models (direction="dl") beside the
# uplink's, CQI reports, DL HARQ with the HARQ-ACK timing; the fixture adds the DL arrivals of each step.  The "d3"
# cases run config 3's three cells: the DL reference from each robot's own N+I estimate, the DL inter-cell
# interference, DL handovers (oracle only: the kernels refuse the downlink with several cells).
def dl_traffic(i, R):
    """The DL traffic models of the DL cases next to workload i's uplink models."""
    TM = importlib.import_module("isaac-net_b200.traffic").TrafficModel
    ul = importlib.import_module("isaac-net_b200.presets").workload(i).fields["traffic"]
    half = R // 2
    return tuple(ul) + (TM.bursty(3000, rate_hz=120, burst_size=1, on_off=(1.0, 0.0), direction="dl",
                                  deadline_ms=25.0),
                        TM.periodic(400, period_ms=5.0, jitter_ms=1.0, direction="dl", tag=9).on(range(0, half)))


DL_CASES = {
    "d1": (1, 4, 16, 24, {11: [1]}, 1, dict(tdd_pattern="DDDSU", dl=True)),
    "d2": (2, 3, 32, 20, {9: [2]}, 2, dict(tdd_pattern="DDSUU", dl=True)),
    # weak links both ways: DL HARQ failures and exhaustion, purged and refused DL frames; the PF switches
    "d2s": (2, 3, 32, 20, {9: [0]}, 1, dict(tdd_pattern="DDDSU", dl=True, ue_tx_dbm=-8.0, gnb_tx_dbm=12.0,
                                             timeout_steps=6, frame_buffer=8, max_harq_tx=2, pf_update="rbg")),
    "d3": (3, 2, 64, 20, {9: [1]}, 2, dict(tdd_pattern="DDDSU", dl=True)),
    # frequent handovers on weak links both ways, the N+I estimates as EWMAs (li_alpha < 1)
    "d3s": (3, 2, 64, 20, {9: [0]}, 2, dict(tdd_pattern="DDSUU", dl=True, a3_ttt_ms=2.0, a3_hyst_db=0.5,
                                             ho_interruption_ms=1.5, ue_tx_dbm=-6.0, gnb_tx_dbm=14.0, li_alpha=0.5,
                                             n_harq=4, max_harq_tx=3, frame_buffer=10, timeout_steps=8), 2000.0),
    # the lena_like switches on the downlink (one cell; oracle only): DL PDCP discard, overhead, wideband PF
    "d2L": (2, 3, 32, 20, {9: [2]}, 2, dict(tdd_pattern="DDDSU", dl=True, pf_metric="wideband", discard="pdcp_arrival",
                                             pkt_overhead_bytes=50, timeout_steps=4, gnb_tx_dbm=14.0,
                                             ue_tx_dbm=-8.0)),
    # fixed noise: neither link adds interference, the DL reference still comes from the (constant) N+I estimate
    "d3n": (3, 2, 64, 16, {9: [1]}, 2, dict(tdd_pattern="DDDSU", dl=True, noise_model="fixed")),
}


def run_case(i, E, R, steps, resets, every, over, speed=1.0):
    from isaac_net import make_engine as ref_make
    b200 = importlib.import_module("isaac-net_b200")
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(i)
    cfg = ref_config(wl, **over)
    eng = ref_make("L2", E, R, "cpu", cfg, strict=None, seed=wl.seed)
    cap = []
    tstep = eng.traffic.step

    def grab(clock=None, triggers=None):
        a = tstep(clock, triggers)
        cap.append(a)
        return a
    eng.traffic.step = grab
    cap_dl = []
    if eng.traffic_dl is not None:
        tstep_dl = eng.traffic_dl.step

        def grab_dl(clock=None, triggers=None):
            a = tstep_dl(clock, triggers)
            cap_dl.append(a)
            return a
        eng.traffic_dl.step = grab_dl
    mot = presets.Motion(i, E, R, seed=wl.seed, step_ms=cfg.control_step_ms)
    mot.speed = mot.speed * speed
    rec = {"E": np.int64(E), "R": np.int64(R), "steps": np.int64(steps), "workload": np.int64(i)}
    st0 = ref_state(eng)
    for k, v in st0.items():
        rec["init/" + k] = v
    pos = mot.current()
    reset_rows = np.full((steps, E), False)
    for s in range(steps):
        if s in resets:
            ids = resets[s]
            reset_rows[s, ids] = True
            eng.reset(torch.tensor(ids))
        out = eng.step(None, pos)
        a = cap[-1]
        rec[f"s{s}/pos"] = pos.numpy()
        for n in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det"):
            rec[f"s{s}/arr.{n}"] = getattr(a, n).numpy()
        if cap_dl:
            for n in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det"):
                rec[f"s{s}/dlarr.{n}"] = getattr(cap_dl[-1], n).numpy()
        for k, v in out.items():
            rec[f"s{s}/out.{k}"] = v.detach().cpu().clone().numpy()
        if s % every == 0 or s == steps - 1 or (s + 1) in resets:
            for k, v in ref_state(eng).items():
                rec[f"s{s}/st.{k}"] = v
        pos = mot.advance()
    rec["resets"] = reset_rows
    if cfg.channel == "radio_map":
        mk = importlib.import_module("isaac-net_b200.data.make_radio_map")
        rec["radio_map_sha256"] = np.array(mk.gain_digest(np.load(cfg.radio_map_path)["gain_db"]))
    return rec


# Policy-driven cases (no traffic models): each step the policy submits messages (engine.submit with per-message
# tag / priority / deadline extras) and the step takes an SNR input instead of poses: [E,R] through x, or per RBG
# [E,R,S] through snr_db=; one step (with an [E,R] SNR) uses the legacy form step(t, snr, cur_hid).
# name: (workload id, E, R, steps, resets {step: env ids}, state every k steps, config overrides, legacy step)
POLICY_CASES = {
    "1p": (1, 6, 16, 30, {11: [2]}, 1, dict(traffic=None, msg_sizes=(1500.0, 4000.0), timeout_steps=6), 21),
    # submits under PDCP discard with a per-packet overhead (oracle only)
    "1pL": (1, 6, 16, 30, {11: [2]}, 2, dict(traffic=None, msg_sizes=(1500.0, 4000.0), timeout_steps=3,
                                             discard="pdcp_arrival", pkt_overhead_bytes=40, pkt_payload_bytes=1000,
                                             ue_tx_dbm=-10.0), 21),
}


def policy_inputs(E, R, S, steps, seed=17):
    """The seeded policy and SNR inputs of a policy case (one dict per step, CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for s in range(steps):
        send = torch.where(torch.rand(E, R, generator=g) < 0.35, torch.randint(1, 3, (E, R), generator=g),
                           torch.zeros(E, R, dtype=torch.long))
        det = torch.rand(E, R, generator=g) < 0.3
        hid = torch.randint(0, 5, (E,), generator=g)
        tag = torch.randint(1, 5, (E, R), generator=g)
        prio = torch.randint(0, 3, (E, R), generator=g)
        dl = torch.where(torch.rand(E, R, generator=g) < 0.5, torch.full((E, R), math.inf),
                         torch.where(torch.rand(E, R, generator=g) < 0.5, 15.0, 40.0)).double()
        if s % 3 == 2:
            snr = torch.randn(E, R, S, generator=g) * 6.0 + 8.0
        else:
            snr = torch.randn(E, R, generator=g) * 8.0 + 10.0
        out.append({"send": send, "det": det, "hid": hid, "tag": tag, "prio": prio, "dline": dl, "snr": snr,
                    "cur_hid": torch.randint(0, 5, (E,), generator=g)})
    return out


def run_policy_case(i, E, R, steps, resets, every, over, legacy_step):
    from isaac_net import make_engine as ref_make
    from isaac_net.core.proto.netsim import Requests as RefReq
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(i)
    cfg = ref_config(wl, **over)
    eng = ref_make("L2", E, R, "cpu", cfg, strict=None, seed=wl.seed)
    rec = {"E": np.int64(E), "R": np.int64(R), "steps": np.int64(steps), "workload": np.int64(i),
           "policy": np.int64(1), "legacy_step": np.int64(legacy_step)}
    for k, v in ref_state(eng).items():
        rec["init/" + k] = v
    reset_rows = np.full((steps, E), False)
    for s, inp in enumerate(policy_inputs(E, R, cfg.n_subbands, steps)):
        if s in resets:
            reset_rows[s, resets[s]] = True
            eng.reset(torch.tensor(resets[s]))
        acc = eng.submit(None, RefReq(inp["send"], inp["det"], inp["hid"]), tag=inp["tag"], priority=inp["prio"],
                         deadline_ms=inp["dline"])
        rec[f"s{s}/accepted"] = acc.numpy()
        for k, v in inp.items():
            rec[f"s{s}/in.{k}"] = v.numpy()
        if s == legacy_step:
            newest, det_env = eng.step(None, inp["snr"], inp["cur_hid"])
            out = {"newest": newest, "det_env": det_env}
        elif inp["snr"].dim() == 3:
            out = eng.step(None, None, snr_db=inp["snr"])
        else:
            out = eng.step(None, inp["snr"])
        for k, v in out.items():
            rec[f"s{s}/out.{k}"] = v.detach().cpu().clone().numpy()
        if s % every == 0 or s == steps - 1 or (s + 1) in resets:
            for k, v in ref_state(eng).items():
                rec[f"s{s}/st.{k}"] = v
    rec["resets"] = reset_rows
    return rec


# Checkpoint cases: the reference's own engine.state_dict() (isaac_net/core/checkpoint.py, the flat dict of its object
# graph) after `warm` control steps, then `n` more steps with their poses, arrivals, the path gains the reference
# computed and its outputs, and the counters at the end.  The B200 engine loads the checkpoint
# (NRB200Engine.load_reference_checkpoint) and continues from it.
# name: (workload id, E, R, warm steps, steps after the checkpoint, config overrides)
CKPT_CASES = {
    "k2": (2, 3, 32, 9, 3, dict(ue_tx_dbm=-8.0)),
    "k3": (3, 2, 64, 7, 3, {}),
    "k5": (5, 2, 48, 6, 3, {}),
}


def run_ckpt_case(i, E, R, warm, n, over):
    from isaac_net import make_engine as ref_make
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(i)
    cfg = ref_config(wl, **over)
    eng = ref_make("L2", E, R, "cpu", cfg, strict=None, seed=wl.seed)
    cap = []
    tstep = eng.traffic.step

    def grab(clock=None, triggers=None):
        a = tstep(clock, triggers)
        cap.append(a)
        return a
    eng.traffic.step = grab
    mot = presets.Motion(i, E, R, seed=wl.seed, step_ms=cfg.control_step_ms)
    for _ in range(warm):
        eng.step(None, mot.advance())
    rec = {"E": np.int64(E), "R": np.int64(R), "steps": np.int64(n), "workload": np.int64(i)}
    for k, v in eng.state_dict().items():
        if torch.is_tensor(v) and v.dtype != torch.uint8:
            rec["ckpt/" + k] = v.detach().cpu().clone().numpy()
        elif isinstance(v, (bool, int, float)) and not isinstance(v, bool):
            rec["ckpt/" + k] = np.array(v)
    for k, v in ref_state(eng).items():
        rec["ckst/" + k] = v
    pgs = []
    rpg = eng.radio.pathgain_db

    def grab_pg(pos, *a, **k):
        pg = rpg(pos, *a, **k)
        pgs.append(pg)
        return pg
    eng.radio.pathgain_db = grab_pg
    for s in range(n):
        pos = mot.advance()
        out = eng.step(None, pos)
        rec[f"s{s}/pos"] = pos.numpy()
        rec[f"s{s}/pg"] = pgs[-1].detach().cpu().numpy()
        for nm in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det"):
            rec[f"s{s}/arr.{nm}"] = getattr(cap[-1], nm).numpy()
        for k, v in out.items():
            rec[f"s{s}/out.{k}"] = v.detach().cpu().clone().numpy()
    for k, v in eng.net.ul.ctr.items():
        rec["end/ctr." + k] = v.detach().cpu().numpy()
    rec["end/ntx_hist"] = eng.net.ul.ntx_hist.cpu().numpy()
    rec["overrides"] = np.array(repr(over))
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ISAAC_NET_REF"),
                    help="source tree of the reference (isaac-net); default $ISAAC_NET_REF, else it must be importable")
    ap.add_argument("--cases", default=",".join([str(k) for k in CASES] + list(POLICY_CASES) + list(CKPT_CASES) +
                                                 list(DL_CASES)))
    a = ap.parse_args()
    if a.ref:
        sys.path.insert(0, a.ref)
    sys.path.insert(0, ROOT)
    torch.set_num_threads(8)
    for c in a.cases.split(","):
        if c in CKPT_CASES:
            rec = run_ckpt_case(*CKPT_CASES[c])
        elif c in DL_CASES:
            i, E, R, steps, resets, every, over, *speed = DL_CASES[c]
            over = dict(over, traffic=dl_traffic(i, R))
            rec = run_case(i, E, R, steps, resets, every, over, *speed)
            rec["overrides"] = np.array(repr(DL_CASES[c][6]))
            rec["dl_traffic"] = np.int64(1)
        elif c in POLICY_CASES:
            rec = run_policy_case(*POLICY_CASES[c])
            rec["overrides"] = np.array(repr(POLICY_CASES[c][6]))
        else:
            rec = run_case(*CASES[c])
            rec["overrides"] = np.array(repr(CASES[c][6]))
        path = os.path.join(HERE, f"cfg{c}.npz")
        np.savez_compressed(path, **rec)
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
