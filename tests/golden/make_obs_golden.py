"""Generate the golden fixtures of the network-observation packing from the reference (isaac-net v0.2.0).

Run where the reference is importable (its source tree on PYTHONPATH or given with --ref):

    python tests/golden/make_obs_golden.py --ref /path/to/isaac-net

The reference's Isaac-side module (isaac_net.isaac.net_module.NetModule, level "L2", backend "reference", the
engine's own radio: IsaacNetCfg(radio="engine")) is driven on the CPU with this repository's seeded poses, random
per-robot message submissions (TrafficRequest with tags) and a per-env current tag, with partial resets on the way.
Per step the fixture keeps the engine's step dict (what NetModule.step receives from make_engine's engine), the
current tag, NetModule.step's output dict and NetModule.obs() (isaac_net/isaac/obs.py NetObs.update).  The
observation packing is pinned against these by feeding it the recorded engine outputs (tests/test_net_obs.py).
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

ALL_FEATURES = ("msg_delay", "aoi", "delivered_mask", "queue_len", "queue_bytes", "sinr", "rsrp", "serving_cell",
                "last_delivered", "delay_history", "blocked", "los")
# the engine outputs NetModule.step reads (isaac_net/isaac/net_module.py:340-373)
ENG_KEYS = ("newest", "t", "queue_len", "queue_bytes", "sinr_db", "serving_cell", "blocked", "los", "delivered",
            "timed_out", "cap", "cls", "delay", "det_env")
# name: (workload id, E, R, steps, resets {step: env ids}, features, history, time scale (s) or None, config overrides)
CASES = {
    "o1": (1, 4, 16, 30, {12: [1], 22: [0, 3]}, ALL_FEATURES, 4, None, {}),
    # three cells: the one-hot serving cell; a short time scale so that the clamp to 1 engages
    "o3": (3, 2, 64, 16, {9: [1]}, ("serving_cell", "aoi", "rsrp", "sinr", "delay_history", "msg_delay", "los",
                                     "blocked"), 3, 0.2, {}),
    # blockage model A on the single-cell channel: the engine's blocked / LOS outputs
    "o1b": (1, 3, 16, 16, {8: [2]}, ("blocked", "los", "last_delivered", "queue_bytes", "queue_len",
                                      "delivered_mask", "delay_history"), 2, 0.4,
            dict(blockage=True, blockage_model="stochastic", ue_tx_dbm=-10.0, gnb_height_m=3.0)),
}


def run_case(name):
    from isaac_net.isaac.config import IsaacNetCfg
    from isaac_net.isaac.net_module import NetModule, TrafficRequest
    sys.path.insert(0, HERE)
    from make_golden import ref_config
    presets = importlib.import_module("isaac-net_b200.presets")
    wl_i, E, R, steps, resets, feats, hist, ts, over = CASES[name]
    wl = presets.workload(wl_i)
    cfg = ref_config(wl, **over)
    isc = IsaacNetCfg(radio="engine", obs_features=feats, obs_history=hist, obs_time_scale_s=ts)
    net = NetModule("L2", E, R, "cpu", cfg, backend="reference", isaac=isc, seed=wl.seed)
    eng_out = {}
    step0 = net.eng.step

    def rec(*a, **k):
        o = step0(*a, **k)
        eng_out.clear()
        eng_out.update(o)
        return o

    net.eng.step = rec
    mot = presets.Motion(wl_i, E, R, seed=wl.seed + 11, step_ms=cfg.control_step_ms)
    gen = torch.Generator().manual_seed(1234 + wl_i)
    d = {"E": E, "R": R, "steps": steps, "workload": wl_i, "overrides": repr(over), "features": np.array(feats),
         "history": hist, "time_scale": -1.0 if ts is None else ts}
    rs = np.zeros((steps, E), dtype=bool)
    pos = mot.current()
    n_cls = len(cfg.msg_sizes)
    for s in range(steps):
        if s in resets:
            rs[s, resets[s]] = True
            net.reset(resets[s])
        send = torch.where(torch.rand(E, R, generator=gen) < 0.3,
                           torch.randint(1, n_cls + 1, (E, R), generator=gen), torch.zeros(E, R, dtype=torch.long))
        tag = torch.where(torch.rand(E, R, generator=gen) < 0.5, torch.randint(0, 4, (E, R), generator=gen),
                          torch.full((E, R), -1, dtype=torch.long))
        cur = torch.randint(-1, 4, (E,), generator=gen)
        net.submit(None, TrafficRequest(send, tag))
        poses = torch.cat([pos, torch.zeros(E, R, 1)], -1)
        out = net.step(None, poses, cur)
        x = net.obs()
        d[f"s{s}/in.cur_tag"] = cur.numpy()
        for k, v in eng_out.items():
            if torch.is_tensor(v) and k in ENG_KEYS:
                d[f"s{s}/eng.{k}"] = v.detach().cpu().clone().numpy()
        for k, v in out.items():
            d[f"s{s}/net.{k}"] = v.detach().cpu().clone().numpy()
        d[f"s{s}/obs"] = x.detach().cpu().clone().numpy()
        pos = mot.advance()
    d["resets"] = rs
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="source tree of the reference (isaac-net)")
    ap.add_argument("cases", nargs="*", default=sorted(CASES))
    a = ap.parse_args()
    if a.ref:
        sys.path.insert(0, a.ref)
    sys.path.insert(0, ROOT)
    for c in a.cases:
        d = run_case(c)
        path = os.path.join(HERE, f"{c}.npz")
        np.savez_compressed(path, **d)
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
