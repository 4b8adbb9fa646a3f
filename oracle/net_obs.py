"""ORACLE — test infrastructure only.  Never imported by the product path (isaac-net_b200/), only by tests/, as the
checker of the device observation packing.

A restatement, in plain torch ops, of what isaac-net v0.2.0's Isaac-side module does with one engine step dict when
it runs on the engine's own radio (IsaacNetCfg(radio="engine")):
  * NetModule.step's post-processing (isaac_net/isaac/net_module.py:324, 340-374): the freshness state
    last_cap = max(last_cap, newest), aoi_s = (t + 1 - last_cap).float() * step_dt, delay_s = delay * step_dt,
    rsrp_dbm = sinr_db + the config's subband noise, blocked / los from the engine or their defaults, tag_delivered;
  * NetObs.update (isaac_net/isaac/obs.py:48-87): the delay history (the delay of the newest delivered message, the
    first slot of the largest capture step among delivered slots, shifted in when the robot had a delivery) and the
    selected features in order, each normalised as the reference does;
  * the partial reset of both (net_module.py:221-235 fill_rows of last_cap; obs.py:43-46).
On the same device this is bitwise the reference (the same torch ops in the same order): pinned on CPU against the
fixtures tests/golden/o*.npz written by tests/golden/make_obs_golden.py from the reference itself.  Cross-device note:
torch divides a float tensor by a python scalar exactly on CPU but multiplies by the float32 reciprocal on CUDA; the
oracle inherits the device's rule.
"""
from __future__ import annotations

import torch

DB_SCALE = 40.0           # isaac_net/isaac/config.py:60
TIME_SCALE_STEPS = 50     # isaac_net/isaac/config.py:61
FEATURES = ("delivered_mask", "msg_delay", "aoi", "queue_len", "queue_bytes", "sinr", "rsrp", "serving_cell",
            "last_delivered", "delay_history", "blocked", "los")


def widths(features, F, G, K):
    """{feature: width} in order (isaac_net/isaac/config.py:102-106)."""
    w = {"delivered_mask": F, "msg_delay": F, "serving_cell": G, "delay_history": K}
    return {f: w.get(f, 1) for f in features}


class NetObsOracle:
    def __init__(self, features, E, R, F, G, history, time_scale, step_dt, noise_db, q_bytes, device):
        self.features = tuple(features)
        self.dims = widths(self.features, F, G, history)
        self.dim = sum(self.dims.values())
        self.E, self.R, self.F, self.G, self.K = E, R, F, G, history
        self.time_scale, self.step_dt, self.noise, self.q_bytes = float(time_scale), float(step_dt), \
            float(noise_db), float(q_bytes)
        self.dev = torch.device(device)
        self.last_cap = torch.zeros(E, R, dtype=torch.long, device=self.dev)
        self.x = torch.zeros(E, R, self.dim, device=self.dev)
        self.hist = torch.zeros(E, R, history, device=self.dev)

    def reset(self, ids):
        ids = torch.as_tensor(ids, dtype=torch.long, device=self.dev)
        self.last_cap[ids] = 0
        self.x[ids] = 0.0
        self.hist[ids] = 0.0

    def _t(self, s):
        return (s / self.time_scale).clamp(0.0, 1.0)                          # obs.py:40-41

    def step(self, o, cur_tag=None):
        """NetModule.step's output dict (the keys it derives from the engine dict `o`) and the observation."""
        newest = o["newest"]
        self.last_cap = torch.maximum(self.last_cap, newest)                  # net_module.py:348
        blocked = o.get("blocked")
        out = dict(
            delivered=newest >= 0,
            newest_cap=newest,
            last_cap=self.last_cap.clone(),
            aoi_s=(o["t"][:, None] + 1 - self.last_cap).float() * self.step_dt,
            queue_len=o["queue_len"],
            queue_bytes=o["queue_bytes"],
            sinr_db=o["sinr_db"],
            rsrp_dbm=o["sinr_db"] + self.noise,
            serving=o["serving_cell"],
            blocked=blocked if blocked is not None else torch.zeros_like(newest, dtype=torch.bool),
            los=o["los"] if "los" in o else (~blocked if blocked is not None
                                             else torch.ones_like(newest, dtype=torch.bool)),
            msg_delivered=o["delivered"],
            timed_out=o["timed_out"],
            cap=o["cap"],
            cls=o["cls"],
            delay_s=o["delay"] * self.step_dt,
            t=o["t"],
        )                                                                     # net_module.py:349-368
        if cur_tag is not None:
            out["tag_delivered"] = o["det_env"] & (cur_tag >= 0)              # net_module.py:369-370
        # NetObs.update (obs.py:48-87)
        dlv = out["msg_delivered"]
        delay = torch.nan_to_num(out["delay_s"], nan=0.0)
        if "delay_history" in self.dims:
            cap = torch.where(dlv, out["cap"], torch.full_like(out["cap"], -(2 ** 62)))
            idx = cap.argmax(-1, keepdim=True)
            nw = self._t(delay.gather(-1, idx))
            any_d = dlv.any(-1, keepdim=True)
            shifted = torch.cat([nw, self.hist[..., :-1]], -1)
            self.hist = torch.where(any_d, shifted, self.hist)
        cols = []
        for f in self.features:
            if f == "delivered_mask":
                cols.append(dlv.float())
            elif f == "msg_delay":
                cols.append(torch.where(dlv, self._t(delay), torch.zeros_like(delay)))
            elif f == "aoi":
                cols.append(self._t(out["aoi_s"])[..., None])
            elif f == "queue_len":
                cols.append((out["queue_len"].float() / self.F)[..., None])
            elif f == "queue_bytes":
                cols.append((out["queue_bytes"].float() / self.q_bytes)[..., None])
            elif f == "sinr":
                cols.append((out["sinr_db"] / DB_SCALE)[..., None])
            elif f == "rsrp":
                cols.append(((out["rsrp_dbm"] - self.noise) / DB_SCALE)[..., None])
            elif f == "serving_cell":
                cols.append(torch.nn.functional.one_hot(out["serving"].long().clamp(0, self.G - 1), self.G).float())
            elif f == "last_delivered":
                cols.append(out["delivered"].float()[..., None])
            elif f == "delay_history":
                cols.append(self.hist)
            elif f == "blocked":
                cols.append(out["blocked"].float()[..., None])
            elif f == "los":
                cols.append(out["los"].float()[..., None])
        self.x = torch.cat(cols, -1) if cols else self.x
        return out, self.x
