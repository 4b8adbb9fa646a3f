"""The five benchmark workloads of the B200 engine as NRConfig builders, plus their synthetic robot motion.

Each workload is expressed with reference NRConfig fields only, so the same field values build the reference engine
(isaac_net.make_engine("L2", ...)) for parity checks.  The motion generators are seeded CPU torch generators; the
positions they produce are the engine's pose input.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .config import NRConfig
from .traffic import TrafficModel

_DATA = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data")
RADIO_MAP_CFG5 = os.path.join(_DATA, "radio_map_cfg5.npz")     # baked by data/make_radio_map.py (build() runs it)


@dataclass(frozen=True)
class Workload:
    name: str
    E: int            # envs of the whole workload
    R: int
    steps: int
    seed: int
    fields: dict
    E_gpu: int = 0    # envs per GPU of its weak-scaling runs (0: E)

    @property
    def envs_per_gpu(self):
        return self.E_gpu or self.E

    def config(self, **overrides):
        return NRConfig(**{**self.fields, **overrides})


def _common(**kw):
    base = dict(mu=1, tdd_pattern="U", dl=False, rng="engine", fading=True, noise_model="thermal")
    base.update(kw)
    return base


def workload(i: int) -> Workload:
    """BASELINE config i (1..5) as a Workload."""
    if i == 1:
        f = _common(bandwidth_mhz=20, control_step_ms=5.0, channel="tr38901", tr38901_scenario="UMi",
                    tr38901_los="los", gnb_height_m=10.0, carrier_ghz=3.5, scheduler="rr", n_harq=4, max_harq_tx=4,
                    msg_sizes=(1500.0,),
                    traffic=(TrafficModel.bursty(1500, rate_hz=200, burst_size=1, on_off=(1.0, 0.0)),), seed=0)
        return Workload("cfg1_64x16_umi_rr", 64, 16, 200, 0, f)
    if i in (2, 4):
        R = 32 if i == 2 else 128
        n_ctl = round(0.6 * R) if i == 2 else round(0.6 * R)
        f = _common(bandwidth_mhz=100, control_step_ms=5.0, channel="tr38901", tr38901_scenario="UMi",
                    tr38901_los="los", gnb_height_m=10.0, carrier_ghz=3.5, scheduler="pf", pf_window=100.0,
                    msg_sizes=(200.0, 8192.0),
                    traffic=(TrafficModel.periodic(200, period_ms=10.0).on(range(0, n_ctl)),
                             TrafficModel.bursty(8192, rate_hz=20, burst_size=1, on_off=(1.0, 0.0)).on(range(n_ctl, R))),
                    seed=1 if i == 2 else 3)
        if i == 2:
            f.update(fading_rician=True, rician_k_db=5.0)
            return Workload("cfg2_4096x32_pf_rician", 4096, 32, 1000, 1, f)
        return Workload("cfg4_65536x128_pf", 65536, 128, 500, 3, f, E_gpu=8192)
    if i == 3:
        f = _common(bandwidth_mhz=100, control_step_ms=10.0, n_cells=3, cell_layout="hex", cell_isd_m=200.0,
                    channel="log_distance", shadow_sigma_db=6.0, shadow_acf="exp", shadow_dcorr_m=20.0,
                    a3_hyst_db=3.0, scheduler="pf", n_harq=8, max_harq_tx=5, msg_sizes=(1500.0,),
                    traffic=(TrafficModel.bursty(1500, rate_hz=500, burst_size=1, on_off=(1.0, 0.0)),), seed=2)
        return Workload("cfg3_1024x64_3cell", 1024, 64, 500, 2, f)
    if i == 5:
        f = _common(bandwidth_mhz=20, control_step_ms=5.0, n_cells=2, cell_layout="custom",
                    cell_positions_m=((64.0, 128.0), (192.0, 128.0)), channel="radio_map",
                    radio_map_path=RADIO_MAP_CFG5,
                    blockage=True, blockage_model="stochastic", scheduler="rr", n_harq=4, msg_sizes=(1500.0,),
                    traffic=(TrafficModel.bursty(1500, rate_hz=200, burst_size=1, on_off=(1.0, 0.0)),), seed=4)
        return Workload("cfg5_8192x48_radiomap", 8192, 48, 500, 4, f)
    raise ValueError(f"no workload {i}")


class Motion:
    """Seeded synthetic robot positions [E,R,2] (float32) for a workload, advanced once per control step.

    cfg 1: uniform in a 100 x 100 m square centred on the gNB, random walk at 1 m/s.
    cfg 2, 4: uniform in a disc of radius 150 m around the gNB, per-robot constant speed U(0, 2) m/s on a random
    heading that re-draws every step (a random walk), reflected at the disc edge.
    cfg 3: uniform over the hex cluster (disc of radius 1.2 ISD around its centroid), random walk at 1 m/s.
    cfg 5: uniform in the 256 x 256 m map, random walk at 1 m/s."""

    def __init__(self, i: int, E: int, R: int, seed: int = 0, step_ms: float = 5.0):
        self.i, self.E, self.R = i, E, R
        self.dt = step_ms * 1e-3
        self.g = torch.Generator().manual_seed(1000 + seed)
        u = lambda *s: torch.rand(*s, generator=self.g, dtype=torch.float64)
        if i == 1:
            self.center, self.half = (0.0, 0.0), 50.0
            self.pos = (u(E, R, 2) - 0.5) * 100.0
            self.speed = torch.full((E, R), 1.0, dtype=torch.float64)
            self.box = True
        elif i in (2, 4):
            self.center, self.radius = (0.0, 0.0), 150.0
            r = 150.0 * torch.sqrt(u(E, R))
            a = 2 * math.pi * u(E, R)
            self.pos = torch.stack([r * torch.cos(a), r * torch.sin(a)], -1)
            self.speed = 2.0 * u(E, R)
            self.box = False
        elif i == 3:
            self.center, self.radius = (75.0, 75.0), 240.0
            r = 240.0 * torch.sqrt(u(E, R))
            a = 2 * math.pi * u(E, R)
            self.pos = torch.stack([75.0 + r * torch.cos(a), 75.0 + r * torch.sin(a)], -1)
            self.speed = torch.full((E, R), 1.0, dtype=torch.float64)
            self.box = False
        else:
            self.center, self.half = (128.0, 128.0), 128.0
            self.pos = u(E, R, 2) * 256.0
            self.speed = torch.full((E, R), 1.0, dtype=torch.float64)
            self.box = True

    def current(self):
        return self.pos.float()

    def advance(self):
        a = 2 * math.pi * torch.rand(self.E, self.R, generator=self.g, dtype=torch.float64)
        step = (self.speed * self.dt)[..., None] * torch.stack([torch.cos(a), torch.sin(a)], -1)
        p = self.pos + step
        cx, cy = self.center
        if self.box:
            lo_x, hi_x, lo_y, hi_y = cx - self.half, cx + self.half, cy - self.half, cy + self.half
            p[..., 0] = torch.where(p[..., 0] < lo_x, 2 * lo_x - p[..., 0], p[..., 0])
            p[..., 0] = torch.where(p[..., 0] > hi_x, 2 * hi_x - p[..., 0], p[..., 0])
            p[..., 1] = torch.where(p[..., 1] < lo_y, 2 * lo_y - p[..., 1], p[..., 1])
            p[..., 1] = torch.where(p[..., 1] > hi_y, 2 * hi_y - p[..., 1], p[..., 1])
        else:
            d = torch.stack([p[..., 0] - cx, p[..., 1] - cy], -1)
            n = d.norm(dim=-1, keepdim=True)
            out = n > self.radius
            d = torch.where(out, d * (2 * self.radius / n.clamp(min=1e-9) - 1), d)
            p = torch.stack([d[..., 0] + cx, d[..., 1] + cy], -1)
        self.pos = p
        return self.current()


__all__ = ["Workload", "workload", "Motion"]
