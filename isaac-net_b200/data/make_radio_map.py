"""Bake the radio map of benchmark config 5 into radio_map_cfg5.npz (the reference's radio-map file format).

The format is the one isaac-net's ``RadioMap.load`` reads (isaac_net/core/channels/radio_map.py:1-16, 68-79):
``gain_db`` float32 [C, H, W], path gain in dB between cell c and a UE at grid point (x_j, y_i) (row i along y,
column j along x), ``bounds`` float64 (x0, y0, x1, y1) with x_j = x0 + j (x1 - x0) / (W - 1), plus scalar or small
metadata arrays (``fc_ghz``, ``ue_height_m``, ``gnb_xy``, ``gnb_z``, ``diffraction``, ``source``).

The reference ships no generator for such a scene (its synthetic maps are a wall or warehouse racks), so this map is
built here, deterministically, from:

* a 512 x 512 grid at 0.5 m spacing over a 255.5 m x 255.5 m arena (bounds (0, 0, 255.5, 255.5)),
* two gNBs at (64, 128) and (192, 128), 25 m high, UEs at 1.5 m, carrier 3.5 GHz,
* TR 38.901 UMa LOS path loss (Table 7.4.1-1: PL1 = 28 + 22 log10 d3D + 20 log10 fc below the breakpoint distance
  d'BP = 4 h'BS h'UT fc / c with effective heights h - 1 m, PL2 = 28 + 40 log10 d3D + 20 log10 fc
  - 9 log10(d'BP^2 + (hBS - hUT)^2) above it; d2D floored at 10 m),
* 20 axis-aligned box obstacles drawn from numpy's PCG64 generator with seed 20 (centre uniform in [16, 240]^2, side
  lengths uniform in [6, 24] m, height uniform in [6, 20] m; a draw whose footprint comes within 8 m of a gNB is
  drawn again),
* single knife-edge diffraction (ITU-R P.526 eq. 31, J(v) = 6.9 + 20 log10(sqrt((v - 0.1)^2 + 1) + v - 0.1) for
  v > -0.78, else 0) over every box edge that the direct gNB-UE path crosses: for each crossed box the entry and exit
  points of the 2-D segment are edge candidates, the clearance h of the box top above the straight 3-D ray gives
  v = h sqrt(2 (d1 + d2) / (lambda d1 d2)) with d1, d2 the 3-D distances to both ends (each at least 0.5 m), and the
  link takes the largest J over all candidates, capped at 40 dB.

gain_db = -(PL + J) in float32.  All arithmetic is float64 numpy with a fixed op order, so the file is the same on
every run; its SHA-256 over ``gain_db`` is ``gain_digest()`` and is stored in the golden fixtures made with it.

    python isaac-net_b200/data/make_radio_map.py          # writes radio_map_cfg5.npz beside this script
"""
from __future__ import annotations

import hashlib
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MAP_PATH = os.path.join(HERE, "radio_map_cfg5.npz")

GNB_XY = ((64.0, 128.0), (192.0, 128.0))
H_BS, H_UT, FC_GHZ = 25.0, 1.5, 3.5
N_GRID, SPACING = 512, 0.5
N_BOXES, BOX_SEED = 20, 20
J_CAP_DB = 40.0
C_LIGHT = 299_792_458.0


def _boxes():
    """[N_BOXES, 5] (x_lo, y_lo, x_hi, y_hi, height)."""
    rng = np.random.Generator(np.random.PCG64(BOX_SEED))
    out = []
    while len(out) < N_BOXES:
        cx, cy = rng.uniform(16.0, 240.0, 2)
        w, d = rng.uniform(6.0, 24.0, 2)
        h = rng.uniform(6.0, 20.0)
        lo_x, hi_x, lo_y, hi_y = cx - w / 2, cx + w / 2, cy - d / 2, cy + d / 2
        near = any(lo_x - 8.0 <= gx <= hi_x + 8.0 and lo_y - 8.0 <= gy <= hi_y + 8.0 for gx, gy in GNB_XY)
        if not near:
            out.append((lo_x, lo_y, hi_x, hi_y, h))
    return np.asarray(out, dtype=np.float64)


def _uma_los_db(d2, d3):
    fc = FC_GHZ * 1e9
    dbp = 4 * (H_BS - 1.0) * (H_UT - 1.0) * fc / C_LIGHT
    lf = 20 * math.log10(FC_GHZ)
    pl1 = 28.0 + 22.0 * np.log10(d3) + lf
    pl2 = 28.0 + 40.0 * np.log10(d3) + lf - 9.0 * math.log10(dbp ** 2 + (H_BS - H_UT) ** 2)
    return np.where(d2 <= dbp, pl1, pl2)


def _knife_edge_db(v):
    j = 6.9 + 20.0 * np.log10(np.sqrt((v - 0.1) ** 2 + 1.0) + v - 0.1)
    return np.where(v > -0.78, j, 0.0)


def _segment_box(gx, gy, X, Y, box):
    """Slab test of the 2-D segments gNB -> (X, Y) against one box: (crossed, s_in, s_out) with s the fraction of the
    way from the gNB."""
    lo_x, lo_y, hi_x, hi_y, _ = box
    dx, dy = X - gx, Y - gy
    s0 = np.zeros_like(X)
    s1 = np.ones_like(X)
    for d, o, lo, hi in ((dx, gx, lo_x, hi_x), (dy, gy, lo_y, hi_y)):
        par = np.abs(d) < 1e-12
        inside = (o >= lo) & (o <= hi)
        with np.errstate(divide="ignore", invalid="ignore"):
            ta = (lo - o) / d
            tb = (hi - o) / d
        t_lo = np.where(par, np.where(inside, -np.inf, np.inf), np.minimum(ta, tb))
        t_hi = np.where(par, np.where(inside, np.inf, -np.inf), np.maximum(ta, tb))
        s0 = np.maximum(s0, t_lo)
        s1 = np.minimum(s1, t_hi)
    return s0 <= s1, s0, s1


def bake():
    """{gain_db [C,H,W] float32, bounds, metadata} of the config-5 scene."""
    xs = np.arange(N_GRID, dtype=np.float64) * SPACING
    X, Y = np.meshgrid(xs, xs)                       # [H, W]: row i = y_i, column j = x_j
    lam = C_LIGHT / (FC_GHZ * 1e9)
    boxes = _boxes()
    gains = []
    for gx, gy in GNB_XY:
        d2 = np.maximum(np.hypot(X - gx, Y - gy), 10.0)
        d3 = np.sqrt(d2 ** 2 + (H_BS - H_UT) ** 2)
        pl = _uma_los_db(d2, d3)
        seg2 = np.hypot(X - gx, Y - gy)
        seg3 = np.sqrt(seg2 ** 2 + (H_BS - H_UT) ** 2)
        j_max = np.zeros_like(X)
        for box in boxes:
            hit, s_in, s_out = _segment_box(gx, gy, X, Y, box)
            for s in (s_in, s_out):
                s = np.clip(s, 0.0, 1.0)
                ray = H_BS + (H_UT - H_BS) * s
                clear = box[4] - ray
                d1 = np.maximum(s * seg3, 0.5)
                dd = np.maximum((1.0 - s) * seg3, 0.5)
                v = clear * np.sqrt(2.0 * (d1 + dd) / (lam * d1 * dd))
                j = np.where(hit, _knife_edge_db(v), 0.0)
                j_max = np.maximum(j_max, j)
        gains.append(-(pl + np.minimum(j_max, J_CAP_DB)))
    gain = np.stack(gains).astype(np.float32)
    top = (N_GRID - 1) * SPACING
    return {"gain_db": gain, "bounds": np.asarray((0.0, 0.0, top, top), dtype=np.float64),
            "fc_ghz": np.asarray(FC_GHZ), "ue_height_m": np.asarray(H_UT),
            "gnb_xy": np.asarray(GNB_XY, dtype=np.float64), "gnb_z": np.asarray([H_BS] * len(GNB_XY)),
            "diffraction": np.asarray(True), "source": np.asarray("isaac-net_b200 UMa + 20 boxes + knife edge")}


def gain_digest(gain_db):
    return hashlib.sha256(np.ascontiguousarray(gain_db, dtype=np.float32).tobytes()).hexdigest()


def write(path=MAP_PATH):
    d = bake()
    np.savez_compressed(path, **d)
    return path, gain_digest(d["gain_db"])


def ensure(path=MAP_PATH):
    """Bake the map if the file is missing; returns its path."""
    if not os.path.exists(path):
        write(path)
    return path


if __name__ == "__main__":
    p, dig = write()
    print(p, os.path.getsize(p), dig)
