"""Known answers for the control step's slot schedule: the reference's own NRNet._schedule (isaac_net/core/
nr_engine.py:506-523) over a seeded grid of TDD patterns, numerologies, control-step lengths, link switches, K1,
SR / CQI periods and special-slot splits, at several control steps g0 each.

    python tests/golden/make_schedule_golden.py --ref /path/to/isaac-net      # writes tests/golden/schedule.json

Each entry holds the config fields it set, and per g0 the reference's rows (rel, DL data symbols, UL data symbols,
SR opportunity, CQI report, HARQ-ACK slot relative to g0).  tests/test_schedule_golden.py checks
isaac-net_b200's NRConfig.schedule() and the oracle's Derived.schedule() against them.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

PATTERNS = ("U", "DDDSU", "DDSUU", "DSUUU", "DDDSUDDSUU", "DDDDDDDSUU", "DU", "DDDS", "SU", "DDSU")


def grid(n=80, seed=7):
    """n seeded config settings (fields of NRConfig) whose pattern has an UL-capable slot."""
    rnd = random.Random(seed)
    out = []
    while len(out) < n:
        pat = rnd.choice(PATTERNS)
        split = rnd.choice(((10, 2, 2), (6, 4, 4), (12, 2, 0), (3, 10, 1)))
        if not any(c == "U" or (c == "S" and split[2] > 0) for c in pat):
            continue
        mu = rnd.choice((0, 1, 2))
        slot_ms = 1.0 / 2 ** mu
        steps = rnd.choice((1, 2, 3, 4, 5, 8, 10, 20))
        f = dict(tdd_pattern=pat, mu=mu, control_step_ms=steps * slot_ms, dl=rnd.random() < 0.6,
                 ul=rnd.random() < 0.9, k1=rnd.choice((1, 2, 3, 4)), k2=rnd.choice((1, 2, 4)),
                 sr_period_slots=rnd.choice((1, 2, 4, 10, 20)), cqi_period_slots=rnd.choice((1, 5, 10, 40)),
                 special_split=split, special_dl_data=rnd.random() < 0.7, special_ul_data=rnd.random() < 0.3,
                 dl_ctrl_symbols=rnd.choice((1, 2, 3)), ul_data_symbols=rnd.choice((12, 13, 14)))
        if not (f["dl"] or f["ul"]):
            continue
        out.append(f)
    return out


def g0s(f):
    n = int(round(f["control_step_ms"] * 2 ** f["mu"]))
    return [0, n, 3 * n, 7 * n, 13 * n, 40 * n + n]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ISAAC_NET_REF"),
                    help="source tree of the reference (isaac-net); default $ISAAC_NET_REF, else it must be importable")
    a = ap.parse_args()
    if a.ref:
        sys.path.insert(0, a.ref)
    from isaac_net import make_engine
    from isaac_net.core.config import NRConfig
    entries = []
    for f in grid():
        try:       # the reference refuses some settings (e.g. the uplink on a pattern without UL data symbols)
            cfg = NRConfig(**{**f, "special_split": tuple(f["special_split"])})
            eng = make_engine("L2", 1, 1, "cpu", cfg, strict=None, seed=0)
        except (ValueError, AssertionError, StopIteration):
            continue
        rows = {str(g0): [[int(r[0]), int(r[1]), int(r[2]), bool(r[3]), bool(r[4]), int(r[5])]
                          for r in eng.net._schedule(g0)] for g0 in g0s(f)}
        entries.append({"fields": f, "rows": rows})
    path = os.path.join(HERE, "schedule.json")
    with open(path, "w") as fh:
        json.dump(entries, fh, separators=(",", ":"))
    print(path, os.path.getsize(path), len(entries))


if __name__ == "__main__":
    main()
