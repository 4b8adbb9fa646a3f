"""Known answers for the link-adaptation tables the engine builds on the host (isaac-net_b200/phy.py PhyTables): the
reference's own PHY (isaac_net/core/phy.py:181-263) over a seeded sample of MCS tables, BLER targets, data-slot
symbol counts, DMRS and overhead REs, at every PRB count 0..273.

    python tests/golden/make_phy_golden.py --ref /path/to/isaac-net      # writes tests/golden/phy_tables.npz

Per sample: TBS (bits) [274, M], the BLER table's code-block index and weight, the number of code blocks, and the
MCS thresholds thr_ref [M] at the sample's BLER target.  tests/test_phy_golden.py checks PhyTables against them.
"""
from __future__ import annotations

import argparse
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
NPRB = 273


def samples(n=18, seed=5):
    rnd = random.Random(seed)
    out = []
    while len(out) < n:
        s = (rnd.choice((1, 2)), rnd.choice((0.1, 0.1, 0.01, 0.2)), rnd.randint(1, 14), rnd.choice((0, 6, 12, 18, 24)),
             rnd.choice((0, 0, 6, 18)))
        if s not in out and 12 * s[2] - s[3] - s[4] > 0:
            out.append(s)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ISAAC_NET_REF"),
                    help="source tree of the reference (isaac-net); default $ISAAC_NET_REF, else it must be importable")
    a = ap.parse_args()
    if a.ref:
        sys.path.insert(0, a.ref)
    from isaac_net.core.phy import PHY, segment
    rec = {}
    smp = samples()
    rec["samples"] = np.array(smp, dtype=np.float64)
    n = torch.arange(NPRB + 1, dtype=torch.float32)
    for j, (table, target, nsym, dmrs, oh) in enumerate(smp):
        phy = PHY("ul", table, "cpu", bler_target=target)
        tbs = phy.tbs_all(n, nsym, dmrs, oh)
        cbs, c = segment(tbs, phy.r)
        i0, wi = phy._cidx(cbs.float())
        rec[f"{j}/tbs"] = tbs.to(torch.int32).numpy()
        rec[f"{j}/i0"] = i0.to(torch.int32).numpy()
        rec[f"{j}/wi"] = wi.float().numpy()
        rec[f"{j}/ncb"] = c.float().numpy()
        rec[f"{j}/thr_ref"] = phy.thr_ref.float().numpy()
    path = os.path.join(HERE, "phy_tables.npz")
    np.savez_compressed(path, **rec)
    print(path, os.path.getsize(path), len(smp))


if __name__ == "__main__":
    main()
