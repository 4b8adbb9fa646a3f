"""Export the BLER / EESM tables the NR engine's link abstraction uses into phy_tables.npz.

The tables are Sionna SYS 2.2.0 AWGN LDPC link-level curves (Apache-2.0), post-processed by isaac-net's
``build_bler_table`` (isaac_net/core/phy.py:405-482: missing rows filled, waterfall continued above the last simulated
point, grid extended down to -15 dB, forced non-increasing) and loaded by its ``PHY`` class (phy.py:188-232).  The
B200 engine must look up the very same numbers to make the same MCS and decode decisions, so this script takes them
from an installed reference rather than re-deriving them:

    python isaac-net_b200/data/make_phy_tables.py --ref /path/to/isaac-net

Saved arrays (float32): bler_t1 [29, C, G], bler_t2 [28, C, G] (MCS x code-block-size axis x SNR grid), snr_grid [G],
cbs_axis [C], beta_t1 [29], beta_t2 [28] (EESM betas per MCS).
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("ISAAC_NET_REF"),
                    help="source tree of the reference (isaac-net); default $ISAAC_NET_REF, else it must be importable")
    a = ap.parse_args()
    if a.ref:
        sys.path.insert(0, a.ref)
    from isaac_net.core.phy import PHY
    out = {}
    for t in (1, 2):
        p = PHY("ul", t, "cpu")
        out[f"bler_t{t}"] = p.bler[0].numpy().astype(np.float32)
        out[f"beta_t{t}"] = p.beta.numpy().astype(np.float32)
        out["snr_grid"] = p.snr_grid.numpy().astype(np.float32)
        out["cbs_axis"] = p.cbs_axis.numpy().astype(np.float32)
    path = os.path.join(HERE, "phy_tables.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))
