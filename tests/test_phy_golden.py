"""The link-adaptation tables the engine builds on the host (PhyTables: TBS, the BLER table's code-block index and
weight, the code-block count over every PRB count 0..273 and MCS, and the MCS thresholds) against the reference's own
PHY (isaac_net/core/phy.py:181-263) over a seeded sample of MCS tables, BLER targets, symbol counts, DMRS and
overhead REs (tests/golden/phy_tables.npz, written by tests/golden/make_phy_golden.py): bitwise equal."""
import importlib
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
D = np.load(os.path.join(ROOT, "tests", "golden", "phy_tables.npz"))
SAMPLES = [tuple(x) for x in D["samples"]]
NRConfig = importlib.import_module("isaac-net_b200.config").NRConfig
PhyTables = importlib.import_module("isaac-net_b200.phy").PhyTables


def test_sample_covers_the_settings():
    assert {int(s[0]) for s in SAMPLES} == {1, 2}
    assert len({s[1] for s in SAMPLES}) >= 2 and len({s[2] for s in SAMPLES}) >= 8
    assert any(s[3] == 0 for s in SAMPLES) and any(s[4] > 0 for s in SAMPLES)


@pytest.mark.parametrize("j", range(len(SAMPLES)))
def test_link_adaptation_tables_equal_the_reference(j):
    table, target, nsym, dmrs, oh = SAMPLES[j]
    cfg = NRConfig(mu=1, bandwidth_mhz=100, mcs_table=int(table), bler_target=float(target),
                   dmrs_re_per_prb=int(dmrs), overhead_re_per_prb=int(oh))
    assert cfg.nprb == 273
    t = PhyTables(cfg, cfg.subband_prbs, "cpu")
    tbs, i0, wi, ncb = t.la_tables(int(nsym))
    np.testing.assert_array_equal(tbs.numpy(), D[f"{j}/tbs"])
    np.testing.assert_array_equal(i0.numpy(), D[f"{j}/i0"])
    np.testing.assert_array_equal(wi.numpy(), D[f"{j}/wi"])
    np.testing.assert_array_equal(ncb.numpy(), D[f"{j}/ncb"])
    np.testing.assert_array_equal(t.thr_ref.numpy(), D[f"{j}/thr_ref"])
