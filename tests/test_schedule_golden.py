"""The control step's slot schedule against the reference's own NRNet._schedule (isaac_net/core/nr_engine.py:506-523):
tests/golden/schedule.json (written by tests/golden/make_schedule_golden.py from the reference) holds its rows for a
seeded grid of TDD patterns, numerologies, control-step lengths, link switches, K1, SR / CQI periods and special-slot
splits.  NRConfig.schedule() (the rows the engine turns into its launch table) and the oracle's Derived.schedule()
must give the same rows; the HARQ-ACK slot is compared where the downlink is on (it is read only there)."""
import importlib
import json
import os

import pytest

from oracle.nr_oracle import Derived

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

NRConfig = importlib.import_module("isaac-net_b200.config").NRConfig
ENTRIES = json.load(open(os.path.join(ROOT, "tests", "golden", "schedule.json")))


def _rows(rows, dl):
    return [(int(r[0]), int(r[1]), int(r[2]), bool(r[3]), bool(r[4]), int(r[5]) if dl else 0) for r in rows]


def test_grid_covers_the_switches():
    f = [e["fields"] for e in ENTRIES]
    assert len(ENTRIES) >= 60
    assert {x["mu"] for x in f} == {0, 1, 2}
    assert any(not x["ul"] for x in f) and any(not x["dl"] for x in f)
    assert any("S" in x["tdd_pattern"] and x["special_ul_data"] for x in f)
    assert any(any(r[3] for rows in e["rows"].values() for r in rows) for e in ENTRIES)       # SR opportunities
    assert any(any(r[4] for rows in e["rows"].values() for r in rows) for e in ENTRIES)       # CQI reports


@pytest.mark.parametrize("i", range(len(ENTRIES)))
def test_schedule_rows_equal_the_reference(i):
    e = ENTRIES[i]
    f = dict(e["fields"], special_split=tuple(e["fields"]["special_split"]))
    cfg = NRConfig(**f)
    d = Derived(cfg)
    for g0, ref in e["rows"].items():
        want = _rows(ref, cfg.dl)
        assert _rows(cfg.schedule(int(g0)), cfg.dl) == want, (f, g0)
        assert _rows(d.schedule(int(g0)), cfg.dl) == want, (f, g0)
