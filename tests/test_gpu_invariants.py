"""The engine's state and message conservation checked after every step (NRB200Engine.debug_invariants) over every
config with a partial reset, the policy / SNR-input case, and poses with NaN entries (a fault injected on the host:
the kernels must neither fault nor break an invariant, and the robots with a NaN pose simply never get a grant)."""
import importlib
import math

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wl_i,E,R", [(1, 8, 16), (2, 16, 32), (3, 4, 64), (5, 4, 48), (4, 2, 128)])
def test_invariants_hold_every_step(wl_i, E, R):
    wl = presets.workload(wl_i)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    eng.debug_invariants = True
    mo = presets.Motion(wl_i, E, R, seed=8, step_ms=cfg.control_step_ms)
    pos = mo.current()
    for s in range(12):
        if s == 5:
            eng.reset([0])
        eng.step(None, pos.to(dev))                 # raises on a violation
        pos = mo.advance()


def test_nan_poses_fault_nothing():
    wl = presets.workload(2)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    E, R = 8, 32
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    eng.debug_invariants = True
    mo = presets.Motion(2, E, R, seed=8, step_ms=cfg.control_step_ms)
    for s in range(8):
        pos = mo.current().clone()
        pos[1, :4] = math.nan
        pos[3, 7, 0] = math.inf
        out = eng.step(None, pos.to(dev))
        mo.advance()
        assert bool(out["sinr_db"][1, :4].isnan().all())
    assert eng.counters()["ul"]["tb_new"] > 0


def test_invariants_policy_case():
    from golden_io import Golden
    from test_oracle_golden import run_policy_step
    g = Golden("1p")
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", g.E, g.R, dev, g.config(), seed=g.workload().seed)
    eng.debug_invariants = True
    for s in range(g.steps):
        if g.reset_ids(s):
            eng.reset(g.reset_ids(s))
        run_policy_step(eng, g, s, dev, oracle=False)
