"""The bounds-checked build (INB_CHECK: every global index of the MAC kernel checked against its array, an
out-of-range one recorded in the device status word and redirected to element 0) runs the configs' step sequences
with a partial reset, graph and eager steps, radio map and blockage, several cells, the SR / BSR grant pipeline,
policy submits and SNR input, and ends with status 0.  It runs in a child process because the library variant is chosen when the package loads."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

DRIVER = r"""
import importlib, sys, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
ib = importlib.import_module("isaac-net_b200"); nat = importlib.import_module("isaac-net_b200._native")
presets = importlib.import_module("isaac-net_b200.presets")
assert nat.LIB_PATH.endswith("_check.so"), nat.LIB_PATH
dev = torch.device("cuda:0")
bad = []
for wl_i, E, R, over in ((1, 8, 16, {}), (2, 16, 32, {}), (2, 8, 32, dict(scheduler="rr", retx_priority=False)),
                         (3, 4, 64, {}), (5, 4, 48, {}), (1, 4, 16, dict(blockage=True, blockage_model="stochastic")),
                         (4, 2, 128, {}), (2, 8, 32, dict(ul_grant_model="bsr")),
                         (3, 4, 64, dict(ul_grant_model="bsr", a3_ttt_ms=2.0, a3_hyst_db=0.5)),
                         (2, 4, 32, dict(tdd_pattern="DDSUU", dl=True))):
    wl = presets.workload(wl_i)
    cfg = wl.config(**over)
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    mo = presets.Motion(wl_i, E, R, seed=3, step_ms=cfg.control_step_ms)
    pos = mo.current()
    for s in range(8):
        if s == 4:
            eng.reset([1])
        eng.step(None, pos.to(dev))
        pos = mo.advance()
    torch.cuda.synchronize()
    st = int(eng.status.item())
    if st != 0:
        bad.append((wl_i, over, hex(st)))
from golden_io import Golden
from test_oracle_golden import run_policy_step
g = Golden("1p")
eng = ib.make_engine("L2", g.E, g.R, dev, g.config(), seed=g.workload().seed)
for s in range(g.steps):
    if g.reset_ids(s):
        eng.reset(g.reset_ids(s))
    run_policy_step(eng, g, s, dev, oracle=False)
torch.cuda.synchronize()
if int(eng.status.item()) != 0:
    bad.append(("1p", hex(int(eng.status.item()))))
print("BAD", bad)
sys.exit(1 if bad else 0)
"""


def test_bounds_checked_build_reports_nothing():
    lib = os.path.join(ROOT, "isaac-net_b200", "_lib", "libisaac_net_b200_check.so")
    if not os.path.exists(lib):
        sys.path.insert(0, os.path.join(ROOT, "isaac-net_b200"))
        import build
        build.build(check=True)
    env = dict(os.environ, INB_CHECK="1")
    r = subprocess.run([sys.executable, "-c", DRIVER, ROOT], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
