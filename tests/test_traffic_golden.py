"""The host traffic generator (isaac-net_b200/traffic.py) reproduces the reference's arrivals bitwise on CPU: same
torch.Generator seeding and draw order (isaac_net/core/traffic.py:218-430), partial resets included."""
import importlib

import numpy as np
import pytest
import torch

from golden_io import CASES, Golden

tr = importlib.import_module("isaac-net_b200.traffic")


@pytest.mark.parametrize("case", CASES)
def test_arrivals_bitwise(case):
    g = Golden(case)
    cfg, wl = g.config(), g.workload()
    seed = wl.seed
    tseed = (int(seed) * 6364136223846793005 + 1442695040888963407) % 2 ** 62
    gen = tr.TrafficGen(cfg.traffic, g.E, g.R, "cpu", cfg.control_step_ms, cfg.slots_per_step, seed=tseed)
    clock = torch.zeros(g.E, dtype=torch.long)
    for s in range(g.steps):
        ids = g.reset_ids(s)
        if ids:
            m = torch.zeros(g.E, dtype=torch.bool)
            m[ids] = True
            gen.reset(m)
        a = gen.step(clock, None)
        ref = g.arrivals(s)
        for n in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det"):
            assert np.array_equal(getattr(a, n).numpy(), ref[n]), f"step {s} {n}"
