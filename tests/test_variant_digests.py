"""The oracle against the reference over single-setting variants of the benchmark workloads (HARQ, OLLA, PHR, SR and
HARQ timing, queue limits and discard, MCS tables and caps, symbol counts, TDD patterns, numerologies, fading,
noise, RBG sizes, channel and shadowing parameters, A3 / power-control / interference parameters, schedulers, the BSR
pipeline's timers; and the downlink's CQI, HARQ-ACK, MCS cap, TDD and power settings):
tests/golden/variant_digests.json (written by tests/golden/make_variant_digests.py from the reference) holds a digest
of every step's output dict and, at three steps, of the per-robot MAC / HARQ / queue state; the oracle in "aten" mode,
fed the same seeded poses and the host traffic generator's arrivals (bitwise the reference's,
tests/test_traffic_golden.py), must give the same digests.
"""
import importlib
import json
import os
import sys

import pytest
import torch

from oracle.nr_oracle import OracleEngine

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import make_golden  # noqa: E402
import make_variant_digests as mvd  # noqa: E402

ENTRIES = json.load(open(os.path.join(ROOT, "tests", "golden", "variant_digests.json")))
presets = importlib.import_module("isaac-net_b200.presets")
tr = importlib.import_module("isaac-net_b200.traffic")


@pytest.mark.parametrize("j", range(len(ENTRIES)))
def test_oracle_digests_equal_the_reference(j):
    import ast
    e = ENTRIES[j]
    i, over = e["workload"], ast.literal_eval(e["over"])
    wl = presets.workload(i)
    E, R = mvd.E, mvd.robots(i)
    if e["dl_traffic"]:
        over["traffic"] = make_golden.dl_traffic(i, R)
    cfg = wl.config(**over)
    o = OracleEngine(cfg, E, R, "cpu", seed=wl.seed, reduce="aten")
    tseed = (int(wl.seed) * 6364136223846793005 + 1442695040888963407) % 2 ** 62
    gen = tr.TrafficGen(cfg.traffic, E, R, "cpu", cfg.control_step_ms, cfg.slots_per_step, seed=tseed)
    dgen = None
    if cfg.dl and tr.generates(cfg.traffic, "dl"):     # the DL models' own generator, seeded as the engine seeds it
        dseed = (int(wl.seed) * 2862933555777941757 + 3037000493) % 2 ** 62
        dgen = tr.TrafficGen(cfg.traffic, E, R, "cpu", cfg.control_step_ms, cfg.slots_per_step, seed=dseed,
                             direction="dl")
    mot = presets.Motion(i, E, R, seed=wl.seed, step_ms=cfg.control_step_ms)
    pos = mot.current()
    for s in range(mvd.STEPS):
        if s in mvd.RESETS:
            m = torch.zeros(E, dtype=torch.bool)
            m[mvd.RESETS[s]] = True
            o.reset(mvd.RESETS[s])
            gen.reset(m)
            if dgen is not None:
                dgen.reset(m)
        names = ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")
        a = gen.step(torch.zeros(E, dtype=torch.long), None)
        arr = {n: getattr(a, n) for n in names}
        dla = None
        if dgen is not None:
            b = dgen.step(torch.zeros(E, dtype=torch.long), None)
            dla = {n: getattr(b, n) for n in names}
        out = o.step(pos, arr, dl_arrivals=dla)
        got = mvd.digest({k: v.cpu().numpy() for k, v in out.items()})
        assert got == e["digests"][s], (over, s)
        if str(s) in e["state_digests"]:
            st = o.reference_state()
            assert mvd.digest({k: st[k].cpu().numpy() for k in mvd.STATE_KEYS}) == e["state_digests"][str(s)], \
                (over, s, "state")
        pos = mot.advance()
