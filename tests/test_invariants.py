"""The host-side invariant checker (isaac-net_b200/invariants.py) on CPU: a well-formed state passes, and each
planted mistake is reported."""
import importlib
import types

import torch

inv = importlib.import_module("isaac-net_b200.invariants")


def _state(E=2, R=3, P=4, F=5):
    L = torch.long
    st = {"floor_": torch.zeros(E, R, dtype=L), "sent": torch.full((E, R), 100, dtype=L),
          "enq": torch.full((E, R), 300, dtype=L), "bsr": torch.full((E, R), 200, dtype=L),
          "h_state": torch.zeros(E, R, P, dtype=L), "h_lo": torch.zeros(E, R, P, dtype=L),
          "h_hi": torch.zeros(E, R, P, dtype=L), "cap": torch.full((E, R, F), -1, dtype=L),
          "start": torch.zeros(E, R, F, dtype=L), "end_": torch.zeros(E, R, F, dtype=L)}
    st["cap"][..., :2] = 3
    st["start"][..., 0], st["end_"][..., 0] = 0, 150
    st["start"][..., 1], st["end_"][..., 1] = 150, 300
    st["h_state"][..., 0], st["h_lo"][..., 0], st["h_hi"][..., 0] = 1, 0, 100
    return types.SimpleNamespace(st=st, F=F)


def test_well_formed_state_passes():
    assert inv.state_violations(_state()) == []


def test_planted_state_mistakes_are_reported():
    for plant, what in ((lambda st: st["sent"].__setitem__((0, 1), 400), "floor <= sent <= enq"),
                        (lambda st: st["h_state"].__setitem__((1, 2, 3), 2), "HARQ state"),
                        (lambda st: st["h_lo"].__setitem__((0, 0, 0), 120), "h_lo <= h_hi"),
                        (lambda st: st["cap"].__setitem__((1, 0, 0), -1), "prefix"),
                        (lambda st: st["end_"].__setitem__((0, 2, 1), 150), "bytes"),
                        (lambda st: st["start"].__setitem__((1, 1, 1), 100), "stream order"),
                        (lambda st: st["bsr"].__setitem__((0, 0), -5), "bsr")):
        e = _state()
        plant(e.st)
        bad = inv.state_violations(e)
        assert any(what in b for b in bad), (what, bad)


def test_step_conservation():
    E, R, F = 2, 3, 4
    z = torch.zeros(E, R, F, dtype=torch.bool)
    out = {"delivered": z.clone(), "timed_out": z.clone(), "dropped": z.clone(),
           "queue_len": torch.full((E, R), 2, dtype=torch.long)}
    out["delivered"][0, 0, 0] = True
    q_before = torch.full((E, R), 2, dtype=torch.long)
    acc = torch.zeros(E, R, dtype=torch.long)
    acc[0, 0] = 1
    assert inv.step_violations(q_before, acc, out) == []
    acc[1, 1] = 1                                   # a message accepted but neither queued nor gone
    assert inv.step_violations(q_before, acc, out)
