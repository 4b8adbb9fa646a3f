"""Checkpoints: state_dict() of a running engine loaded into a fresh engine of the same config continues exactly
like the original (every output of the following steps and the final state bitwise equal, CUDA graphs on), through a
file as well; mismatched sizes and configs are refused."""
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")

pytestmark = pytest.mark.gpu


def _same(a, b):
    if not torch.is_tensor(a):
        return a == b
    if a.dtype.is_floating_point:
        return torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0))
    return torch.equal(a, b)


@pytest.mark.parametrize("wl_i,E,R", [(2, 32, 32), (3, 4, 64), (5, 6, 48), (1, 8, 16)])
def test_resume_is_bitwise_the_uninterrupted_run(wl_i, E, R, tmp_path):
    wl = presets.workload(wl_i)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    a = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    mo = presets.Motion(wl_i, E, R, seed=6, step_ms=cfg.control_step_ms)
    frames = [mo.current()] + [mo.advance() for _ in range(11)]
    for s in range(5):
        if s == 3:
            a.reset([1])
        a.step(None, frames[s].to(dev))
    sd = a.state_dict()
    b = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    b.step(None, frames[0].to(dev))              # b has its own history (and captured radio) before the restore
    b.load_state_dict(sd)
    a.save(tmp_path / "ck.pt", extra={"iter": 5})
    c = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    assert c.load(tmp_path / "ck.pt") == {"iter": 5}
    for s in range(5, 12):
        outs = [e.step(None, frames[s].to(dev)) for e in (a, b, c)]
        for k, v in outs[0].items():
            for o in outs[1:]:
                assert _same(v, o[k]), (s, k)
    fa, fb, fc = a.state_dict(), b.state_dict(), c.state_dict()
    for k, v in fa.items():
        assert _same(v, fb[k]) and _same(v, fc[k]), k
    assert a.counters() == b.counters() == c.counters()


def test_refusals():
    wl = presets.workload(1)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    a = ib.make_engine("L2", 8, 16, dev, cfg, seed=0)
    sd = a.state_dict()
    with pytest.raises(ValueError):
        ib.make_engine("L2", 4, 16, dev, cfg, seed=0).load_state_dict(sd)
    with pytest.raises(ValueError):
        ib.make_engine("L2", 8, 16, dev, cfg.with_(n_harq=8), seed=0).load_state_dict(sd)
    bad = dict(sd)
    bad.pop("st.sent")
    with pytest.raises(KeyError):
        ib.make_engine("L2", 8, 16, dev, cfg, seed=0).load_state_dict(bad)
    ib.make_engine("L2", 8, 16, dev, cfg, seed=0).load_state_dict(bad, strict=False)
