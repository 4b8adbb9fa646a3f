"""ShardedEngine on the GPU (isaac_net/core/sharded.py:80-191): two shards on cuda:0 behind one engine's API.

With the counter-keyed traffic stream every draw of an env is keyed by (seed, global env id, episode), so the sharded
engine's step dicts (gathered on the first device) equal one engine over the whole batch bitwise, partial resets by
global env id included, and so do its counters; host poses in and fetch= host outputs through the sharded engine give
the same step; a state_dict() of the sharded engine loaded into a fresh one continues exactly like the original."""
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")

pytestmark = pytest.mark.gpu


def _same(a, b):
    if a.is_floating_point():
        return torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0))
    return torch.equal(a, b)


@pytest.mark.parametrize("wl_i,split", [(1, [3, 5]), (2, None)])
def test_sharded_engine_equals_one_engine(wl_i, split):
    wl = presets.workload(wl_i)
    cfg = wl.config()
    E, R, dev = 8, wl.R, torch.device("cuda:0")
    one = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed, traffic_rng="counter")
    sh = ib.ShardedEngine("L2", E, R, [dev, dev], cfg, seed=wl.seed, split=split, traffic_rng="counter")
    assert sh.shard_invariant and [s.E for s in sh.shards] == (split or [4, 4])
    mo = presets.Motion(wl_i, E, R, seed=9, step_ms=cfg.control_step_ms)
    delivered = 0
    for s in range(10):
        if s == 5:
            one.reset([1, 6])
            sh.reset([1, 6])
        pos = mo.current().to(dev)
        o, w = one.step(None, pos), sh.step(None, pos)
        assert o.keys() == w.keys()
        for k, v in o.items():
            if torch.is_tensor(v) and v.dim() > 0:
                assert _same(v, w[k]), (s, k)
        delivered += int(o["delivered"].sum())
        mo.advance()
    assert delivered > 0
    assert torch.equal(one.clock, sh.clock) and torch.equal(one.queued(), sh.queued())
    assert one.counters() == sh.counters()
    # host poses in, host outputs out: each shard copies its rows on its own streams
    pos = mo.current()
    host = {"newest": torch.empty(E, R, dtype=torch.long).pin_memory(),
            "sinr_db": torch.empty(E, R, dtype=torch.float32).pin_memory()}
    o = one.step(None, pos.to(dev))
    w = sh.step(None, pos.pin_memory(), fetch=host)
    sh.sync_fetch()
    for k in host:
        assert _same(o[k], w[k]) and _same(o[k].cpu(), host[k]), k


def test_sharded_engine_resume(tmp_path):
    wl = presets.workload(1)
    cfg = wl.config()
    E, R, dev = 8, wl.R, torch.device("cuda:0")
    a = ib.ShardedEngine("L2", E, R, [dev, dev], cfg, seed=wl.seed, split=[5, 3])
    assert not a.shard_invariant                     # Poisson traffic on the generator stream: derived seeds
    mo = presets.Motion(1, E, R, seed=6, step_ms=cfg.control_step_ms)
    frames = [mo.current()] + [mo.advance() for _ in range(9)]
    for s in range(5):
        if s == 3:
            a.reset([1, 6])
        a.step(None, frames[s].to(dev))
    sd = a.state_dict()
    b = ib.ShardedEngine("L2", E, R, [dev, dev], cfg, seed=wl.seed, split=[5, 3])
    b.step(None, frames[0].to(dev))
    b.load_state_dict(sd)
    a.save(tmp_path / "sh.pt", extra={"iter": 5})
    c = ib.ShardedEngine("L2", E, R, [dev, dev], cfg, seed=wl.seed, split=[5, 3])
    assert c.load(tmp_path / "sh.pt") == {"iter": 5}
    for s in range(5, 10):
        outs = [e.step(None, frames[s].to(dev)) for e in (a, b, c)]
        for k, v in outs[0].items():
            if torch.is_tensor(v) and v.dim() > 0:
                assert _same(v, outs[1][k]) and _same(v, outs[2][k]), (s, k)
    assert a.counters() == b.counters() == c.counters()
