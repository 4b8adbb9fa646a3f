"""ShardedEngine's host logic on CPU: the split, global env ids -> shards, the input slicing (tensors, Requests,
fetch= host rows), the gather on the first device, resets by index list and by mask, counters summed over shards,
the shard seeds, and checkpoints under "shards[i]." (isaac_net/core/sharded.py:80-191, checkpoint.py's list-element
naming).  The shards here are a CPU stand-in engine whose outputs are a function of the global env id and the inputs,
so a sharded run must equal one stand-in over the whole batch; tests/test_gpu_sharded_engine.py runs the real engine.
"""
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
sharded = importlib.import_module("isaac-net_b200.sharded")
presets = importlib.import_module("isaac-net_b200.presets")
tr = importlib.import_module("isaac-net_b200.traffic")


class StandIn:
    """The contract surface of NRB200Engine that ShardedEngine drives, on the CPU."""

    def __init__(self, level, E, R, device, cfg, backend, seed=None, traffic_rng="generator"):
        self.E, self.R, self.dev, self.seed = E, R, torch.device(device), seed
        self.env_id = torch.arange(E)
        self.episode = torch.zeros(E, dtype=torch.long)
        self.acc = torch.zeros(E, R, dtype=torch.float64)
        self.T = 0
        self.fetched = 0

    def set_env_offset(self, offset):
        self.env_id = torch.arange(self.E) + offset

    def _mask(self, env_ids):
        if env_ids is None:
            return torch.ones(self.E, dtype=torch.bool)
        if torch.is_tensor(env_ids) and env_ids.dtype == torch.bool:
            return env_ids
        m = torch.zeros(self.E, dtype=torch.bool)
        m[torch.as_tensor(env_ids, dtype=torch.long)] = True
        return m

    def reset(self, env_ids=None):
        m = self._mask(env_ids)
        self.acc[m] = 0.0
        self.episode[m] += 1

    def submit(self, t, requests, snr_db=None, **kw):
        acc = (requests.send > 0).long()
        self.acc += acc
        return acc

    def step(self, t=None, x=None, cur_hid=None, *, fetch=None, snr_db=None):
        assert x.shape[0] == self.E
        self.acc += x.double().sum(-1) * (self.env_id + 1)[:, None] + (self.seed % 7)
        self.T += 1
        out = {"newest": self.acc.long(), "queue_bytes": self.acc.float(), "det_env": self.env_id % 2 == 0,
               "t": torch.full((self.E,), self.T), "scalar": torch.tensor(3)}
        if fetch:
            for k, dst in fetch.items():
                dst.copy_(out[k])
            self.fetched += 1
        if cur_hid is not None:
            return out["newest"], out["det_env"]
        return out

    def sync_fetch(self):
        pass

    @property
    def clock(self):
        return torch.full((self.E,), self.T) - self.episode

    def output_schema(self):
        return {"newest": {"shape": (self.E, self.R), "dtype": "int64"}, "t": {"shape": (self.E,), "dtype": "int64"}}

    def queued(self):
        return (self.acc > 0).sum(-1)

    def counters(self):
        # integer-valued totals, as the engine's counters are (sums over shards are then exact)
        n = self.acc.floor()
        return {"ul": {"tb_ok": float(n.sum()), "ntx_hist": [float(n[:, 0].sum()), float(n[:, 1].sum())]}}

    def state_dict(self):
        return {"acc": self.acc.clone(), "T": self.T, "episode": self.episode.clone()}

    def load_state_dict(self, sd, strict=True):
        self.acc.copy_(sd["acc"])
        self.T = sd["T"]
        self.episode.copy_(sd["episode"])

    def reference_checkpoint(self):
        return {"net.acc": self.acc.clone(), "T": self.T}

    def load_reference_checkpoint(self, sd, strict=False):
        self.acc.copy_(sd["net.acc"])
        self.T = sd["T"]
        return [k for k in sd if k not in ("net.acc", "T")]


@pytest.fixture
def standin(monkeypatch):
    made = []

    def make(level, E, R, device, cfg, backend, **kw):
        e = StandIn(level, E, R, device, cfg, backend, **kw)
        made.append(e)
        return e
    monkeypatch.setattr(sharded, "_make", make)
    return made


def _cfg():
    return presets.workload(1).config(traffic=None)


def _poses(E, R, steps):
    g = torch.Generator().manual_seed(5)
    return [torch.rand(E, R, 2, generator=g) for _ in range(steps)]


def test_split_and_locate(standin):
    sh = sharded.ShardedEngine("L2", 10, 4, ["cpu", "cpu", "cpu"], _cfg(), seed=1)
    assert sh.split == [4, 3, 3] and sh.offsets == [0, 4, 7]
    assert [s.E for s in standin] == [4, 3, 3]
    assert [int(s.env_id[0]) for s in standin] == [0, 4, 7]
    assert sh.locate(0) == (0, 0) and sh.locate(4) == (1, 0) and sh.locate(9) == (2, 2)
    assert sh.shard_of.tolist() == [0] * 4 + [1] * 3 + [2] * 3
    assert sh.local_of.tolist() == [0, 1, 2, 3, 0, 1, 2, 0, 1, 2]
    with pytest.raises(IndexError):
        sh.locate(10)
    sh2 = sharded.ShardedEngine("L2", 10, 4, ["cpu", "cpu"], _cfg(), seed=1, split=[7, 3])
    assert sh2.offsets == [0, 7] and sh2.locate(7) == (1, 0)
    for bad in ([5, 4], [10, 0], [10]):
        with pytest.raises(ValueError):
            sharded.ShardedEngine("L2", 10, 4, ["cpu", "cpu"], _cfg(), seed=1, split=bad)
    with pytest.raises(AttributeError):
        sh.no_such_attribute


@pytest.mark.parametrize("split", [None, [2, 6], [5, 3]])
def test_sharded_equals_one_engine(standin, split):
    E, R = 8, 4
    sh = sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=3, split=split)
    one = StandIn("L2", E, R, "cpu", _cfg(), "b200", seed=3)
    assert sh.shard_invariant and all(s.seed == 3 for s in sh.shards)
    for t, x in enumerate(_poses(E, R, 6)):
        if t == 2:
            sh.reset([1, 6])
            one.reset([1, 6])
        if t == 4:
            m = torch.zeros(E, dtype=torch.bool)
            m[[0, 5, 7]] = True
            sh.reset(m)
            one.reset(m)
        send = (torch.arange(E * R).reshape(E, R) + t) % 3
        a, b = sh.submit(None, tr.Requests(send=send)), one.submit(None, tr.Requests(send=send))
        assert torch.equal(a, b)
        oa, ob = sh.step(None, x), one.step(None, x)
        assert oa.keys() == ob.keys()
        for k in oa:
            assert torch.equal(oa[k], ob[k]), (t, k)
        assert torch.equal(sh.clock, one.clock)
        assert torch.equal(sh.queued(), one.queued())
    assert sh.counters() == one.counters()
    newest, det = sh.step(None, _poses(E, R, 1)[0], torch.zeros(E, dtype=torch.long))
    assert newest.shape == (E, R) and det.shape == (E,)
    sh.reset(None)
    assert all(float(s.acc.abs().sum()) == 0.0 for s in sh.shards)


def test_fetch_fills_each_shards_rows(standin):
    E, R = 6, 4
    sh = sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=2, split=[4, 2])
    host = {"newest": torch.zeros(E, R, dtype=torch.long), "queue_bytes": torch.zeros(E, R)}
    out = sh.step(None, _poses(E, R, 1)[0], fetch=host)
    sh.sync_fetch()
    assert torch.equal(host["newest"], out["newest"]) and torch.equal(host["queue_bytes"], out["queue_bytes"])
    assert [s.fetched for s in sh.shards] == [1, 1]


def test_output_schema_covers_the_whole_batch(standin):
    sh = sharded.ShardedEngine("L2", 9, 4, ["cpu", "cpu"], _cfg(), seed=2)
    sch = sh.output_schema()
    assert sch["newest"]["shape"] == (9, 4) and sch["t"]["shape"] == (9,)


def test_seeds_follow_the_reference_rule(standin):
    cfg = presets.workload(1).config()          # a Poisson traffic model: a sequential generator per engine
    assert not sharded.shard_invariant("L2", cfg)
    assert sharded.shard_invariant("L2", cfg, traffic_rng="counter")
    assert sharded.shard_invariant("L2", _cfg())
    assert not sharded.shard_invariant("L1", _cfg())
    sh = sharded.ShardedEngine("L2", 6, 4, ["cpu", "cpu", "cpu"], cfg, seed=11)
    assert not sh.shard_invariant
    assert [s.seed for s in sh.shards] == [(11 + i * 0x9E3779B97F4A7C15) % 2 ** 62 for i in range(3)]
    shc = sharded.ShardedEngine("L2", 6, 4, ["cpu", "cpu"], cfg, seed=11, traffic_rng="counter")
    assert shc.shard_invariant and [s.seed for s in shc.shards] == [11, 11]


def test_checkpoints_by_shard(standin, tmp_path):
    E, R = 7, 4
    a = sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=4)
    xs = _poses(E, R, 6)
    for x in xs[:3]:
        a.step(None, x)
    sd = a.state_dict()
    assert sd["meta.split"] == [4, 3] and "shards[0].acc" in sd and "shards[1].T" in sd
    b = sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=4)
    b.step(None, xs[0])
    b.load_state_dict(sd)
    a.save(tmp_path / "s.pt", extra={"iter": 3})
    c = sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=4)
    assert c.load(tmp_path / "s.pt") == {"iter": 3}
    for x in xs[3:]:
        oa, ob, oc = (e.step(None, x) for e in (a, b, c))
        assert torch.equal(oa["newest"], ob["newest"]) and torch.equal(oa["newest"], oc["newest"])
    with pytest.raises(ValueError):
        sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=4, split=[3, 4]).load_state_dict(sd)
    ref = a.reference_checkpoint()
    assert "shards[0].net.acc" in ref and "shards[1].T" in ref
    ref["shards[1].net.extra"] = torch.zeros(1)
    d = sharded.ShardedEngine("L2", E, R, ["cpu", "cpu"], _cfg(), seed=4)
    unused = d.load_reference_checkpoint(dict(ref, shard_of=torch.zeros(E)))
    assert sorted(unused) == ["shard_of", "shards[1].net.extra"]
    assert torch.equal(d.shards[1].acc, a.shards[1].acc)


def test_package_exports():
    assert ib.ShardedEngine is sharded.ShardedEngine and ib.shard_invariant is sharded.shard_invariant
