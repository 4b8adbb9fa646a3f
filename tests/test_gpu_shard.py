"""Two engine shards on one GPU (global env ids, initial reset redone: isaac_net/core/sharded.py:61-77) against one
unsharded engine: with every draw keyed by (seed, global env id, episode), the concatenated shard outputs and state
equal the unsharded engine's bitwise.  This is the per-rank setup of bench.py's multi-GPU run."""
import importlib

import pytest
import torch

from test_shard_gloo import KEYS, SEED, _config, _inputs

ib = importlib.import_module("isaac-net_b200")
tr = importlib.import_module("isaac-net_b200.traffic")

pytestmark = pytest.mark.gpu


def _arr(d, sl, dev):
    return tr.Arrivals(**{k: v[sl].to(dev) for k, v in d.items()})


def test_two_shards_on_one_gpu_equal_one_engine():
    dev = torch.device("cuda:0")
    cfg = _config()
    E, R = 8, 16
    full = ib.make_engine("L2", 2 * E, R, dev, cfg, seed=SEED)
    shards = [ib.make_engine("L2", E, R, dev, cfg, seed=SEED) for _ in range(2)]
    for i, s in enumerate(shards):
        s.set_env_offset(i * E)
    for t, (pos, arr) in enumerate(_inputs(2 * E, R, 5, cfg.slots_per_step)):
        o_full = full.step(None, pos.to(dev), _arrivals=_arr(arr, slice(None), dev))
        o_sh = [s.step(None, pos[i * E:(i + 1) * E].to(dev), _arrivals=_arr(arr, slice(i * E, (i + 1) * E), dev))
                for i, s in enumerate(shards)]
        for k in KEYS:
            a, b = torch.cat([o[k] for o in o_sh], 0), o_full[k]
            if a.is_floating_point():
                assert torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0)), (t, k)
            else:
                assert torch.equal(a, b), (t, k)
    st_full = full.reference_state()
    st_sh = [s.reference_state() for s in shards]
    for k in ("ul.sent", "ul.olla", "ul.avg", "ul.csi", "net.h", "q.cap", "q.fin"):
        assert torch.equal(torch.cat([s[k] for s in st_sh], 0), st_full[k]), k
