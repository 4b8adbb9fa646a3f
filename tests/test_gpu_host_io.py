"""Poses from host memory and outputs fetched to host memory (the engine's own copy streams) give the same step
dicts as device-resident poses, bitwise, over consecutive CUDA-graph steps, with a partial reset in between."""
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")

pytestmark = pytest.mark.gpu

KEYS = ("newest", "queue_len", "queue_bytes", "sinr_db", "delivered", "delay", "serving_cell", "t")


def _same(a, b):
    if a.dtype.is_floating_point:
        return torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0))
    return torch.equal(a, b)


@pytest.mark.parametrize("wl_i,E,R", [(2, 64, 32), (3, 8, 64)])
def test_host_poses_and_fetch_equal_device_path(wl_i, E, R):
    wl = presets.workload(wl_i)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    a = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    b = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    mo = presets.Motion(wl_i, E, R, seed=2, step_ms=cfg.control_step_ms)
    frames = [mo.current()] + [mo.advance() for _ in range(9)]
    host = torch.stack(frames).pin_memory()
    fetched = {k: torch.empty((E,) if k == "t" else (E, R, cfg.frame_buffer) if k in ("delivered", "delay")
                              else (E, R), dtype=torch.int64 if k in ("newest", "queue_len", "serving_cell", "t")
                              else torch.bool if k == "delivered" else torch.float32).pin_memory() for k in KEYS}
    for s in range(10):
        if s == 6:
            a.reset([1])
            b.reset([1])
        out_a = a.step(None, host[s], fetch=fetched)
        out_b = b.step(None, host[s].to(dev))
        a.sync_fetch()
        for k in KEYS:
            assert _same(out_a[k], out_b[k]), (s, k)
            assert _same(fetched[k], out_b[k].cpu()), (s, k)
    sa, sb = a.reference_state(), b.reference_state()
    for k, v in sa.items():
        if torch.is_tensor(v):
            assert _same(v.to(dev), sb[k].to(dev)), k
