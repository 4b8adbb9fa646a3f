"""The traffic kernel (inb_traffic_step, through the C ABI) against TrafficGen's torch calls on the same CUDA device.

TrafficGen draws every uniform as a float64 torch.rand([E, R]) on a CUDA torch.Generator, exactly as the reference
(isaac_net/core/traffic.py:218-430).  The kernel replays that Philox stream itself; this test requires the arrivals
(every field), the model state and the deferred counts to be bitwise equal step after step, partial resets included,
for periodic / video / bursty mixes and for E x R large enough that torch's grid-stride launch serves several
elements per thread (the layout the kernel reproduces).
"""
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
tr = importlib.import_module("isaac-net_b200.traffic")
nat = importlib.import_module("isaac-net_b200._native")
TM = tr.TrafficModel
ARR = ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")

pytestmark = pytest.mark.gpu

MIXES = {
    "cfg1": (TM.bursty(1500, rate_hz=200, burst_size=1, on_off=(1.0, 0.0)),),
    "cfg2": (TM.periodic(200, period_ms=10.0).on(range(0, 19)),
             TM.bursty(8192, rate_hz=20, burst_size=1, on_off=(1.0, 0.0)).on(range(19, 32))),
    "mixed": (TM.periodic(200, period_ms=3.0, jitter_ms=1.0).on(range(0, 6)),
              TM.periodic(64, period_ms=2.5, phase="aligned", priority=2, deadline_ms=4.0),
              TM.video(30, gop=(8000, 1000, 10), jitter_ms=2.0).on(range(4, 20)),
              TM.bursty(1000, rate_hz=400, burst_size=2, on_off=(0.02, 0.01), tag=7, det=True).on(range(10, 24)),
              TM.bursty(300, rate_hz=50, burst_size=1, on_off=(0.5, 0.0), deadline_ms=20.0)),
}


def _pair(models, E, R, step_ms, N, seed):
    dev = torch.device("cuda:0")
    a = tr.TrafficGen(models, E, R, dev, step_ms, N, seed=seed)
    b = tr.TrafficGen(models, E, R, dev, step_ms, N, seed=seed)
    assert tr.DeviceTrafficGen.supports(b)
    return a, b, tr.DeviceTrafficGen(b, nat.lib())


def _check(a, b, arr_a, arr_b, step):
    for k in ARR:
        x, y = getattr(arr_a, k), getattr(arr_b, k)
        assert x.dtype == y.dtype and x.shape == y.shape, (step, k)
        assert torch.equal(x, y), f"step {step}: arrivals.{k} differ at {(x != y).nonzero()[:5].tolist()}"
    for i, (sa, sb) in enumerate(zip(a.sources, b.sources)):
        for n in sa.names:
            assert torch.equal(getattr(sa, n), getattr(sb, n)), f"step {step}: source {i} state {n}"
        assert int(sa.deferred) == int(sb.deferred), f"step {step}: source {i} deferred"


@pytest.mark.parametrize("mix,E,R,steps,seed", [("cfg1", 64, 16, 60, 11), ("cfg2", 256, 32, 60, 12),
                                                ("mixed", 37, 24, 80, 13)])
def test_traffic_kernel_equals_torch_generator(mix, E, R, steps, seed):
    a, b, d = _pair(MIXES[mix], E, R, 5.0, 10, seed)
    reset_at = steps // 2
    for s in range(steps):
        if s == reset_at:
            m = torch.zeros(E, dtype=torch.bool, device="cuda:0")
            m[::3] = True
            a.reset(m)
            b.reset(m)
        arr_a = a.step()
        arr_b = d.step()
        _check(a, b, arr_a, arr_b, s)


def test_traffic_kernel_large_grid_layout():
    """E x R = 640000 elements: more than twice torch's maximum grid, so threads serve several elements per call
    pair and several calls (curand subsequence / offset / component mapping)."""
    props = torch.cuda.get_device_properties(0)
    cap = 256 * props.multi_processor_count * (props.max_threads_per_multi_processor // 256)
    E, R = 5000, 128
    assert E * R > 2 * cap
    a, b, d = _pair(MIXES["cfg2"][:1] + (TM.bursty(8192, rate_hz=300, burst_size=1, on_off=(0.05, 0.02)),),
                    E, R, 5.0, 10, 21)
    for s in range(6):
        _check(a, b, a.step(), d.step(), s)


def test_engine_uses_the_traffic_kernel_and_graph_replay_matches():
    """Engine with device traffic, eager vs CUDA-graph replay: identical step outputs."""
    from isaac_net_b200.presets import Motion, workload
    wl = workload(2)
    E, R = 64, 32
    cfg = wl.config()
    outs = []
    for graphs in (False, True):
        eng = ib.make_engine("L2", E, R, "cuda:0", cfg, seed=wl.seed)
        eng.graphs = graphs
        assert eng.dtraffic is not None
        mo = Motion(2, E, R, seed=5, step_ms=cfg.control_step_ms)
        seq = []
        for s in range(12):
            o = eng.step(None, mo.current().to("cuda:0"))
            mo.advance()
            seq.append({k: v.clone() for k, v in o.items() if torch.is_tensor(v)})
        outs.append(seq)
    for s, (x, y) in enumerate(zip(*outs)):
        for k in x:
            assert torch.equal(x[k].nan_to_num(nan=7.0), y[k].nan_to_num(nan=7.0)) if x[k].is_floating_point() \
                else torch.equal(x[k], y[k]), (s, k)
