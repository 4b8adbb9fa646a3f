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


@pytest.mark.parametrize("mix,E,R,steps", [("cfg2", 256, 32, 40), ("mixed", 37, 24, 50)])
def test_counter_stream_kernel_equals_host(mix, E, R, steps):
    """traffic_rng="counter": the kernel's counter-keyed uniforms and the host TrafficGen's (CounterDraws, torch
    integer ops) give bitwise the same arrivals and model state, partial resets included (episodes advanced as an
    engine advances them)."""
    dev = torch.device("cuda:0")
    env = torch.arange(E, dtype=torch.long, device=dev) + 1000
    ep_a = torch.zeros(E, dtype=torch.long, device=dev)
    ep_b = ep_a.clone()
    a = tr.TrafficGen(MIXES[mix], E, R, dev, 5.0, 10, seed=3, counter=tr.CounterDraws(77, env, ep_a, R))
    b = tr.TrafficGen(MIXES[mix], E, R, dev, 5.0, 10, seed=3, counter=tr.CounterDraws(77, env, ep_b, R))
    d = tr.DeviceTrafficGen(b, nat.lib())
    for s in range(steps):
        if s == steps // 2:
            m = torch.zeros(E, dtype=torch.bool, device=dev)
            m[::3] = True
            a.reset(m)
            b.reset(m)
            ep_a += m.long()
            ep_b += m.long()
        _check(a, b, a.step(), d.step(), s)


@pytest.mark.parametrize("wl_i", (1, 2))
def test_counter_stream_two_shards_equal_one_engine(wl_i):
    """Engines with traffic_rng="counter": one engine over 8 envs and two shards of 4 (the second keyed by global env
    ids 4..7 through set_env_offset, the same seed) give bitwise the same step outputs, a partial reset included;
    with the reference's generator stream the shards' arrivals differ."""
    from isaac_net_b200.presets import Motion, workload
    wl = workload(wl_i)
    cfg = wl.config()
    E, R, dev = 8, wl.R, torch.device("cuda:0")
    full = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed, traffic_rng="counter")
    sh = [ib.make_engine("L2", E // 2, R, dev, cfg, seed=wl.seed, traffic_rng="counter") for _ in range(2)]
    sh[1].set_env_offset(E // 2)
    mo = Motion(wl_i, E, R, seed=9, step_ms=cfg.control_step_ms)
    delivered = 0
    for s in range(10):
        if s == 5:
            full.reset([1, 6])
            sh[0].reset([1])
            sh[1].reset([2])
        pos = mo.current().to(dev)
        o = full.step(None, pos)
        parts = [x.step(None, pos[i * (E // 2):(i + 1) * (E // 2)]) for i, x in enumerate(sh)]
        for k, v in o.items():
            if not torch.is_tensor(v) or v.dim() == 0:
                continue
            w = torch.cat([p[k] for p in parts])
            same = torch.equal(v.nan_to_num(nan=7.0), w.nan_to_num(nan=7.0)) if v.is_floating_point() \
                else torch.equal(v, w)
            assert same, (s, k)
        delivered += int(o["delivered"].sum())
        mo.advance()
    assert delivered > 0
    # the reference's stream: the second shard's arrivals are not the whole batch's rows 4..7
    gf = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    gs = ib.make_engine("L2", E // 2, R, dev, cfg, seed=wl.seed)
    gs.set_env_offset(E // 2)
    x, y = gf.dtraffic.step(), gs.dtraffic.step()
    assert not (torch.equal(x.valid[E // 2:], y.valid) and torch.equal(x.slot[E // 2:], y.slot))
