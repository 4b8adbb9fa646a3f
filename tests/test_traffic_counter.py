"""The opt-in counter-keyed traffic stream (traffic_rng="counter") on the host: shard invariance, and its uniforms
pinned against a scalar restatement of the key chain.

The reference draws every traffic uniform from one torch.Generator per engine, so a batch split over several engines
sees other arrivals than one engine over the whole batch (isaac_net/core/sharded.py:21-25).  The counter stream keys
each uniform by (seed key, global env id, episode, step count, draw index, robot) instead; the models, their draw
order and the float64 arithmetic are unchanged."""
import importlib

import torch

tr = importlib.import_module("isaac-net_b200.traffic")
eng = importlib.import_module("isaac-net_b200.engine")
TM = tr.TrafficModel
ARR = ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")
MIX = (TM.periodic(200, period_ms=3.0, jitter_ms=1.0).on(range(0, 6)),
       TM.video(30, gop=(8000, 1000, 10), jitter_ms=2.0).on(range(4, 12)),
       TM.bursty(1000, rate_hz=400, burst_size=2, on_off=(0.02, 0.01), tag=7, det=True).on(range(6, 16)),
       TM.bursty(300, rate_hz=50, burst_size=1, on_off=(0.5, 0.0), deadline_ms=20.0))


def _gen(ids, R, s0=0x1234567, seed=5):
    env = torch.as_tensor(ids, dtype=torch.long)
    ep = torch.zeros(len(ids), dtype=torch.long)
    g = tr.TrafficGen(MIX, len(ids), R, "cpu", 5.0, 10, seed=seed,
                      counter=tr.CounterDraws(s0, env, ep, R))
    return g, ep


def test_two_shards_equal_one_engine():
    E, R, half = 6, 16, 3
    full, ep_f = _gen(range(E), R)
    a, ep_a = _gen(range(half), R, seed=11)          # the generator seeds play no part in the counter stream
    b, ep_b = _gen(range(half, E), R, seed=12)
    for s in range(14):
        if s == 7:     # reset env 1 and env 4 (an engine resets its traffic, then advances the episode)
            m = torch.zeros(E, dtype=torch.bool)
            m[[1, 4]] = True
            full.reset(m)
            a.reset(m[:half])
            b.reset(m[half:])
            for ep, mm in ((ep_f, m), (ep_a, m[:half]), (ep_b, m[half:])):
                ep += mm.long()
        x, y, z = full.step(), a.step(), b.step()
        for k in ARR:
            assert torch.equal(getattr(x, k), torch.cat([getattr(y, k), getattr(z, k)])), (s, k)
    assert int(full.step().valid.sum()) > 0


def test_generator_stream_is_not_shard_invariant():
    """The reference's stream, for contrast: the same split gives other arrivals."""
    E, R, half = 6, 16, 3
    full = tr.TrafficGen(MIX, E, R, "cpu", 5.0, 10, seed=5)
    a = tr.TrafficGen(MIX, half, R, "cpu", 5.0, 10, seed=5)
    same = True
    for _ in range(4):
        x, y = full.step(), a.step()
        same &= torch.equal(x.valid[:half], y.valid) and torch.equal(x.slot[:half], y.slot)
    assert not same


def test_counter_uniforms_match_a_scalar_key_chain():
    """CounterDraws against the key chain written out on python integers (the engine's _mix32, proto/rng.py:42-60):
    key = mix over (s0, env, episode, channel, counter), stream d, elements 2r and 2r + 1, 53-bit uniform."""
    M32, GOLD = 0xFFFFFFFF, 0x9E3779B9
    mix = eng._mix32
    salt = lambda v: (mix(v & M32) + GOLD) & M32
    elem = lambda base, i: mix(mix((base + i * GOLD) & M32) ^ base)
    s0, envs, eps, R = 0x9ABCDEF1, [7, 123456], [0, 3], 5
    cd = tr.CounterDraws(s0, torch.tensor(envs), torch.tensor(eps), R)
    ctr = torch.tensor([[41] * R, [42] * R])
    cd.begin(tr.CH_TRAFFIC, ctr)
    draws = [cd.next() for _ in range(3)]
    for d in range(3):
        for e in range(2):
            h = mix(s0 ^ salt(envs[e]))
            h = mix(h ^ salt(eps[e]))
            h = mix(h ^ salt(tr.CH_TRAFFIC))
            kenv = mix(h ^ salt(41 + e))
            base = mix(kenv ^ salt(d))
            for r in range(R):
                h0, h1 = elem(base, 2 * r), elem(base, 2 * r + 1)
                u = ((h0 >> 5) * 2 ** 26 + (h1 >> 6)) / 2.0 ** 53
                assert float(draws[d][e, r]) == u, (d, e, r)
    big = tr.CounterDraws(s0, torch.arange(256), torch.zeros(256, dtype=torch.long), 64)
    big.begin(tr.CH_TRAFFIC, 0)
    u = big.next()
    assert float(u.min()) >= 0.0 and float(u.max()) < 1.0 and abs(float(u.mean()) - 0.5) < 0.01
