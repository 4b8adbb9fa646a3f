"""Traffic models that run inside the engine step (level "L2"), and the policy's Requests.

The models and their draw order are isaac_net's (isaac_net/core/traffic.py:51-430): every model draws from one
``torch.Generator`` owned by the engine (step draws) and a second one for resets, in exactly the reference's call
order and shapes, so an engine on the same device with the same seed sees the same arrivals as the reference.  The
draws stay torch calls on purpose: the reference's arrival stream is defined by torch's generator (mt19937 on CPU,
Philox on CUDA), and a re-implementation would change it.  Everything downstream of the arrivals (enqueue, the
per-slot arrival gate, the MAC) runs in the B200 kernels.

Opt-in (traffic_rng="counter", no counterpart in the reference): CounterDraws replaces both generators by a
counter-keyed stream, the same models drawing the same number of uniforms in the same order, each uniform a hash of
(seed key, global env id, episode, step count, draw index, robot).  The reference's arrivals depend on how the envs
are split over engines (one generator per engine, isaac_net/core/sharded.py:21-25); these do not, so a batch split
over GPUs sees the arrivals one engine over the whole batch would see.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Callable, Optional, Union

import torch

KINDS = ("periodic", "bursty", "video", "event", "policy")


# ------------------------------------------------------------------ counter-keyed draws (opt-in)
_M32, _C1, _C2, _GOLD = 0xFFFFFFFF, 0x21F0AAAD, 0x735A2D97, 0x9E3779B9
CH_TRAFFIC, CH_TRAFFIC_RESET = 0x54, 0x55     # counter-RNG channels of this stream (step draws, reset draws)


def _mix32(x):
    """lowbias32 on int64 tensors holding 32-bit values (the counter RNG's mixer, proto/rng.py:42-48)."""
    x = x ^ (x >> 16)
    x = (x * _C1) & _M32
    x = x ^ (x >> 15)
    x = (x * _C2) & _M32
    return x ^ (x >> 15)


def _salt(v):
    return (_mix32(v & _M32) + _GOLD) & _M32


def _elem(base, i):
    return _mix32(_mix32((base + i * _GOLD) & _M32) ^ base)


class CounterDraws:
    """The counter-keyed uniforms of traffic_rng="counter".  The key chain is the engine's counter RNG's
    (proto/rng.py:164-185) under channels of its own: key = (s0, env id, episode, channel, counter), uniform d of
    robot r = 53 bits of the element hashes 2r, 2r + 1 of stream d, ((h0 >> 5) 2^26 + (h1 >> 6)) 2^-53, exact in
    float64.  Step draws use the robot's step count as the counter (CH_TRAFFIC), reset draws counter 0
    (CH_TRAFFIC_RESET); env_id / episode are the engine's tensors, read at every call (updated in place by
    set_env_offset and resets)."""

    def __init__(self, s0, env_id, episode, R):
        self.s0, self.env_id, self.episode = int(s0), env_id, episode
        self.r2 = 2 * torch.arange(R, dtype=torch.long, device=env_id.device)
        self.kenv, self.d = None, 0

    def begin(self, channel, ctr):
        """Start the draws of one step (ctr: [E,R] step counts) or one reset (ctr = 0)."""
        env, ep = self.env_id[:, None], self.episode[:, None]
        h = _mix32(self.s0 ^ _salt(env))
        h = _mix32(h ^ _salt(ep))
        h = _mix32(h ^ _salt(torch.full_like(h, channel)))
        ctr = ctr if torch.is_tensor(ctr) else torch.full_like(h, int(ctr))
        self.kenv = _mix32(h ^ _salt(ctr)).expand(-1, self.r2.numel())
        self.d = 0

    def next(self):
        """The next uniform [E,R] (float64, in [0, 1))."""
        base = _mix32(self.kenv ^ _salt(torch.full_like(self.kenv, self.d)))
        self.d += 1
        h0, h1 = _elem(base, self.r2), _elem(base, self.r2 + 1)
        return (h0 >> 5).double() * 2.0 ** -27 + (h1 >> 6).double() * 2.0 ** -53


@dataclass
class Requests:
    """Messages the policy enqueues in one control step (isaac_net/core/proto/netsim.py:163-172).

    send [E,R] long (0 = nothing, c >= 1 = one message of class c), det [E,R] bool, hid [E] long."""
    send: torch.Tensor
    det: Optional[torch.Tensor] = None
    hid: Optional[torch.Tensor] = None


@dataclass(frozen=True)
class TrafficModel:
    """One traffic generator (isaac_net/core/traffic.py:51-176). Build it with the constructors."""
    kind: str
    size_bytes: float = 0.0
    period_ms: float = 0.0
    jitter_ms: float = 0.0
    phase: str = "random"
    rate_hz: float = 0.0
    burst_size: int = 1
    on_off: tuple = (1.0, 0.0)
    gop: Optional[tuple] = None
    trigger: Union[str, Callable, None] = None
    det: bool = False
    robots: Optional[tuple] = None
    tag: Optional[int] = None
    priority: int = 0
    deadline_ms: float = math.inf
    max_msgs_per_step: Optional[int] = None
    direction: str = "ul"

    @staticmethod
    def periodic(size_bytes, period_ms, jitter_ms=0.0, phase="random", **kw):
        assert period_ms > 0 and 0 <= jitter_ms < period_ms and size_bytes > 0
        assert phase in ("random", "aligned")
        return TrafficModel("periodic", size_bytes=float(size_bytes), period_ms=float(period_ms),
                            jitter_ms=float(jitter_ms), phase=phase, **kw)

    @staticmethod
    def bursty(size_bytes, rate_hz, burst_size, on_off=(1.0, 1.0), **kw):
        assert size_bytes > 0 and rate_hz > 0 and burst_size >= 1 and on_off[0] > 0 and on_off[1] >= 0
        return TrafficModel("bursty", size_bytes=float(size_bytes), rate_hz=float(rate_hz),
                            burst_size=int(burst_size), on_off=(float(on_off[0]), float(on_off[1])), **kw)

    @staticmethod
    def video(fps, mean_frame_bytes=None, gop=None, phase="random", jitter_ms=0.0, **kw):
        assert fps > 0 and (mean_frame_bytes is not None or gop is not None)
        if gop is not None:
            i_b, p_b, n = float(gop[0]), float(gop[1]), int(gop[2])
            if mean_frame_bytes is not None:
                s = float(mean_frame_bytes) / ((i_b + (n - 1) * p_b) / n)
                i_b, p_b = i_b * s, p_b * s
            gop = (i_b, p_b, n)
            size = (i_b + (n - 1) * p_b) / n
        else:
            size = float(mean_frame_bytes)
        period = 1000.0 / fps
        assert 0 <= jitter_ms < period and phase in ("random", "aligned")
        return TrafficModel("video", size_bytes=size, period_ms=period, jitter_ms=float(jitter_ms), phase=phase,
                            gop=gop, **kw)

    @staticmethod
    def event(size_bytes, trigger="event", det=False, **kw):
        assert size_bytes > 0
        return TrafficModel("event", size_bytes=float(size_bytes), trigger=trigger, det=bool(det), **kw)

    @staticmethod
    def policy():
        return TrafficModel("policy")

    def on(self, robots):
        if robots is None:
            return replace(self, robots=None)
        if isinstance(robots, int):
            robots = (robots,)
        return replace(self, robots=tuple(int(r) for r in robots))

    def with_(self, **kw):
        return replace(self, **kw)

    @property
    def generates(self):
        return self.kind != "policy"

    def bursts_per_step(self, step_ms):
        if self.max_msgs_per_step is not None:
            return max(1, int(self.max_msgs_per_step) // self.burst_size)
        lam = self.rate_hz * step_ms / 1000.0
        return int(math.ceil(lam + 4 * math.sqrt(lam))) + 1

    def max_per_step(self, step_ms):
        if self.max_msgs_per_step is not None:
            return int(self.max_msgs_per_step)
        if self.kind in ("periodic", "video"):
            return int(math.floor((step_ms + self.jitter_ms) / self.period_ms)) + 1
        if self.kind == "bursty":
            return self.burst_size * self.bursts_per_step(step_ms)
        return 1 if self.kind == "event" else 0


def normalize_traffic(traffic):
    if traffic is None:
        return None
    if isinstance(traffic, TrafficModel):
        traffic = (traffic,)
    traffic = tuple(traffic)
    for m in traffic:
        if not isinstance(m, TrafficModel) or m.kind not in KINDS:
            raise TypeError(f"NRConfig.traffic takes TrafficModel objects, got {m!r}")
        if m.direction not in ("ul", "dl"):
            raise ValueError(f"traffic model {m.kind}: direction must be 'ul' or 'dl', not {m.direction!r}")
        if m.direction == "dl" and (m.kind == "policy" or m.det):
            raise ValueError(f"traffic model {m.kind}: a downlink model cannot be policy() or carry det=True "
                             "(isaac_net/core/traffic.py:189-195)")
    return traffic or None


def generates(traffic, direction="ul"):
    """A model of `direction` ("ul" / "dl"; None = either) that generates messages (traffic.py:199-203)."""
    return traffic is not None and any(m.generates and (direction is None or m.direction == direction)
                                       for m in traffic)


@dataclass
class Arrivals:
    """Messages of one control step [E,R,M], sorted by arrival slot per robot (invalid entries last)."""
    valid: torch.Tensor
    nbytes: torch.Tensor
    slot: torch.Tensor
    tag: torch.Tensor
    prio: torch.Tensor
    dline: torch.Tensor
    det: torch.Tensor


class _Source:
    """Per-robot state of one model [E,R]; draws from the engine's step / reset generators."""

    def __init__(self, model, idx, E, R, dev, step_ms, gens, counter=None):
        self.m, self.E, self.R, self.dev, self.step_ms = model, E, R, dev, step_ms
        self.gens = gens                      # [step generator, reset generator]
        self.counter = counter                # CounterDraws (traffic_rng="counter") or None
        self.width = model.max_per_step(step_ms)
        self.tag = model.tag if model.tag is not None else idx + 1
        on = torch.zeros(R, dtype=torch.bool, device=dev)
        if model.robots is None:
            on[:] = True
        else:
            bad = [r for r in model.robots if not 0 <= r < R]
            if bad:
                raise ValueError(f"traffic model {model.kind}: robots {bad} outside 0..{R - 1}")
            on[list(model.robots)] = True
        self.mask = on[None, :].expand(E, R)
        full = lambda dt, v: torch.full((E, R), v, dtype=dt, device=dev)
        if model.kind in ("periodic", "video"):
            self.nom, self.nxt, self.cnt = full(torch.float64, 0.0), full(torch.float64, 0.0), full(torch.long, 0)
            self.names = ("nom", "nxt", "cnt")
        elif model.kind == "bursty":
            self.on, self.t_tog, self.t_bur = (full(torch.bool, False), full(torch.float64, 0.0),
                                               full(torch.float64, 0.0))
            self.names = ("on", "t_tog", "t_bur")
        else:
            self.names = ()
        self.deferred = torch.zeros((), dtype=torch.long, device=dev)
        self._gen = gens[0]

    def loops(self):
        """Iterations of a bursty model's event loop per step (bursts plus two toggles per ON/OFF period)."""
        md, T = self.m, self.step_ms
        nb = self.width // md.burst_size
        on_ms, off_ms = md.on_off[0] * 1000.0, md.on_off[1] * 1000.0
        loops = nb + 2 * (int(math.ceil(T / max(min(on_ms, off_ms if off_ms > 0 else on_ms), 1e-9))) + 1)
        return min(loops, nb + 64)

    def _u(self):
        if self.counter is not None:
            return self.counter.next()
        return torch.rand(self.E, self.R, generator=self._gen, device=self.dev, dtype=torch.float64)

    def _expo(self, mean_ms):
        return -torch.log1p(-self._u()) * mean_ms

    def _write_back(self, bufs):
        for n, b in bufs.items():          # in place: captured graphs and callers keep the same buffers
            b.copy_(getattr(self, n))
            setattr(self, n, b)

    def reset(self, me):
        bufs = {n: getattr(self, n) for n in self.names}
        self._gen = self.gens[1]
        try:
            m, md = me[:, None], self.m
            if md.kind in ("periodic", "video"):
                nom = self._u() * md.period_ms if md.phase == "random" else torch.zeros_like(self.nom)
                nxt = nom + self._u() * md.jitter_ms
                self.nom = torch.where(m, nom, self.nom)
                self.nxt = torch.where(m, nxt, self.nxt)
                self.cnt = torch.where(m, torch.zeros_like(self.cnt), self.cnt)
            elif md.kind == "bursty":
                on_ms, off_ms = md.on_off[0] * 1000.0, md.on_off[1] * 1000.0
                on = self._u() < on_ms / (on_ms + off_ms)
                a = self._expo(on_ms)
                b = self._expo(off_ms)
                t_tog = torch.where(on, a, b)
                t_bur = self._expo(1000.0 / md.rate_hz)
                if off_ms == 0:
                    t_tog = torch.full_like(t_tog, math.inf)
                self.on = torch.where(m, on, self.on)
                self.t_tog = torch.where(m, t_tog, self.t_tog)
                self.t_bur = torch.where(m, t_bur, self.t_bur)
        finally:
            self._gen = self.gens[0]
        self._write_back(bufs)

    def step(self, clock, trig):
        bufs = {n: getattr(self, n) for n in self.names}
        out = self._draw(clock, trig)
        self._write_back(bufs)
        return out

    def _draw(self, clock, trig):
        md, E, R, W, T = self.m, self.E, self.R, self.width, self.step_ms
        if md.kind in ("periodic", "video"):
            vs, bs, ts = [], [], []
            for _ in range(W):
                hit = (self.nxt < T) & self.mask
                if md.kind == "video" and md.gop is not None:
                    i_b, p_b, n = md.gop
                    size = torch.where(self.cnt % n == 0, torch.full_like(self.nxt, i_b), torch.full_like(self.nxt, p_b))
                else:
                    size = torch.full_like(self.nxt, md.size_bytes)
                vs.append(hit), bs.append(size), ts.append(self.nxt)
                self.cnt = self.cnt + hit.long()
                self.nom = torch.where(hit, self.nom + md.period_ms, self.nom)
                self.nxt = torch.where(hit, self.nom + self._u() * md.jitter_ms, self.nxt)
            self.deferred += ((self.nxt < T) & self.mask).sum()
            self.nom = self.nom - T
            self.nxt = self.nxt - T
            return torch.stack(vs, -1), torch.stack(bs, -1), torch.stack(ts, -1)
        if md.kind == "bursty":
            nb = W // md.burst_size
            on_ms, off_ms = md.on_off[0] * 1000.0, md.on_off[1] * 1000.0
            iat = 1000.0 / md.rate_hz
            loops = self.loops()
            cnt = torch.zeros(E, R, dtype=torch.long, device=self.dev)
            times = torch.full((E, R, nb), math.inf, dtype=torch.float64, device=self.dev)
            slots = torch.arange(nb, device=self.dev)
            for _ in range(loops):
                t_b = torch.where(self.on, self.t_bur, torch.full_like(self.t_bur, math.inf))
                due = self.mask & self.on & (t_b <= self.t_tog) & (t_b < T)
                burst = due & (cnt < nb)
                blocked = due & (cnt >= nb)
                tog = self.mask & ~burst & ~blocked & (self.t_tog < T) & (self.t_tog < t_b)
                times = torch.where((cnt[..., None] == slots) & burst[..., None], t_b[..., None], times)
                cnt = cnt + burst.long()
                self.t_bur = torch.where(burst, self.t_bur + self._expo(iat), self.t_bur)
                now_on = ~self.on
                d_on = self._expo(on_ms)
                d_off = self._expo(off_ms) if off_ms > 0 else torch.full_like(self.t_tog, math.inf)
                new_tog = self.t_tog + torch.where(now_on, d_on, d_off)
                self.t_bur = torch.where(tog & now_on, self.t_tog + self._expo(iat), self.t_bur)
                self.t_tog = torch.where(tog, new_tog, self.t_tog)
                self.on = torch.where(tog, now_on, self.on)
            t_b = torch.where(self.on, self.t_bur, torch.full_like(self.t_bur, math.inf))
            self.deferred += (self.mask & (torch.minimum(t_b, self.t_tog) < T)).sum()
            self.t_bur = self.t_bur - T
            self.t_tog = self.t_tog - T
            valid = torch.isfinite(times).repeat_interleave(md.burst_size, -1)
            t = times.repeat_interleave(md.burst_size, -1)
            return valid, torch.full(valid.shape, md.size_bytes, dtype=torch.float32, device=self.dev), t
        if md.kind == "event":
            if callable(md.trigger):
                mask = md.trigger(clock)
            elif torch.is_tensor(trig):
                mask = trig
            elif isinstance(trig, dict) and md.trigger in trig:
                mask = trig[md.trigger]
            else:
                mask = None
            if mask is None:
                valid = torch.zeros(E, R, dtype=torch.bool, device=self.dev)
            else:
                mask = mask.to(self.dev, torch.bool)
                valid = (mask[:, None].expand(E, R) if mask.dim() == 1 else mask) & self.mask
            z = torch.zeros(E, R, 1, dtype=torch.float64, device=self.dev)
            return valid[..., None], torch.full((E, R, 1), md.size_bytes, dtype=torch.float32, device=self.dev), z
        raise AssertionError(md.kind)


class TrafficGen:
    """All generating uplink models of a config for E envs x R robots; step() -> Arrivals [E,R,M]."""

    def __init__(self, traffic, E, R, device, step_ms, slots_per_step, seed=None, counter=None, direction="ul"):
        """counter: a CounterDraws for the opt-in counter-keyed stream (the generators are then unused); direction:
        the models of that link only ("dl": the downlink's generator, isaac_net/core/traffic.py:373-391)."""
        self.E, self.R, self.dev = E, R, torch.device(device)
        self.counter = counter
        self.calls = torch.zeros(E, R, dtype=torch.long, device=self.dev)   # steps generated (the counter stream's key)
        self.N = int(slots_per_step)
        self.step_ms, self.slot_ms = float(step_ms), float(step_ms) / self.N
        seed = 0 if seed is None else int(seed)
        self.gen = torch.Generator(device=self.dev)
        self.gen.manual_seed(seed)
        self.rgen = torch.Generator(device=self.dev)
        self.rgen.manual_seed((seed + 0x9E3779B97F4A7C15) % 2 ** 63)
        models = normalize_traffic(traffic) or ()
        gens = (self.gen, self.rgen)
        self.sources = [_Source(m, i, E, R, self.dev, self.step_ms, gens, counter)
                        for i, m in enumerate(models) if m.generates and m.direction == direction]
        self.M = sum(s.width for s in self.sources)
        self.reset(None)

    @property
    def deferred(self):
        return sum((s.deferred for s in self.sources), torch.zeros((), dtype=torch.long, device=self.dev))

    def reset(self, env_mask_e=None):
        m = torch.ones(self.E, dtype=torch.bool, device=self.dev) if env_mask_e is None else env_mask_e
        if self.counter is not None:
            self.counter.begin(CH_TRAFFIC_RESET, 0)
        for s in self.sources:
            s.reset(m)
        if env_mask_e is None:
            for s in self.sources:
                s.deferred.zero_()

    def step(self, clock=None, triggers=None) -> Arrivals:
        E, R, d = self.E, self.R, self.dev
        cols = {k: [] for k in ("v", "b", "t", "tag", "prio", "dl", "det")}
        if self.counter is not None:
            self.counter.begin(CH_TRAFFIC, self.calls)
        self.calls += 1
        for s in self.sources:
            v, b, t = s.step(clock, triggers)
            k = v.shape[-1]
            cols["v"].append(v), cols["b"].append(b.float()), cols["t"].append(t)
            cols["tag"].append(torch.full((E, R, k), s.tag, dtype=torch.long, device=d))
            cols["prio"].append(torch.full((E, R, k), s.m.priority, dtype=torch.long, device=d))
            cols["dl"].append(torch.full((E, R, k), s.m.deadline_ms, dtype=torch.float64, device=d))
            cols["det"].append(torch.full((E, R, k), s.m.det, dtype=torch.bool, device=d))
        if not cols["v"]:
            z = torch.zeros(E, R, 0, device=d)
            return Arrivals(z.bool(), z.float(), z.long(), z.long(), z.long(), z.double(), z.bool())
        valid, nbytes, t = torch.cat(cols["v"], -1), torch.cat(cols["b"], -1), torch.cat(cols["t"], -1)
        t = torch.where(valid, t, torch.zeros_like(t))
        slot = torch.floor(t.clamp(min=0) / self.slot_ms).long().clamp(0, self.N - 1)
        M = valid.shape[-1]
        key = torch.where(valid, slot, torch.full_like(slot, self.N)) * M + torch.arange(M, device=d)
        order = key.argsort(-1)
        g = lambda x: x.gather(-1, order)
        return Arrivals(g(valid), g(nbytes), g(slot), g(torch.cat(cols["tag"], -1)), g(torch.cat(cols["prio"], -1)),
                        g(torch.cat(cols["dl"], -1)), g(torch.cat(cols["det"], -1)))


class DeviceTrafficGen:
    """TrafficGen.step as one kernel (inb_traffic_step) for periodic, video and bursty models.

    The kernel reproduces the torch.Generator stream TrafficGen.step would consume: it owns the step generator's
    position from construction on (a per-robot step counter on the device, so captured CUDA graphs replay
    correctly) and leaves the torch generator object untouched; resets keep running TrafficGen.reset on the reset
    generator.  The model state buffers are TrafficGen's own (updated in place by both)."""

    KINDS = {"periodic": 0, "video": 1, "bursty": 2}

    @classmethod
    def supports(cls, tg):
        from . import _native as nat
        return (tg is not None and 0 < len(tg.sources) <= nat.MAX_SRC and 0 < tg.M <= 64
                and all(s.m.kind in cls.KINDS for s in tg.sources) and tg.dev.type == "cuda")

    def __init__(self, tg, lib):
        from . import _native as nat
        self.nat, self.L, self.tg = nat, lib, tg
        E, R, M, d = tg.E, tg.R, tg.M, tg.dev
        numel = E * R
        props = torch.cuda.get_device_properties(d)
        # torch's launch for a float64 uniform fill of numel elements (ATen DistributionTemplates.h): 256-thread
        # blocks, at most (threads per SM / 256) blocks per SM, two doubles per curand_uniform2_double call
        blocks = min((numel + 255) // 256, props.multi_processor_count * (props.max_threads_per_multi_processor // 256))
        stride = 256 * blocks
        a = nat.InbTrafficArgs()
        a.E, a.R, a.M, a.N, a.n_src = E, R, M, tg.N, len(tg.sources)
        a.seed, a.off0 = tg.gen.initial_seed(), tg.gen.get_offset()
        a.stride, a.inc = stride, ((numel - 1) // (stride * 2) + 1) * 4
        if tg.counter is not None:   # the counter-keyed stream: keys from the engine's env ids and episodes
            a.counter, a.s0 = 1, tg.counter.s0
            a.env_id, a.episode = tg.counter.env_id.data_ptr(), tg.counter.episode.data_ptr()
        a.step_ms, a.inv_slot_ms = tg.step_ms, 1.0 / tg.slot_ms
        self._keep = []
        col, nd = 0, 0
        for k, s in enumerate(tg.sources):
            m, c = s.m, a.src[k]
            c.kind, c.width, c.col = self.KINDS[m.kind], s.width, col
            c.det, c.tag, c.prio, c.dline, c.size = int(m.det), int(s.tag), int(m.priority), float(m.deadline_ms), \
                float(m.size_bytes)
            mask = s.mask[0].to(torch.uint8).contiguous()
            self._keep.append(mask)
            c.mask, c.deferred = mask.data_ptr(), s.deferred.data_ptr()
            if m.kind in ("periodic", "video"):
                c.period, c.jitter = m.period_ms, m.jitter_ms
                if m.kind == "video" and m.gop is not None:
                    c.gop_i, c.gop_p, c.gop_n = float(m.gop[0]), float(m.gop[1]), int(m.gop[2])
                c.nom, c.nxt, c.cnt = s.nom.data_ptr(), s.nxt.data_ptr(), s.cnt.data_ptr()
                nd += s.width
            else:
                c.nb, c.burst, c.loops = s.width // m.burst_size, m.burst_size, s.loops()
                c.on_ms, c.off_ms, c.iat = m.on_off[0] * 1000.0, m.on_off[1] * 1000.0, 1000.0 / m.rate_hz
                assert s.on.dtype == torch.bool and s.on.element_size() == 1
                c.on, c.t_tog, c.t_bur = s.on.data_ptr(), s.t_tog.data_ptr(), s.t_bur.data_ptr()
                nd += c.loops * (4 if c.off_ms > 0 else 3)
            col += s.width
        a.ndraws = nd
        # steps generated: the torch stream's position (from construction on), or the counter stream's key (shared
        # with the host TrafficGen, whose resets and host steps use the same count)
        self.calls = tg.calls if tg.counter is not None else torch.zeros(E, R, dtype=torch.long, device=d)
        a.calls = self.calls.data_ptr()
        z = lambda dt: torch.zeros(E, R, M, dtype=dt, device=d)
        self.out = Arrivals(valid=z(torch.bool), nbytes=z(torch.float32), slot=z(torch.long), tag=z(torch.long),
                            prio=z(torch.long), dline=z(torch.float64), det=z(torch.bool))
        for n in nat.TRAFFIC_OUT:
            setattr(a, n, getattr(self.out, n).data_ptr())
        self.args = a

    def step(self):
        """Arrivals of the next step, written into the same [E,R,M] buffers every step (views returned)."""
        import ctypes
        st = torch.cuda.current_stream(self.tg.dev).cuda_stream
        self.nat.check(self.L.inb_traffic_step(ctypes.byref(self.args), ctypes.c_void_p(st)), "inb_traffic_step")
        return self.out


__all__ = ["Requests", "TrafficModel", "TrafficGen", "DeviceTrafficGen", "CounterDraws", "Arrivals",
           "normalize_traffic", "generates"]
