"""A batch of envs split over several GPUs: the in-process ShardedEngine, and statistics over env shards held by
several processes (one GPU each).

In one process (isaac_net/core/sharded.py:80-191, the reference's ShardedEngine API):

  net = ShardedEngine("L2", E, R, ["cuda:0", "cuda:1"], cfg, seed=0, traffic_rng="counter")
  out = net.step(None, poses)           # poses [E,R,2]; every output concatenated on devices[0], global env order
  net.reset(done_ids)                   # global env ids (or a bool mask [E], or None); each shard resets its own

Shard i is an NRB200Engine over the contiguous global envs offsets[i] .. offsets[i] + split[i] - 1 on devices[i]
(a device may repeat), its counter-RNG rows keyed by global env id (NRB200Engine.set_env_offset).  A step launches
every shard's kernels from this thread without synchronizing, so shards on different GPUs run at the same time.

Across processes, the step itself has no collective: envs are independent and every rank steps its own shard (global
env ids through NRB200Engine.set_env_offset, as isaac_net/core/sharded.py:61-77).  What crosses ranks is bookkeeping,
done between steps or at the end of an episode, over torch.distributed (NCCL over NVLink on GPU ranks, gloo on CPU):

  global_counters(engine)       counters() of the whole batch: one all_reduce of the summed counter words and the
                                PRBs offered
  gather_env_rows(t)            a per-env tensor [E_shard, ...] of every rank, concatenated in global env order on
                                every rank (one all_gather; shards must be equal-sized, as bench.py makes them)

The reference's ShardedEngine concatenates every step's outputs on its first device (sharded.py:130-140); these
helpers are the opt-in, per-episode form of that and are never part of a timed step.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist

from .traffic import generates

# the reference's step between derived shard seeds (isaac_net/core/sharded.py:103)
SEED_STEP = 0x9E3779B97F4A7C15


def global_counters(engine, group=None):
    """engine.counters() summed over every rank of the process group (every rank gets the result)."""
    c = engine.ctr.sum(0).to(torch.float64)
    v = torch.cat([c, torch.tensor([float(engine.prb_avail)], dtype=torch.float64, device=c.device)])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(v, op=dist.ReduceOp.SUM, group=group)
    return engine.fold_counters(v[:-1].round().long(), float(v[-1]))


def gather_env_rows(t, group=None):
    """[E_shard, ...] on every rank -> [world * E_shard, ...] in rank (global env id) order, on every rank."""
    if not (dist.is_available() and dist.is_initialized()):
        return t.clone()
    world = dist.get_world_size(group)
    out = torch.empty((world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out




def shard_invariant(level, cfg, traffic_rng="generator"):
    """True when every draw of an env is keyed by (seed, global env id, episode), so shards that share the seed equal
    one engine over the whole batch bitwise (isaac_net/core/sharded.py:44-58): level "L2" (the only level here; its
    radio, fading, BLER and reset draws are counter-keyed) with no traffic model that generates messages, or with the
    counter-keyed traffic stream (traffic_rng="counter"), whose arrivals are keyed the same way."""
    if level != "L2" or getattr(cfg, "rng", "engine") != "engine":
        return False
    return traffic_rng == "counter" or not generates(cfg.traffic, None)


def shard_seed(seed, i, cfg, traffic_rng="generator", level="L2"):
    """Seed of shard i: the common seed when the shards are shard-invariant, else (seed + i * SEED_STEP) mod 2^62,
    the reference's derived seeds (sharded.py:103), so the shards' traffic generators draw independent streams."""
    if shard_invariant(level, cfg, traffic_rng):
        return int(seed)
    return (int(seed) + i * SEED_STEP) % 2 ** 62


def _make(level, E, R, device, cfg, backend, **kw):
    from .engine import make_engine
    return make_engine(level, E, R, device, cfg, backend, **kw)


class ShardedEngine:
    """E envs split over `devices` behind the contract API of one engine (isaac_net/core/sharded.py:80-191).

    split: envs per shard (default: near-equal, the first E % n shards one larger).  Seeds follow shard_seed: shared
    when shard_invariant (then the sharded engine equals one NRB200Engine over all E envs bitwise), derived per shard
    otherwise.  Inputs whose first dimension is E are cut into the shards' rows and moved to their devices (host
    poses stay on the host: each shard copies its rows on its own input stream); step outputs are concatenated on
    devices[0].  fetch= {key: host tensor [E, ...]} hands every shard the rows of those host tensors it fills;
    sync_fetch() waits for all of them.  Per-shard engines are in `shards`."""

    def __init__(self, level, E, R, devices, config=None, backend="b200", *, seed=None, split=None,
                 traffic_rng="generator", **kw):
        from .config import NRConfig
        devices = [torch.device(d) for d in devices]
        n = len(devices)
        if n < 1:
            raise ValueError("ShardedEngine needs at least one device")
        if split is None:
            split = [E // n + (1 if i < E % n else 0) for i in range(n)]
        split = [int(v) for v in split]
        if len(split) != n or sum(split) != E or min(split) < 1:
            raise ValueError(f"split {split}: one positive env count per device, summing to E={E}")
        cfg = config if config is not None else NRConfig()
        if seed is None:
            seed = cfg.seed if cfg.seed is not None else int(torch.randint(0, 2 ** 62, ()).item())
        self.level, self.E, self.R, self.config = level, int(E), int(R), cfg
        self.devices, self.split, self.dev = devices, split, devices[0]
        self.offsets = [sum(split[:i]) for i in range(n)]
        self.traffic_rng = traffic_rng
        self.shard_invariant = shard_invariant(level, cfg, traffic_rng)
        self.seed = int(seed)
        self.shards = []
        for i, (d, e) in enumerate(zip(devices, split)):
            eng = _make(level, e, R, d, cfg, backend, seed=shard_seed(seed, i, cfg, traffic_rng, level),
                        traffic_rng=traffic_rng, **kw)
            eng.set_env_offset(self.offsets[i])
            self.shards.append(eng)
        self.shard_of = torch.repeat_interleave(torch.arange(n), torch.tensor(split)).to(self.dev)
        self.local_of = torch.cat([torch.arange(e) for e in split]).to(self.dev)

    # ------------------------------------------------------------------ global env id <-> (shard, local id)
    def locate(self, env_id):
        """(shard index, local env id) of global env env_id."""
        e = int(env_id)
        for i, (o, n) in enumerate(zip(self.offsets, self.split)):
            if o <= e < o + n:
                return i, e - o
        raise IndexError(f"env {env_id} is outside 0..{self.E - 1}")

    def _part(self, x, i, move=True):
        """Shard i's rows of x: a tensor whose first dimension is E is sliced (and moved to the shard's device unless
        move=False); dataclasses (Requests, Arrivals) and dicts are cut field by field; anything else passes."""
        if torch.is_tensor(x):
            if x.dim() >= 1 and x.shape[0] == self.E:
                o = self.offsets[i]
                x = x[o:o + self.split[i]]
                return x.to(self.devices[i], non_blocking=True) if move else x
            return x
        if dataclasses.is_dataclass(x) and not isinstance(x, type):
            return dataclasses.replace(x, **{f.name: self._part(getattr(x, f.name), i, move)
                                             for f in dataclasses.fields(x) if f.init})
        if isinstance(x, dict):
            return {k: self._part(v, i, move) for k, v in x.items()}
        return x

    def _gather(self, parts):
        """Per-shard results -> one result on devices[0]: tensors concatenated along the env axis (0-dim tensors:
        shard 0's), dicts and tuples element by element, anything else shard 0's."""
        p0 = parts[0]
        if torch.is_tensor(p0):
            if p0.dim() == 0:
                return p0.to(self.dev)
            return torch.cat([p.to(self.dev, non_blocking=True) for p in parts], 0)
        if isinstance(p0, dict):
            return {k: self._gather([p[k] for p in parts]) for k in p0}
        if isinstance(p0, tuple):
            return tuple(self._gather(list(z)) for z in zip(*parts))
        return p0

    def _each(self, name, *args, **kw):
        return [getattr(s, name)(*(self._part(a, i) for a in args), **{k: self._part(v, i) for k, v in kw.items()})
                for i, s in enumerate(self.shards)]

    # ------------------------------------------------------------------ contract API
    @property
    def clock(self):
        return self._gather([s.clock for s in self.shards])

    def reset(self, env_ids=None):
        """Re-initialize global envs env_ids (None: all; an index list / tensor or a bool mask [E])."""
        if env_ids is None or (isinstance(env_ids, slice) and env_ids == slice(None)):
            for s in self.shards:
                s.reset(None)
            return
        if torch.is_tensor(env_ids) and env_ids.dtype == torch.bool:
            m = env_ids.reshape(-1).to(self.dev)
            if m.numel() != self.E:
                raise ValueError(f"reset mask of {m.numel()} envs, expected {self.E}")
        else:
            m = torch.zeros(self.E, dtype=torch.bool, device=self.dev)
            ids = torch.as_tensor(env_ids if torch.is_tensor(env_ids) else list(env_ids), dtype=torch.long)
            m[ids.reshape(-1).to(self.dev)] = True
        for i, s in enumerate(self.shards):
            s.reset(self._part(m, i))

    def submit(self, t, requests, snr_db=None, **kw):
        return self._gather(self._each("submit", t, requests, snr_db, **kw))

    def add_frames(self, t, send, det, hid, snr_db):
        self._each("add_frames", t, send, det, hid, snr_db)

    def add_dl_frames(self, t, nbytes, cls=None):
        self._each("add_dl_frames", t, nbytes, cls)

    def step(self, t=None, x=None, cur_hid=None, *, fetch=None, **kw):
        """Advance every shard [t, t+1) and return the whole batch's step dict on devices[0] (or (newest, det_env) in
        the legacy form step(t, snr, cur_hid))."""
        outs = []
        for i, s in enumerate(self.shards):
            host_poses = torch.is_tensor(x) and x.device.type == "cpu" and x.dim() == 3
            xi = self._part(x, i, move=not host_poses)
            kwi = {k: self._part(v, i) for k, v in kw.items()}
            if fetch:
                kwi["fetch"] = {k: self._part(v, i, move=False) for k, v in fetch.items()}
            if cur_hid is None:
                outs.append(s.step(t, xi, **kwi))
            else:
                outs.append(s.step(t, xi, self._part(cur_hid, i), **kwi))
        return self._gather(outs)

    def sync_fetch(self):
        """Block the host until every shard's fetch= copies of the last step are complete."""
        for s in self.shards:
            s.sync_fetch()

    def output_schema(self):
        """{key: {"shape", "dtype"}} of the keys step() returns, for the whole batch of E envs."""
        out = {}
        for k, v in self.shards[0].output_schema().items():
            out[k] = dict(v, shape=(self.E, *tuple(v["shape"])[1:]))
        return out

    def queued(self):
        return self._gather([s.queued() for s in self.shards])

    def counters(self):
        """counters() of the whole batch: every shard's totals summed (per-robot lists element by element)."""
        def add(a, b):
            if isinstance(a, dict):
                return {k: add(v, b[k]) for k, v in a.items()}
            if isinstance(a, list):
                return [x + y for x, y in zip(a, b)]
            return a + b
        tot = None
        for s in self.shards:
            c = s.counters()
            tot = c if tot is None else add(tot, c)
        return tot

    # ------------------------------------------------------------------ checkpoints: shard i under "shards[i]."
    def _prefixed(self, per_shard):
        out = {"meta.level": self.level, "meta.E": self.E, "meta.R": self.R, "meta.split": list(self.split)}
        for i, sd in enumerate(per_shard):
            out.update({f"shards[{i}].{k}": v for k, v in sd.items()})
        return out

    def _split_keys(self, sd):
        for k, want in (("meta.E", self.E), ("meta.R", self.R), ("meta.split", list(self.split))):
            if k in sd and sd[k] != want:
                raise ValueError(f"checkpoint {k} = {sd[k]}, this ShardedEngine has {want}")
        parts = [{} for _ in self.shards]
        rest = []
        for k, v in sd.items():
            if k.startswith("shards["):
                i, _, key = k[len("shards["):].partition("].")
                if i.isdigit() and int(i) < len(parts) and key:
                    parts[int(i)][key] = v
                    continue
            rest.append(k)
        return parts, rest

    def state_dict(self):
        """Every shard's state_dict() under "shards[i].<key>", with the batch's E, R and split."""
        return self._prefixed([s.state_dict() for s in self.shards])

    def load_state_dict(self, sd, strict=True):
        """Restore a state_dict() of a ShardedEngine with the same E, R and split (each shard in place)."""
        parts, _ = self._split_keys(sd)
        for s, p in zip(self.shards, parts):
            s.load_state_dict(p, strict=strict)
        return self

    def save(self, path, extra=None):
        torch.save({"format": 1, "state": self.state_dict(), "extra": extra}, path)

    def load(self, path, strict=True):
        d = torch.load(path, map_location="cpu", weights_only=False)
        self.load_state_dict(d["state"], strict=strict)
        return d.get("extra")

    def reference_checkpoint(self):
        """The batch's state under the keys of the reference ShardedEngine's state_dict(): shard i's reference
        engine keys under "shards[i]." (isaac_net/core/checkpoint.py names list elements "[i]")."""
        return self._prefixed([s.reference_checkpoint() for s in self.shards])

    def load_reference_checkpoint(self, sd, strict=False):
        """Continue from a checkpoint a reference ShardedEngine of the same split wrote; returns the keys not used."""
        parts, rest = self._split_keys(sd)
        unused = [k for k in rest if not k.startswith("meta.")]
        for i, (s, p) in enumerate(zip(self.shards, parts)):
            unused += [f"shards[{i}].{k}" for k in (s.load_reference_checkpoint(p, strict=strict) or ())]
        return unused

    def __getattr__(self, name):
        if name == "shards":
            raise AttributeError(name)
        raise AttributeError(f"ShardedEngine has no attribute {name!r}; per-shard state is in .shards[i]")


__all__ = ["ShardedEngine", "shard_invariant", "shard_seed", "global_counters", "gather_env_rows"]
