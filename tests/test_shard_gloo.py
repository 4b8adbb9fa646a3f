"""Env sharding on CPU with two gloo ranks (the multi-GPU path of bench.py, without GPUs).

Each rank runs the oracle on its shard of the envs: rows keyed by global env id with the initial reset redone under
them (isaac_net/core/sharded.py:61-77).  With no traffic-model generator every draw is keyed by (seed, global env id,
episode), so the shards, gathered over the process group, must equal one unsharded engine bitwise.  bench.py's
max-over-ranks timing reduction and its shard seeds are checked on the same process group.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E_SHARD, R, STEPS, WORLD, SEED = 4, 16, 4, 2, 5
KEYS = ("newest", "delivered", "queue_len", "queue_bytes", "sinr_db", "delay", "cap")


def _inputs(E_all, R, steps, N):
    g = torch.Generator().manual_seed(11)
    out = []
    for _ in range(steps):
        pos = (torch.rand(E_all, R, 2, generator=g) - 0.5) * 100.0
        valid = torch.rand(E_all, R, 2, generator=g) < 0.4
        slot = torch.randint(0, N, (E_all, R, 2), generator=g)
        key = torch.where(valid, slot, torch.full_like(slot, N)) * 2 + torch.arange(2)
        order = key.argsort(-1)
        valid, slot = valid.gather(-1, order), slot.gather(-1, order)
        nbytes = torch.where(torch.rand(E_all, R, 2, generator=g) < 0.5, 200.0, 1500.0).float()
        arr = {"valid": valid, "nbytes": nbytes, "slot": torch.where(valid, slot, torch.zeros_like(slot)),
               "tag": torch.ones(E_all, R, 2, dtype=torch.long), "prio": torch.zeros(E_all, R, 2, dtype=torch.long),
               "dline": torch.full((E_all, R, 2), float("inf"), dtype=torch.float64),
               "det": torch.zeros(E_all, R, 2, dtype=torch.bool)}
        out.append((pos, arr))
    return out


def _run(orc, inputs, sl):
    res = []
    for pos, arr in inputs:
        o = orc.step(pos[sl], {k: v[sl] for k, v in arr.items()})
        res.append({k: o[k].clone() for k in KEYS})
    return res


def _config():
    import importlib
    presets = importlib.import_module("isaac-net_b200.presets")
    return presets.workload(1).config(traffic=None)


def _worker(rank, port, root, errq):
    try:
        import sys
        sys.path.insert(0, root)
        import importlib
        importlib.import_module("isaac-net_b200")
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
        torch.set_num_threads(1)
        from oracle.nr_oracle import OracleEngine
        import bench
        cfg = _config()
        orc = OracleEngine(cfg, E_SHARD, R, "cpu", seed=bench.shard_seed(SEED, rank, cfg), reduce="aten")
        orc.set_env_offset(rank * E_SHARD)
        inputs = _inputs(WORLD * E_SHARD, R, STEPS, cfg.slots_per_step)
        mine = _run(orc, inputs, slice(rank * E_SHARD, (rank + 1) * E_SHARD))
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            full = OracleEngine(cfg, WORLD * E_SHARD, R, "cpu", seed=SEED, reduce="aten")
            ref = _run(full, inputs, slice(None))
            for t in range(STEPS):
                for k in KEYS:
                    cat = torch.cat([gathered[r][t][k] for r in range(WORLD)], 0)
                    a, b = cat, ref[t][k]
                    if a.is_floating_point():
                        ok = torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0))
                    else:
                        ok = torch.equal(a, b)
                    assert ok, f"step {t}: {k} of the gathered shards differs from the unsharded engine"
        mx = bench.max_over_ranks([float(rank), 10.0 - rank], dist, torch.device("cpu"))
        assert mx == [float(WORLD - 1), 10.0], mx
        _check_stats(rank, cfg)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as ex:  # report to the parent; the other rank ends on the process-group timeout
        errq.put(f"rank {rank}: {type(ex).__name__}: {ex}")
        raise


def _check_stats(rank, cfg):
    """The shard statistics helpers: counters summed over ranks, per-env rows gathered in global env order."""
    import importlib
    import types
    sharded = importlib.import_module("isaac-net_b200.sharded")
    engine = importlib.import_module("isaac-net_b200.engine")
    fake = types.SimpleNamespace(ctr=torch.arange(E_SHARD * 64, dtype=torch.long).view(E_SHARD, 64) * (rank + 1),
                                 prb_avail=100.0 * (rank + 1), config=cfg)
    fake.fold_counters = types.MethodType(engine.NRB200Engine.fold_counters, fake)
    got = sharded.global_counters(fake)["ul"]
    both = sum(torch.arange(E_SHARD * 64, dtype=torch.long).view(E_SHARD, 64) * (r + 1) for r in range(WORLD)).sum(0)
    want = fake.fold_counters(both, 100.0 * sum(r + 1 for r in range(WORLD)))["ul"]
    assert got == want, (got, want)
    rows = torch.full((E_SHARD, 3), float(rank))
    g = sharded.gather_env_rows(rows)
    assert torch.equal(g, torch.cat([torch.full((E_SHARD, 3), float(r)) for r in range(WORLD)]))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shards_over_gloo_equal_one_engine():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, root, errq)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_shard_seeds_follow_the_reference_rule():
    import bench
    cfg = _config()
    assert bench.shard_seed(SEED, 3, cfg) == SEED                      # shard-invariant: one seed
    import importlib
    presets = importlib.import_module("isaac-net_b200.presets")
    cfg2 = presets.workload(2).config()
    assert bench.shard_seed(SEED, 1, cfg2) == (SEED + 0x9E3779B97F4A7C15) % 2 ** 62
