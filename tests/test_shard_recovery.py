"""Failure detection and recovery of env shards on CPU (gloo ranks running the oracle, no GPU involved).

Two ranks step their shards in lockstep (a barrier after every step, process-group timeout of a few seconds) and
checkpoint their state every few steps.  Rank 1 dies after step 5 (it exits mid-run); rank 0 learns of it at the
next barrier (an error instead of a hang) and exits with a distinct code; the launcher sees both failures, restarts
both ranks from the last checkpoint, and the resumed run's outputs equal one uninterrupted unsharded run bitwise.
"""
import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_shard_gloo import E_SHARD, KEYS, R, SEED, WORLD, _config, _inputs

STEPS, DIE_AFTER, CKPT_EVERY = 8, 5, 3
FAILED_PEER = 17


def _ckpt(o):
    st = {k: v.clone() for k, v in o.reference_state().items()}
    st.update({"eng.T": torch.tensor(o.T), "net.last_g": torch.tensor(-1 if o.last_g is None else o.last_g),
               "eng.last_snr": o.last_snr.clone(), "eng.last_hid": o.last_hid.clone()})
    return st


def _rank(rank, port, root, tmp, resume_from):
    import sys
    sys.path.insert(0, root)
    import importlib
    importlib.import_module("isaac-net_b200")
    from oracle.nr_oracle import OracleEngine
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=5))
    torch.set_num_threads(1)
    cfg = _config()
    o = OracleEngine(cfg, E_SHARD, R, "cpu", seed=SEED, reduce="aten")
    o.set_env_offset(rank * E_SHARD)
    inputs = _inputs(WORLD * E_SHARD, R, STEPS, cfg.slots_per_step)
    sl = slice(rank * E_SHARD, (rank + 1) * E_SHARD)
    start = 0
    if resume_from is not None:
        o.load_reference_state(torch.load(os.path.join(tmp, f"ck{rank}_{resume_from}.pt")))
        start = resume_from + 1
    for t in range(start, STEPS):
        pos, arr = inputs[t]
        out = o.step(pos[sl], {k: v[sl] for k, v in arr.items()})
        torch.save({k: out[k] for k in KEYS}, os.path.join(tmp, f"out{rank}_{t}.pt"))
        if t % CKPT_EVERY == 0:
            torch.save(_ckpt(o), os.path.join(tmp, f"ck{rank}_{t}.pt"))
        if resume_from is None and rank == 1 and t == DIE_AFTER:
            os._exit(3)                          # the rank dies between steps
        try:
            dist.barrier()
        except Exception:
            os._exit(FAILED_PEER)                # a peer is gone: report it instead of waiting
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _launch(root, tmp, resume_from):
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, port, root, tmp, resume_from)) for r in range(WORLD)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    for p in ps:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in ps]


def test_a_dead_rank_is_detected_and_the_run_resumes_from_a_checkpoint(tmp_path):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    codes = _launch(root, str(tmp_path), None)
    assert codes[1] == 3 and codes[0] == FAILED_PEER, codes
    last = max(t for t in range(DIE_AFTER + 1) if t % CKPT_EVERY == 0)
    codes = _launch(root, str(tmp_path), last)
    assert codes == [0, 0], codes
    from oracle.nr_oracle import OracleEngine
    cfg = _config()
    full = OracleEngine(cfg, WORLD * E_SHARD, R, "cpu", seed=SEED, reduce="aten")
    for t, (pos, arr) in enumerate(_inputs(WORLD * E_SHARD, R, STEPS, cfg.slots_per_step)):
        ref = full.step(pos, arr)
        parts = [torch.load(os.path.join(tmp_path, f"out{r}_{t}.pt")) for r in range(WORLD)]
        for k in KEYS:
            a, b = torch.cat([p[k] for p in parts], 0), ref[k]
            if a.is_floating_point():
                ok = torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0))
            else:
                ok = torch.equal(a, b)
            assert ok, (t, k)
