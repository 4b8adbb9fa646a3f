"""Benchmark of the B200 NR uplink engine: env-steps/s (envs x control steps per second).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload 4]
                    [--scaling strong|weak]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N ...

One step = one control step of the engine over its whole batch, through the public API (engine.step), replayed as a
CUDA graph of 5 launches: the control words (inb_store2), traffic arrivals (traffic.cu), AR(1) fading (nr_fading.cu),
the MAC kernel (enqueue and arrival gate, radio, the K = 10 slots; nr_step.cuh) and the frame-parallel finish
(nr_finish.cu), which writes the step dict into a fresh output block.  The default workload is BASELINE config 4, the
largest (65536 envs x 128 robots, 100 MHz / 18 RBGs, 16 HARQ processes, PF, mixed periodic + Poisson traffic), split
evenly over the N GPUs ("scaling": "strong": 65536 envs on one GPU, 8192 per GPU at N = 8); every rank steps its own
contiguous env shard (global env ids rank * E + i, no collective inside the step).  --scaling weak runs the
workload's per-GPU batch on every rank instead (config 4: 8192 envs per GPU); --workload 1-5 picks another config.

  value   env-steps/s with the poses already resident in HBM, K steps between a barrier + synchronize pair, timed
          with CUDA events, max over ranks;
  e2e     the same through the public API from pinned host memory: every step copies its poses host -> device and
          reads the per-robot observations (newest, queue_len, queue_bytes, sinr_db) back device -> host
          (engine.step(None, host_poses, fetch=host_buffers): the engine runs both copies on its own streams,
          overlapped with the kernels of the neighbouring steps; the timed region ends after the last copy);
  roofline  algorithmic bytes of one step (every per-robot state field read and written once at the reference's
          widths, the step-dict outputs and the pose input: 6680 B per robot for config 4) / the average duration of
          the step's four kernels (traffic, fading, MAC, finish: CUDA events around them on their stream, eager
          launches), against the measured HBM copy bandwidth; traffic = DRAM bytes of those four kernels per step
          from an ncu capture (profiles/nr_step_traffic.json);
  cpu_baseline  the oracle port (oracle/nr_oracle.py, torch on the host cores, the reference's own op sequence) on a
          bounded sample of the same workload: the median of 3 windows, at the workload's full E where the oracle
          steps it in seconds (configs 1, 2), else on a stated reduced E (256 envs).
The state of one step is several GB (config 4: ~2.8 KB per robot), larger than the 126 MB L2, so no L2 flush is
needed between steps.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def b_env(cfg, R):
    """Algorithmic bytes per env-step (reference widths): per-robot state read + written once, outputs, pose."""
    S, P, F, C = cfg.n_subbands, cfg.n_harq, cfg.frame_buffer, cfg.n_cells
    tr = 1 if cfg.traffic else 0
    mc = 1 if C > 1 else 0
    per = 2 * (56 + 4 * S + 8 * C * S + 76 * P + 50 * F + 32 * F * tr + 40 * mc) + (23 * F + 32) + \
        (41 * F + 16) * tr + 8
    return R * per + 16 * C * S * mc


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, None

    def start(self):
        """Start sampling every 50 ms into a temporary file and wait (up to 3 s) for the first sample, so that even a
        short timed region is covered."""
        try:
            fd, self.path = tempfile.mkstemp(prefix="inb_clocks_", suffix=".csv")
            self.f = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 3.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                break
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx = float(c[2])
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n):
    if int(os.environ.get("WORLD_SIZE", "1")) <= 1:
        return 0, 1, None
    import datetime
    import torch.distributed as dist
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return rank, dist.get_world_size(), dist


def cpu_baseline(wl, cfg, E_sample, steps, warm=1, windows=3):
    """The oracle port (reference op sequence, torch on the host cores) on E_sample envs of the workload: `warm`
    untimed steps, then `windows` windows of `steps` steps each; the value is the median window's env-steps/s."""
    from oracle.nr_oracle import OracleEngine
    tr = importlib.import_module("isaac-net_b200.traffic")
    presets = importlib.import_module("isaac-net_b200.presets")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    E, R = E_sample, wl.R
    o = OracleEngine(cfg, E, R, "cpu", seed=wl.seed, reduce="aten")
    tseed = (int(wl.seed) * 6364136223846793005 + 1442695040888963407) % 2 ** 62
    gen = tr.TrafficGen(cfg.traffic, E, R, "cpu", cfg.control_step_ms, cfg.slots_per_step, seed=tseed) \
        if cfg.traffic else None
    mot = presets.Motion(wl_id(wl), E, R, seed=wl.seed, step_ms=cfg.control_step_ms)
    pos = mot.current()

    def one():
        nonlocal pos
        arr = None
        if gen is not None:
            a = gen.step(o.T - o.epoch, None)
            arr = {k: getattr(a, k) for k in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")}
        o.step(pos, arr)
        pos = mot.advance()
    for _ in range(warm):
        one()
    rates = []
    for _ in range(windows):
        t0 = time.perf_counter()
        for _ in range(steps):
            one()
        rates.append(E * steps / (time.perf_counter() - t0))
    reduced = "" if E == wl.E else f" (reduced E: {E} of the workload's {wl.E} envs)"
    return {"value": statistics.median(rates), "unit": "env-steps/s", "cores": threads, "kind": "port",
            "windows": rates,
            "sample": f"oracle port (torch CPU, reference op order) on {E} envs x {R} robots{reduced}, "
                      f"{warm} warm-up step(s), then the median of {windows} windows of {steps} control steps"}


def wl_id(wl):
    return int(wl.name[3])


def shard_seed(seed, rank, cfg, traffic_rng="generator"):
    """Seed of shard `rank` (isaac_net/core/sharded.py:95-103): the common seed when every draw is keyed by global env
    id (no traffic models, or the counter-keyed traffic stream), else (seed + rank * 0x9E3779B97F4A7C15) mod 2^62 (the
    traffic models draw from one generator per engine); the rule ShardedEngine applies to its shards."""
    return importlib.import_module("isaac-net_b200.sharded").shard_seed(seed, rank, cfg, traffic_rng)


def max_over_ranks(vals, dist, dev):
    """Element-wise max of a list of floats over all ranks (identity without a process group)."""
    if dist is None:
        return list(vals)
    t = torch.tensor(list(vals), dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def shard_envs(wl, world, scaling):
    """Envs per GPU: the workload's envs split evenly over `world` GPUs (strong), or its per-GPU batch (weak)."""
    if scaling == "strong":
        if wl.E % world:
            raise SystemExit(f"{wl.E} envs do not split evenly over {world} GPUs")
        return wl.E // world
    return wl.envs_per_gpu


def arm_config(wl, cfg, world, E=None):
    E = E or wl.envs_per_gpu
    return {"workload": wl.name, "envs": E * world, "envs_per_gpu": E, "robots": wl.R,
            "slots_per_step": cfg.slots_per_step,
            "rbgs": cfg.n_subbands, "harq": cfg.n_harq, "frames": cfg.frame_buffer,
            "parallelism": f"env shards x{world}", "l2": "state > L2 (no flush needed)"}


def cpu_envs(a, wl):
    """Envs of the CPU sample: --cpu-envs, else the workload's whole per-GPU batch when the oracle steps it in a
    few seconds (configs 1 and 2: 64 x 16 and 4096 x 32 robots), else 256 envs (a labelled reduced E: the oracle
    needs ~1 s per step for 256 x 128 robots on 16 cores)."""
    if a.cpu_envs:
        return a.cpu_envs
    return wl.E if wl.E * wl.R <= 4096 * 32 else 256


def run_reference(a):
    """--impl reference: the reference's CPU path (the oracle port, the reference's own op sequence) on all host
    cores, rank 0 only; each step is a bounded sample of the workload's envs, sized so K steps take ~1-2 minutes."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if a.workload == "ul":
        ib = importlib.import_module("isaac-net_b200")
        cfg = ib.NRConfig(msg_sizes=(4000.0, 30000.0))
        res = ul_cpu_baseline(cfg, 4, UL_R, 1)
        v = res["value"]
        print(json.dumps({"metric": "env-steps/sec", "value": v, "unit": "env-steps/s", "n_gpus": a.gpus, "steps": 1,
                          "warmup": 1, "ms_per_step": 4 / v * 1e3, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                          "config": {"workload": "ul_4096x100_nrconfig_default"}, "cpu_baseline": res,
                          "e2e": {"value": v, "unit": "env-steps/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(a.workload)
    cfg = wl.config()
    steps = max(3, a.steps)
    envs = cpu_envs(a, wl)
    res = cpu_baseline(wl, cfg, envs, max(1, steps // 3), warm=max(1, min(a.warmup, 2)))
    v = res["value"]
    line = {"metric": "env-steps/sec", "value": v, "unit": "env-steps/s", "n_gpus": a.gpus, "steps": steps,
            "warmup": a.warmup, "ms_per_step": envs / v * 1e3, "higher_is_better": True, "scaling": a.scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded poses and the engine's traffic models)",
            "impl": "reference", "config": arm_config(wl, cfg, a.gpus, shard_envs(wl, a.gpus, a.scaling)),
            "cpu_baseline": res, "e2e": {"value": v, "unit": "env-steps/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def net_obs_bytes(F, K, dim, R):
    """Algorithmic bytes per robot of one observation-packing launch: the step-dict fields it reads (newest,
    queue_len, serving 8 B each; queue_bytes, sinr 4 B; delivered F B, cap 8F B, delay 4F B), its state read and
    written (last_cap 8 B, history 4K B), its outputs (last_cap 8 B, aoi 4 B, delay_s 4F B, rsrp 4 B, x 4 dim B,
    three flags) and the per-env t / det_env / cur_tag (17 B per env, shared by the R robots)."""
    return 8 * 3 + 4 * 2 + 13 * F + 2 * (8 + 4 * K) + 8 + 4 + 4 * F + 4 + 4 * dim + 3 + 17.0 / R


def net_obs_timing(o, cfg, E, R, dev, n=20, reps=5):
    """Average device time of the observation packing (inb_net_obs, every feature selected, history 4) on the bench
    engine's step dict `o`: n launches captured in a CUDA graph (the python launch path costs more host time than
    the kernel takes, so eager back-to-back launches would time the host), the graph replayed reps times between
    CUDA events on the replay stream."""
    nm = importlib.import_module("isaac-net_b200.net_module")
    pk = nm.ObsPacker(nm.OBS_FEATURES, E, R, cfg.frame_buffer, cfg.n_cells, 4, cfg.control_step_ms / 1000.0,
                      cfg.subband_noise_dbm, 50 * cfg.control_step_ms / 1000.0,
                      cfg.frame_buffer * max(cfg.msg_sizes), dev)
    cur = torch.zeros(E, dtype=torch.long, device=dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            pk.step(o, cur)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(n):
            pk.step(o, cur)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) / (n * reps) * 1e3
    del g
    per = net_obs_bytes(cfg.frame_buffer, 4, pk.dim, R)
    return {"kernel_us": us, "bytes_per_launch": per * E * R, "features": "all 12, history 4",
            "launches_per_step": 1, "timing": f"CUDA graph of {n} launches, replayed {reps} times"}


# The reference's own published NR benchmark (benchmarks/uncontended/bench_net.py --case L2 --cfg ul --E 4096 --R 100;
# docs/performance.md:201): NRConfig() defaults with messages of 4 kB / 30 kB, seed 1, every control step
# submit(send, det, hid) + step(None, snr[E,R]); 67.8 ms per step with its triton backend on an RTX 4090.
UL_PUBLISHED_MS = 67.8
UL_E, UL_R = 4096, 100


class UlInputs:
    """Pool of 16 input sets on the device, drawn as the reference's benchmark draws them (bench_net.py:152-171):
    every robot sends w.p. 0.3 (a third of those the 30 kB class), detection flags w.p. 0.1, an SNR [E,R] drifting
    around a U(0, 25) dB draw (+ N(0, 0.5^2) per step, clamped to [-5, 30])."""

    def __init__(self, E, R, dev, seed=0):
        g = torch.Generator(device=dev).manual_seed(seed)
        self.sends, self.dets, self.snrs = [], [], []
        snr = 25 * torch.rand(E, R, device=dev, generator=g)
        for _ in range(16):
            u = torch.rand(E, R, device=dev, generator=g)
            self.sends.append((u < 0.3).long() * (1 + (u < 0.1).long()))
            self.dets.append(torch.rand(E, R, device=dev, generator=g) < 0.1)
            snr = (snr + 0.5 * torch.randn(E, R, device=dev, generator=g)).clamp(-5, 30)
            self.snrs.append(snr.clone())
        self.hid = torch.zeros(E, dtype=torch.long, device=dev)


def ul_cpu_baseline(cfg, E, R, steps):
    """The oracle port (torch on the host cores, the reference's op sequence) on E envs of the ul workload."""
    from oracle.nr_oracle import OracleEngine
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    o = OracleEngine(cfg, E, R, "cpu", seed=1, reduce="aten")
    inp = UlInputs(E, R, "cpu")
    for k in range(1 + steps):
        if k == 1:
            t0 = time.perf_counter()
        o.submit(inp.sends[k % 16], inp.dets[k % 16], inp.hid)
        o.step(snr=inp.snrs[k % 16])
    dt = time.perf_counter() - t0
    return {"value": E * steps / dt, "unit": "env-steps/s", "cores": threads, "kind": "port",
            "sample": f"oracle port (torch CPU, reference op order) on {E} of {UL_E} envs x {R} robots, {steps} "
                      f"control steps after 1 warm-up"}


def run_ul(a, rank, world, dist, dev):
    """--workload ul: the reference's published network-only NR case (see UL_PUBLISHED_MS), E = 4096 envs x 100
    robots per GPU, through the public API (submit + step with an SNR input, the eager launch path of that input)."""
    ib = importlib.import_module("isaac-net_b200")
    cfg = ib.NRConfig(msg_sizes=(4000.0, 30000.0))
    E, R = UL_E, UL_R
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=1)
    eng.set_env_offset(rank * E)
    inp = UlInputs(E, R, dev, seed=rank)
    Rq = ib.Requests

    def one(k, fetch=None):
        eng.submit(None, Rq(inp.sends[k % 16], inp.dets[k % 16], inp.hid))
        return eng.step(None, inp.snrs[k % 16])

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for k in range(a.warmup):
        one(k)
    clocks = Clocks(dev.index)
    barrier()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for k in range(a.steps):
        one(a.warmup + k)
    e1.record()
    barrier()
    clk = clocks.stop()
    t_ms = e0.elapsed_time(e1)
    # e2e: sends and SNR from pinned host memory every step, the newest / queue_len outputs back to pinned memory
    hs = [x.cpu().pin_memory() for x in inp.sends]
    hr = [x.cpu().pin_memory() for x in inp.snrs]
    ho = {k: torch.empty(E, R, dtype=torch.long).pin_memory() for k in ("newest", "queue_len")}
    barrier()
    e0.record()
    for k in range(a.steps):
        send = hs[k % 16].to(dev, non_blocking=True)
        snr = hr[k % 16].to(dev, non_blocking=True)
        eng.submit(None, Rq(send, inp.dets[k % 16], inp.hid))
        out = eng.step(None, snr)
        for n, buf in ho.items():
            buf.copy_(out[n], non_blocking=True)
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
    for i in range(10):
        eng._kernel_events = kev[i]
        one(i)
    eng._kernel_events = None
    barrier()
    k_ms = sum(x.elapsed_time(y) for x, y in kev) / 10
    t_ms, e2e_ms, k_ms = max_over_ranks([t_ms, e2e_ms, k_ms], dist, dev)
    value = E * world * a.steps / (t_ms / 1e3)
    peak, peak_kind = peaks()
    per_launch = b_env(cfg, R) * E
    achieved = per_launch / (k_ms / 1e3) / 1e9
    published = UL_E / (UL_PUBLISHED_MS / 1e3)
    line = {"metric": "env-steps/sec", "value": value, "unit": "env-steps/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": t_ms / a.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / world / published, "dtype": "f32",
            "data": "synthetic (the reference benchmark's send / SNR distributions, seeded)",
            "config": {"workload": "ul_4096x100_nrconfig_default", "envs_per_gpu": E, "robots": R,
                       "slots_per_step": cfg.slots_per_step, "rbgs": cfg.n_subbands, "harq": cfg.n_harq,
                       "frames": cfg.frame_buffer, "parallelism": f"env shards x{world}",
                       "l2": "state > L2 (no flush needed)"},
            "baseline": {"ms_per_step": UL_PUBLISHED_MS, "value_per_gpu": published,
                         "source": "isaac-net triton backend on an RTX 4090, docs/performance.md:201"},
            "e2e": {"value": E * world * a.steps / (e2e_ms / 1e3), "unit": "env-steps/s",
                    "h2d_bytes_per_step": E * R * (8 + 4), "d2h_bytes_per_step": E * R * 16},
            "gpu_launches": a.steps * 3,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind, "kernel": "fading + MAC + finish kernels of one step",
                         "kernel_ms": k_ms, "algorithmic_bytes_per_launch": per_launch},
            "clocks": clk}
    if rank == 0 and world == 1 and not a.no_cpu:
        line["cpu_baseline"] = ul_cpu_baseline(cfg, 4, R, 1)
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--workload", default="4", help="BASELINE config 1-5 (default 4: 65536 envs x 128 robots), or "
                                                     "'ul': the reference's published NR benchmark case (NRConfig() "
                                                     "defaults, 4096 x 100 per GPU)")
    ap.add_argument("--cpu-envs", type=int, default=0, help="envs of the CPU sample (0: see cpu_envs)")
    ap.add_argument("--cpu-steps", type=int, default=2, help="steps per window of the CPU sample (3 windows)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--traffic-rng", default="generator", choices=("generator", "counter"),
                    help="the traffic models' stream: the reference's torch.Generator (default) or the opt-in "
                         "counter-keyed one, whose arrivals do not depend on the split over GPUs")
    ap.add_argument("--envs", type=int, default=0, help="envs per GPU (0: set by --scaling); a smaller batch of the "
                                                       "same workload, for profiling captures")
    ap.add_argument("--scaling", default="strong", choices=("weak", "strong"),
                    help="strong (default): the workload's envs split evenly over the GPUs (config 4: 65536 in all, "
                         "8192 per GPU at N = 8); weak: every GPU runs the workload's per-GPU envs (config 4: 8192)")
    a = ap.parse_args()
    if a.workload != "ul":
        a.workload = int(a.workload)
    if a.impl == "reference":
        return run_reference(a)
    a.warmup = max(3, a.warmup)
    rank, world, dist = dist_setup(a.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    if a.workload == "ul":
        return run_ul(a, rank, world, dist, dev)
    ib = importlib.import_module("isaac-net_b200")
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(a.workload)
    cfg = wl.config()
    R = wl.R
    E = a.envs or shard_envs(wl, world, a.scaling)
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=shard_seed(wl.seed, rank, cfg, a.traffic_rng),
                         traffic_rng=a.traffic_rng)
    eng.set_env_offset(rank * E)              # global env ids, initial reset redone under them
    mot = presets.Motion(a.workload, E, R, seed=wl.seed + 7919 * rank, step_ms=cfg.control_step_ms)
    # a ring of NPOS consecutive pose frames of the random walk (at most 512 MB), cycled: the trajectory jumps back
    # every NPOS steps
    NPOS = max(4, min(128, (512 << 20) // (E * R * 2 * 4)))
    host_pos = torch.empty(NPOS, E, R, 2, dtype=torch.float32).pin_memory()
    host_pos[0] = mot.current()
    for i in range(1, NPOS):
        host_pos[i] = mot.advance()
    dev_ring = host_pos.to(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(a.warmup):
        eng.step(None, dev_ring[i % NPOS])
    clocks = Clocks(dev.index)
    barrier()
    clocks.start()
    ev0.record()
    for i in range(a.steps):
        eng.step(None, dev_ring[(a.warmup + i) % NPOS])
    ev1.record()
    barrier()
    t_ms = ev0.elapsed_time(ev1)
    # e2e: poses from pinned host memory each step, observations read back each step
    obs_keys = ("newest", "queue_len", "queue_bytes", "sinr_db")
    host_obs = {k: torch.empty(E, R, dtype=torch.int64 if k in ("newest", "queue_len") else torch.float32)
                .pin_memory() for k in obs_keys}
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(a.steps):
        # the public API with host buffers: poses from pinned host memory in, observations to pinned host memory
        # out (the engine copies on its own input / output streams, overlapping the copies with the kernels)
        eng.step(None, host_pos[(a.warmup + a.steps + i) % NPOS], fetch=host_obs)
    torch.cuda.current_stream(dev).wait_event(eng.fetch_done)
    e1.record()
    barrier()
    clk = clocks.stop()     # sampled over the device-resident and the end-to-end timed regions
    e2e_ms = e0.elapsed_time(e1)
    # duration of the step's kernels alone: CUDA events around them on their stream (eager launches, same kernels)
    nk = min(a.steps, 20)
    for i in range(nk):
        eng._kernel_events = kev[i]
        last_o = eng.step(None, dev_ring[(a.warmup + i) % NPOS])
    eng._kernel_events = None
    barrier()
    k_ms = sum(s.elapsed_time(e) for s, e in kev[:nk]) / nk
    h2d = E * R * 2 * 4
    d2h = sum(host_obs[k].numel() * host_obs[k].element_size() for k in obs_keys)
    obs = net_obs_timing(last_o, cfg, E, R, dev)
    t_ms, e2e_ms, k_ms, obs_us = max_over_ranks([t_ms, e2e_ms, k_ms, obs["kernel_us"]], dist, dev)
    obs["kernel_us"] = obs_us
    obs["achieved_gbs"] = obs["bytes_per_launch"] / (obs_us * 1e-6) / 1e9
    # whole-batch MAC counters of the run: one all_reduce over the ranks (NCCL), after the timed regions
    sharded = importlib.import_module("isaac-net_b200.sharded")
    gc = sharded.global_counters(eng)["ul"]
    stats = {k: gc[k] for k in ("tb_new", "tb_retx", "tb_ok", "tb_fail", "prb_used", "prb_avail")}
    total_envs = E * world
    value = total_envs * a.steps / (t_ms / 1e3)
    e2e = total_envs * a.steps / (e2e_ms / 1e3)
    radio = bool(eng._args.rm.on)
    # per graph step: store2, [traffic], [radio], fading, MAC, finish
    launches = 4 + (1 if eng.dtraffic is not None else 0) + (1 if radio else 0)
    peak, peak_kind = peaks()
    per_launch = b_env(cfg, R) * E
    achieved = per_launch / (k_ms / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "nr_step_traffic.json")
    if os.path.exists(tp):
        try:
            tj = json.load(open(tp))
            traffic = tj.get("bytes_per_launch_scaled", {}).get(wl.name)
            if traffic is not None:      # captured at the workload's whole batch on one GPU: this rank's share
                traffic = traffic * E / wl.E
        except Exception:
            traffic = None
    line = {"metric": "env-steps/sec", "value": value, "unit": "env-steps/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": t_ms / a.steps, "higher_is_better": True, "scaling": a.scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded poses and the engine's traffic models)",
            "config": {**arm_config(wl, cfg, world, E), "traffic_rng": a.traffic_rng},
            "e2e": {"value": e2e, "unit": "env-steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": a.steps * launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": ("traffic + radio + fading + MAC + finish kernels of one step" if radio else
                                    "traffic + fading + MAC + finish kernels of one step"),
                         "kernel_ms": k_ms, "algorithmic_bytes_per_launch": per_launch},
            "clocks": clk, "mac_counters": stats}
    obs["frac"] = obs["achieved_gbs"] / peak
    line["net_obs"] = obs
    if rank == 0 and world == 1 and not a.no_cpu:
        line["cpu_baseline"] = cpu_baseline(wl, cfg, cpu_envs(a, wl), a.cpu_steps)
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
