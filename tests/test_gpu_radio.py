"""The radio launch on the GPU for cases the fixtures do not hold: poses outside the map and on its grid lines, and
blockage model A on the log-distance channel with three cells (the formula path of the radio kernel).  The engine's
radio is compared with the oracle's (the reference's torch op sequence) on the CPU, from the oracle's draws."""
import importlib

import pytest
import torch

from oracle.nr_oracle import OracleEngine

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")

pytestmark = pytest.mark.gpu


def _radio_snapshot(orc):
    """The oracle radio's draws under the reference's names (the engine draws the same streams with torch's CUDA
    cos / sin, which differ from the CPU's by an ulp; loading the CPU draws isolates the kernel's evaluation)."""
    rad, snap = orc.radio, {}
    for n, key in (("ld", "radio"), ("sf_los", "radio.sf_los")):
        if n in rad.fields:
            snap[key + ".k"], snap[key + ".phi"] = rad.fields[n]
    if rad.blk is not None:
        b = rad.blk
        snap.update({"radio.blk.k": b.k, "radio.blk.phi": b.phi, "radio.blk.xk": b.xk, "radio.blk.yk": b.yk,
                     "radio.blk.vel": b.vel, "radio.blk.t": b.t})
    return snap


def _compare(cfg, pos_steps, E, R, seed=7):
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=seed)
    orc = OracleEngine(cfg, E, R, "cpu", seed=seed, reduce="aten")
    far = links = bad_blk = 0
    for i, pos in enumerate(pos_steps):
        if i == 0:
            from oracle.nr_oracle import Radio
            orc.radio = Radio(cfg, orc.rng, E, orc.dev)
            eng.load_reference_state(_radio_snapshot(orc))
        out = eng.step(None, pos.to(dev))
        a = eng.last_arrivals
        arr = None if a is None else {k: getattr(a, k).cpu() for k in ("valid", "nbytes", "slot", "tag", "prio",
                                                                         "dline", "det")}
        ref = orc.step(pos, arr)
        pg, pg_ref = eng.pathgain.cpu().reshape(orc.pathgain.shape), orc.pathgain
        assert bool(torch.isfinite(pg).all())
        d = (pg - pg_ref).abs()
        far += int((d > 1e-3).sum())
        links += d.numel()
        if "blocked" in ref:
            bad_blk += int((out["blocked"].cpu() != ref["blocked"]).sum())
    return far, links, bad_blk


def test_radio_map_outside_and_on_grid_lines():
    cfg = presets.workload(5).config()
    E, R = 4, 48
    g = torch.Generator().manual_seed(3)
    steps = []
    for k in range(3):
        pos = torch.rand(E, R, 2, generator=g) * 300.0 - 20.0          # partly outside [0, 255.5]^2
        pos[0, :8] = torch.tensor([[0.0, 0.0], [255.5, 255.5], [-1e3, 50.0], [1e4, 1e4], [0.5, 0.5], [64.0, 128.0],
                                   [127.75, 200.0], [255.5, 0.0]])
        steps.append(pos)
    far, links, bad_blk = _compare(cfg, steps, E, R)
    assert far * 500 <= links and bad_blk * 500 <= E * R * len(steps), (far, links, bad_blk)


def test_blockage_on_log_distance_three_cells():
    cfg = presets.workload(3).config(blockage=True, blockage_model="stochastic")
    E, R = 3, 64
    mo = presets.Motion(3, E, R, seed=5, step_ms=cfg.control_step_ms)
    steps = [mo.current()] + [mo.advance() for _ in range(3)]
    far, links, bad_blk = _compare(cfg, steps, E, R)
    assert far * 500 <= links and bad_blk * 500 <= E * R * len(steps), (far, links, bad_blk)
