"""The downlink MAC (dl=True, one cell; DlMac, isaac_net/core/mac_dl.py:1-49) on the GPU, through the C ABI.

1. kernel == oracle "seq" on the same CUDA device, bitwise, every output (the uplink's and dl_newest, dl_queue_len,
   the dl_* frame outputs, gen_dl_*) and every state tensor (the DL link's net.dl.* / net.dl.q.* included), over the
   DL golden cases (TDD patterns with D / S / U slots, DL and UL traffic models, CQI reports, DL HARQ with failures),
   the oracle fed the kernel's arrivals of both links and its path gains;
2. kernel vs the reference's own outputs (CPU fixtures) teacher-forced: loaded with the reference state (both links)
   before each step and fed the reference's arrivals of both links and its radio's path gains: no robot-step may
   differ in an integer output, floats within 1e-5 relative / 1e-3 absolute;
3. the policy's DL path: add_dl_frames every step with an SNR input (snr + dl_snr_offset_db, and an explicit
   dl_snr_db), engine == oracle bitwise."""
import importlib

import numpy as np
import pytest
import torch

from golden_io import DL_CASES, Golden
from oracle.nr_oracle import OracleEngine, Radio

ib = importlib.import_module("isaac-net_b200")
ARR = ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")

pytestmark = pytest.mark.gpu


def _eq_t(a, b):
    if a.dtype.is_floating_point:
        return torch.equal(torch.nan_to_num(a, nan=12345.0), torch.nan_to_num(b, nan=12345.0)) and \
            torch.equal(torch.isnan(a), torch.isnan(b))
    return torch.equal(a, b)


def _arr(a):
    return {k: getattr(a, k) for k in ARR}


class _Arr:
    def __init__(self, d, dev):
        for k, v in d.items():
            setattr(self, k, torch.as_tensor(v).to(dev))


@pytest.mark.parametrize("case", DL_CASES)
def test_downlink_kernel_equals_oracle_seq(case):
    g = Golden(case)
    cfg, wl = g.config(), g.workload()
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", g.E, g.R, dev, cfg, seed=wl.seed)
    orc = OracleEngine(cfg, g.E, g.R, dev, seed=wl.seed, reduce="seq")
    st_o, st_k = orc.reference_state(), eng.reference_state()
    for k, v in st_o.items():
        assert _eq_t(st_k[k], v), f"initial state {k}"
    for s in range(g.steps):
        ids = g.reset_ids(s)
        if ids:
            eng.reset(ids)
            orc.reset(ids)
        pos = torch.as_tensor(g.pos(s)).to(dev)
        out = eng.step(None, pos)
        ref = orc.step(None, _arr(eng.last_arrivals), pathgain=eng.pathgain.clone(),
                       dl_arrivals=_arr(eng.dl.last_arrivals))
        assert set(out) == set(ref), set(out) ^ set(ref)
        for k in ref:
            assert _eq_t(out[k], ref[k]), f"step {s} output {k}"
        st_o, st_k = orc.reference_state(), eng.reference_state()
        for k, v in st_o.items():
            assert _eq_t(st_k[k], v), f"step {s} state {k}"
    c = eng.counters()
    assert c["dl"]["tb_new"] > 0 and c["dl"]["tb_ok"] + c["dl"]["tb_fail"] == c["dl"]["tb_new"] + c["dl"]["tb_retx"]


@pytest.mark.parametrize("case", DL_CASES)
def test_downlink_vs_reference_teacher_forced(case):
    g = Golden(case)
    cfg, wl = g.config(), g.workload()
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", g.E, g.R, dev, cfg, seed=wl.seed)
    flips = total = n = 0
    for s in range(1, g.steps):
        if not g.has_state(s - 1) or g.reset_ids(s):
            continue
        snap = g.state(s - 1)
        eng.load_reference_state(snap)
        o = OracleEngine(cfg, g.E, g.R, "cpu", seed=wl.seed, reduce="aten")
        o.load_reference_state(snap)
        rad = o.radio if o.radio is not None else Radio(cfg, o.rng, g.E, o.dev)
        pg = rad.pathgain_db(torch.as_tensor(g.pos(s)))[..., 0]
        out = eng.step(None, None, _pathgain=pg.to(dev), _arrivals=_Arr(g.arrivals(s), dev),
                       _dl_arrivals=_Arr(g.dl_arrivals(s), dev))
        ref = g.outputs(s)
        rows = np.ones((g.E, g.R), dtype=bool)
        for k, v in ref.items():
            a = out[k].cpu().numpy()
            if a.dtype.kind == "f":
                eq = np.isclose(a.astype(np.float64), v.astype(np.float64), rtol=1e-5, atol=1e-3, equal_nan=True)
            else:
                eq = a == v
            rows &= eq[:, None] if eq.ndim == 1 else eq.reshape(g.E, g.R, -1).all(-1)
        flips += int((~rows).sum())
        total += g.E * g.R
        n += 1
    assert n > 0
    assert flips == 0, (flips, total)


def test_downlink_policy_frames_and_snr_input():
    """add_dl_frames every step (no DL traffic models) with the SNR input: the DL reference is snr + dl_snr_offset_db,
    and on alternate steps an explicit dl_snr_db per RBG; engine == oracle ("seq", same device) bitwise."""
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(1)
    cfg = wl.config(tdd_pattern="DDSUU", dl=True, traffic=None, msg_sizes=(1500.0,), timeout_steps=6)
    E, R, S = 4, 16, cfg.n_subbands
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    orc = OracleEngine(cfg, E, R, dev, seed=wl.seed, reduce="seq")
    gen = torch.Generator().manual_seed(5)
    for s in range(14):
        if s == 8:
            eng.reset([2])
            orc.reset([2])
        nb = torch.where(torch.rand(E, R, generator=gen) < 0.5, torch.randint(200, 9000, (E, R), generator=gen),
                         torch.zeros(E, R, dtype=torch.long)).float().to(dev)
        cls = torch.randint(1, 4, (E, R), generator=gen).to(dev)
        acc_k = eng.add_dl_frames(None, nb, cls)
        acc_o = orc.add_dl_frames(nb, cls)
        assert torch.equal(acc_k, acc_o), s
        snr = (torch.randn(E, R, generator=gen) * 8.0 + 12.0).to(dev)
        if s % 2:
            dl_snr = (torch.randn(E, R, S, generator=gen) * 6.0 + 10.0).to(dev)
            out = eng.step(None, snr, dl_snr_db=dl_snr)
            ref = orc.step(snr=snr, dl_snr=dl_snr)
        else:
            out = eng.step(None, snr)
            ref = orc.step(snr=snr)
        for k in ref:
            assert _eq_t(out[k], ref[k]), f"step {s} output {k}"
        st_o, st_k = orc.reference_state(), eng.reference_state()
        for k, v in st_o.items():
            assert _eq_t(st_k[k], v), f"step {s} state {k}"
    assert eng.counters()["dl"]["tb_new"] > 0


@pytest.mark.parametrize("case", DL_CASES)
def test_downlink_graph_steps_equal_eager_steps(case):
    """DL configs step through CUDA graphs (the DL traffic models, the DL MAC and finish launches captured with the
    uplink's, the DL outputs in the step's output block): graph steps equal eager steps bitwise, in every output and
    state tensor of both links, with add_dl_frames between steps and a partial reset."""
    g = Golden(case)
    cfg, wl = g.config(), g.workload()
    dev = torch.device("cuda:0")
    eager = ib.make_engine("L2", g.E, g.R, dev, cfg, seed=wl.seed)
    eager.graphs = False
    graph = ib.make_engine("L2", g.E, g.R, dev, cfg, seed=wl.seed)
    gen = torch.Generator().manual_seed(11)
    for s in range(g.steps):
        ids = g.reset_ids(s)
        if ids:
            eager.reset(ids)
            graph.reset(ids)
        if s % 3 == 1:
            nb = torch.where(torch.rand(g.E, g.R, generator=gen) < 0.3,
                             torch.randint(200, 6000, (g.E, g.R), generator=gen),
                             torch.zeros(g.E, g.R, dtype=torch.long)).float().to(dev)
            assert torch.equal(eager.add_dl_frames(None, nb), graph.add_dl_frames(None, nb)), s
        pos = torch.as_tensor(g.pos(s)).to(dev)
        o_e, o_g = eager.step(None, pos), graph.step(None, pos)
        assert set(o_e) == set(o_g), s
        for k in o_e:
            if torch.is_tensor(o_e[k]):
                assert _eq_t(o_e[k], o_g[k]), f"step {s} output {k}"
    assert graph._graphs, "no graph was captured"
    st_e, st_g = eager.reference_state(), graph.reference_state()
    for k, v in st_e.items():
        if torch.is_tensor(v):
            assert _eq_t(st_g[k], v), f"state {k}"
    assert eager.counters() == graph.counters()
