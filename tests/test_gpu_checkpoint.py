"""Checkpoints: state_dict() of a running engine loaded into a fresh engine of the same config continues exactly
like the original (every output of the following steps and the final state bitwise equal, CUDA graphs on), through a
file as well; mismatched sizes and configs are refused."""
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")

pytestmark = pytest.mark.gpu


def _same(a, b):
    if not torch.is_tensor(a):
        return a == b
    if a.dtype.is_floating_point:
        return torch.equal(a.isnan(), b.isnan()) and torch.equal(a.nan_to_num(0.0), b.nan_to_num(0.0))
    return torch.equal(a, b)


@pytest.mark.parametrize("wl_i,E,R", [(2, 32, 32), (3, 4, 64), (5, 6, 48), (1, 8, 16)])
def test_resume_is_bitwise_the_uninterrupted_run(wl_i, E, R, tmp_path):
    wl = presets.workload(wl_i)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    a = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    mo = presets.Motion(wl_i, E, R, seed=6, step_ms=cfg.control_step_ms)
    frames = [mo.current()] + [mo.advance() for _ in range(11)]
    for s in range(5):
        if s == 3:
            a.reset([1])
        a.step(None, frames[s].to(dev))
    sd = a.state_dict()
    b = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    b.step(None, frames[0].to(dev))              # b has its own history (and captured radio) before the restore
    b.load_state_dict(sd)
    a.save(tmp_path / "ck.pt", extra={"iter": 5})
    c = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    assert c.load(tmp_path / "ck.pt") == {"iter": 5}
    for s in range(5, 12):
        outs = [e.step(None, frames[s].to(dev)) for e in (a, b, c)]
        for k, v in outs[0].items():
            for o in outs[1:]:
                assert _same(v, o[k]), (s, k)
    fa, fb, fc = a.state_dict(), b.state_dict(), c.state_dict()
    for k, v in fa.items():
        assert _same(v, fb[k]) and _same(v, fc[k]), k
    assert a.counters() == b.counters() == c.counters()


def test_refusals():
    wl = presets.workload(1)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    a = ib.make_engine("L2", 8, 16, dev, cfg, seed=0)
    sd = a.state_dict()
    with pytest.raises(ValueError):
        ib.make_engine("L2", 4, 16, dev, cfg, seed=0).load_state_dict(sd)
    with pytest.raises(ValueError):
        ib.make_engine("L2", 8, 16, dev, cfg.with_(n_harq=8), seed=0).load_state_dict(sd)
    bad = dict(sd)
    bad.pop("st.sent")
    with pytest.raises(KeyError):
        ib.make_engine("L2", 8, 16, dev, cfg, seed=0).load_state_dict(bad)
    ib.make_engine("L2", 8, 16, dev, cfg, seed=0).load_state_dict(bad, strict=False)


class _Arr:
    def __init__(self, d, dev):
        for k, v in d.items():
            setattr(self, k, torch.as_tensor(v).to(dev))


@pytest.mark.parametrize("case", ("k2", "k3", "k5"))
def test_continue_from_a_reference_checkpoint(case):
    """The reference engine's own state_dict() (isaac_net/core/checkpoint.py format; fixtures cfgk*.npz) loaded into
    the B200 engine: every state key is placed (strict), the engine written back under the reference's keys
    reproduces the loaded values, and the following steps (the reference's arrivals and path gains fed in) give the
    reference's outputs: integers bitwise, floats within 1e-5 relative / 1e-3 absolute; the counters end at the
    reference's totals."""
    import ast
    import numpy as np
    from golden_io import GOLDEN
    d = np.load(f"{GOLDEN}/cfg{case}.npz")
    wl = presets.workload(int(d["workload"]))
    cfg = wl.config(**ast.literal_eval(str(d["overrides"])))
    E, R, n = int(d["E"]), int(d["R"]), int(d["steps"])
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    ckpt = {k[5:]: torch.as_tensor(d[k]) if d[k].ndim else d[k].item() for k in d.files if k.startswith("ckpt/")}
    eng.load_reference_checkpoint(ckpt, strict=True)
    back = eng.reference_checkpoint()
    for k, v in back.items():
        if k in ckpt and not k.startswith("net.ul.ctr[") and k != "net.ul.ntx_hist":
            want = torch.as_tensor(ckpt[k])
            got = torch.as_tensor(v).to(want.dtype)
            assert got.shape == want.shape and _same(got, want), k
    for s in range(n):
        pg = torch.as_tensor(d[f"s{s}/pg"])
        pg = pg[..., 0] if eng.C == 1 else pg
        arr = {m: d[f"s{s}/arr.{m}"] for m in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")}
        out = eng.step(None, None, _pathgain=pg.to(dev), _arrivals=_Arr(arr, dev))
        for k in [x[len(f"s{s}/out."):] for x in d.files if x.startswith(f"s{s}/out.")]:
            if k in ("blocked", "los"):   # obstacle outputs come from the radio; the path gains are fed in here
                continue
            ref = d[f"s{s}/out.{k}"]
            got = out[k].cpu().numpy()
            if ref.dtype.kind == "f":
                assert np.allclose(got.astype(np.float64), ref.astype(np.float64), rtol=1e-5, atol=1e-3,
                                   equal_nan=True), (s, k)
            else:
                assert np.array_equal(got, ref), (s, k)
    c = eng.counters()["ul"]
    for k in ("tb_new", "tb_retx", "tb_ok", "tb_fail", "exhaust", "bytes_ok", "bytes_new", "prb_used", "prb_avail"):
        assert c[k] == float(d[f"end/ctr.{k}"]), k
