"""The network-observation packing (the Isaac-side consumer of the step dict): NetModule.step's post-processing and
NetObs.update of isaac-net v0.2.0 (isaac_net/isaac/net_module.py:340-374, isaac_net/isaac/obs.py:48-87).

CPU: the oracle restatement (oracle/net_obs.py) fed the reference's own engine outputs reproduces the reference's
NetModule outputs and observations bitwise (fixtures tests/golden/o*.npz from tests/golden/make_obs_golden.py:
all twelve features, three cells, blockage outputs, partial resets).  GPU: the inb_net_obs kernel (through the C ABI)
equals the oracle on the same device bitwise, and the reference's CPU outputs within 1e-5 relative (torch divides by
a python scalar on the CPU and multiplies by its float32 reciprocal on a CUDA device); the NetModule end to end
(engine graph steps + the packing launch) equals the oracle fed the engine's own step dicts.
"""
import importlib
import os

import numpy as np
import pytest
import torch

from oracle.net_obs import NetObsOracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ("o1", "o3", "o1b")
nm = importlib.import_module("isaac-net_b200.net_module")
presets = importlib.import_module("isaac-net_b200.presets")


class ObsGolden:
    def __init__(self, case):
        import ast
        self.d = np.load(os.path.join(GOLDEN, f"{case}.npz"))
        self.E, self.R, self.steps = int(self.d["E"]), int(self.d["R"]), int(self.d["steps"])
        self.wl = presets.workload(int(self.d["workload"]))
        self.cfg = self.wl.config(**ast.literal_eval(str(self.d["overrides"])))
        self.features = tuple(str(f) for f in self.d["features"])
        self.K = int(self.d["history"])
        ts = float(self.d["time_scale"])
        self.time_scale = ts if ts > 0 else 50 * self.cfg.control_step_ms / 1000.0

    def eng(self, s, dev):
        pre = f"s{s}/eng."
        return {k[len(pre):]: torch.as_tensor(self.d[k]).to(dev) for k in self.d.files if k.startswith(pre)}

    def net(self, s):
        pre = f"s{s}/net."
        return {k[len(pre):]: self.d[k] for k in self.d.files if k.startswith(pre)}

    def obs(self, s):
        return self.d[f"s{s}/obs"]

    def cur_tag(self, s, dev):
        return torch.as_tensor(self.d[f"s{s}/in.cur_tag"]).to(dev)

    def reset_ids(self, s):
        return np.nonzero(self.d["resets"][s])[0].tolist()

    def params(self):
        c = self.cfg
        return dict(E=self.E, R=self.R, F=c.frame_buffer, G=c.n_cells, history=self.K, time_scale=self.time_scale,
                    step_dt=c.control_step_ms / 1000.0, noise_db=c.subband_noise_dbm,
                    q_bytes=c.frame_buffer * max(c.msg_sizes))

    def oracle(self, dev):
        return NetObsOracle(self.features, device=dev, **self.params())


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_fixture(case):
    g = ObsGolden(case)
    orc = g.oracle("cpu")
    for s in range(g.steps):
        ids = g.reset_ids(s)
        if ids:
            orc.reset(ids)
        out, x = orc.step(g.eng(s, "cpu"), g.cur_tag(s, "cpu"))
        ref = g.net(s)
        assert set(out) == set(ref), set(out) ^ set(ref)
        for k, v in ref.items():
            np.testing.assert_array_equal(_np(out[k]), v, err_msg=f"step {s} {k}")
        np.testing.assert_array_equal(_np(x), g.obs(s), err_msg=f"step {s} obs")


def test_feature_names_and_widths():
    """Aliases, order and widths as isaac/config.py:90-106 gives them; unknown and repeated names refused."""
    assert nm.canonical_features(("snr", "delivered", "delay", "queue")) == ("sinr", "last_delivered", "msg_delay",
                                                                              "queue_len")
    assert nm.feature_dims(("msg_delay", "aoi", "serving_cell", "delay_history"), 16, 3, 5) == \
        {"msg_delay": 16, "aoi": 1, "serving_cell": 3, "delay_history": 5}
    with pytest.raises(ValueError):
        nm.canonical_features(("aoi", "aoi"))
    with pytest.raises(ValueError):
        nm.canonical_features(("nope",))
    cfg = presets.workload(1).config()
    isc = nm.IsaacNetCfg(radio="engine", obs_features=("aoi", "delivered_mask"), obs_history=3)
    assert isc.obs_dim(cfg) == 1 + cfg.frame_buffer
    assert isc.time_scale_s(cfg) == 50 * cfg.control_step_ms / 1000.0


def test_netmodule_refusals_on_cpu():
    """The Isaac radio and the nr overrides are refused before anything is allocated (no GPU needed)."""
    B = importlib.import_module("isaac-net_b200.engine").B200Unsupported
    cfg = presets.workload(1).config()
    with pytest.raises(B):
        nm.NetModule("L2", 2, 16, "cpu", cfg, isaac=nm.IsaacNetCfg(radio="isaac"))
    with pytest.raises(B):
        nm.NetModule("L1", 2, 16, "cpu", cfg, isaac=nm.IsaacNetCfg(radio="engine"))
    with pytest.raises(B):
        nm.NetModule("L2", 2, 16, "cpu", cfg, isaac=nm.IsaacNetCfg(radio="engine", nr={"n_harq": 4}))


def _close(a, b, rtol=1e-5, atol=1e-6):
    if a.dtype.kind == "f":
        return np.allclose(a.astype(np.float64), b.astype(np.float64), rtol=rtol, atol=atol, equal_nan=True)
    return np.array_equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_kernel_matches_oracle_and_reference(case):
    """inb_net_obs on cuda:0 fed the reference's engine outputs: bitwise the oracle on the same device, and the
    reference's CPU outputs and observations within 1e-5 relative (integers and flags exact)."""
    g = ObsGolden(case)
    dev = torch.device("cuda:0")
    p = g.params()
    pk = nm.ObsPacker(g.features, p["E"], p["R"], p["F"], p["G"], p["history"], p["step_dt"], p["noise_db"],
                      p["time_scale"], p["q_bytes"], dev)
    orc = g.oracle(dev)
    for s in range(g.steps):
        ids = g.reset_ids(s)
        if ids:
            pk.reset(torch.as_tensor(ids, device=dev))
            orc.reset(ids)
        o = g.eng(s, dev)
        ct = g.cur_tag(s, dev)
        b = pk.step(o, ct)
        out_o, x_o = orc.step(o, ct)
        got = {"last_cap": b["last_cap_out"], "aoi_s": b["aoi_s"], "delay_s": b["delay_s"], "rsrp_dbm": b["rsrp_dbm"],
               "delivered": b["delivered_any"], "blocked": b["blocked_out"], "los": b["los_out"],
               "tag_delivered": b["tag_delivered"]}
        for k, v in got.items():
            assert torch.equal(torch.nan_to_num(v, nan=7.0) if v.is_floating_point() else v,
                               torch.nan_to_num(out_o[k], nan=7.0) if v.is_floating_point() else out_o[k]), (s, k)
            assert _close(_np(v), g.net(s)[k]), (s, k)
        assert torch.equal(b["x"], x_o), (s, "obs")
        assert _close(_np(b["x"]), g.obs(s)), (s, "obs vs reference")
    assert torch.equal(pk.hist, orc.hist) and torch.equal(pk.last_cap, orc.last_cap)


@pytest.mark.gpu
@pytest.mark.parametrize("wl_i,E,R,feats", [
    (1, 8, 16, nm.OBS_FEATURES),
    (3, 3, 64, ("serving_cell", "delay_history", "aoi", "rsrp", "los", "msg_delay")),
])
def test_netmodule_end_to_end(wl_i, E, R, feats):
    """NetModule on the B200 engine (graph steps after the first) with message submissions, tags and a partial
    reset: every output and the observation equal the oracle fed the engine's own step dicts, bitwise."""
    wl = presets.workload(wl_i)
    cfg = wl.config()
    dev = torch.device("cuda:0")
    net = nm.NetModule("L2", E, R, dev, cfg, isaac=nm.IsaacNetCfg(radio="engine", obs_features=feats, obs_history=3),
                       seed=wl.seed)
    rec = {}
    step0 = net.eng.step

    def wrap(*a, **k):
        o = step0(*a, **k)
        rec.clear()
        rec.update(o)
        return o

    net.eng.step = wrap
    orc = NetObsOracle(net.features, E, R, cfg.frame_buffer, cfg.n_cells, 3, net.isaac.time_scale_s(cfg),
                       cfg.control_step_ms / 1000.0, cfg.subband_noise_dbm, cfg.frame_buffer * max(cfg.msg_sizes), dev)
    mot = presets.Motion(wl_i, E, R, seed=9, step_ms=cfg.control_step_ms)
    gen = torch.Generator().manual_seed(3)
    pos = mot.current()
    for s in range(10):
        if s == 6:
            net.reset([1])
            orc.reset([1])
        send = (torch.rand(E, R, generator=gen) < 0.4).long()
        tag = torch.where(torch.rand(E, R, generator=gen) < 0.5, torch.randint(0, 3, (E, R), generator=gen),
                          torch.full((E, R), -1, dtype=torch.long))
        cur = torch.randint(-1, 3, (E,), generator=gen)
        net.submit(None, nm.TrafficRequest(send.to(dev), tag.to(dev)))
        out = net.step(None, pos.to(dev), cur.to(dev))
        ref, x = orc.step({k: v.clone() for k, v in rec.items()}, cur.to(dev))
        assert set(out) == set(ref)
        for k in ref:
            a, b = out[k], ref[k]
            if a.is_floating_point():
                a, b = torch.nan_to_num(a, nan=7.0), torch.nan_to_num(b, nan=7.0)
            assert torch.equal(a, b), (s, k)
        assert torch.equal(net.obs(), x), s
        pos = mot.advance()


def test_packer_arguments_on_cpu():
    """The launch arguments ObsPacker builds (no launch): every selected feature's first column of x in the order
    given, -1 for the others, and the float32 constants torch uses on a CUDA device (python scalars rounded to
    float32, divisions as float32 reciprocals)."""
    feats = ("sinr", "delay_history", "serving_cell", "msg_delay", "aoi")
    pk = nm.ObsPacker(feats, 2, 3, 16, 3, 5, 0.005, -96.99, 0.25, 16 * 30000.0, "cpu")
    a = pk.args
    assert (a.E, a.R, a.F, a.G, a.K, a.dim) == (2, 3, 16, 3, 5, 1 + 5 + 3 + 16 + 1)
    assert (a.off_sinr, a.off_hist, a.off_serv, a.off_delay, a.off_aoi) == (0, 1, 6, 9, 25)
    for n in ("off_mask", "off_qlen", "off_qbytes", "off_rsrp", "off_last", "off_blocked", "off_los"):
        assert getattr(a, n) == -1, n
    f32 = lambda x: float(np.float32(x))
    assert a.step_dt == f32(0.005) and a.noise_db == f32(-96.99)
    assert a.inv_ts == float(np.float32(1) / np.float32(0.25)) and a.inv_db == float(np.float32(1) / np.float32(40))
    assert a.inv_F == float(np.float32(1) / np.float32(16))
    assert a.inv_qbytes == float(np.float32(1) / np.float32(16 * 30000.0))
    assert pk.last_cap.shape == (2, 3) and pk.hist.shape == (2, 3, 5)
