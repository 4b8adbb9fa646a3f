"""Radio-map and blockage pieces on CPU: the file format, the bilinear sample (known answers, border clamping), the
blockage CDF table and the host loader's refusals.  The oracle functions are pinned bitwise to the reference by the
config-5 golden fixtures; these checks pin them against hand-computed values as well."""
import importlib
import math

import numpy as np
import pytest
import torch

from oracle import nr_oracle as orc

rm = importlib.import_module("isaac-net_b200.radio_map")
mk = importlib.import_module("isaac-net_b200.data.make_radio_map")


def test_bilinear_known_answers_and_border_clamp():
    # 2 cells on a 3 x 4 grid (H = 3 rows along y, W = 4 columns along x) over x in [0, 3], y in [10, 12]
    g = torch.tensor([[[0., 1., 2., 3.], [10., 11., 12., 13.], [20., 21., 22., 23.]],
                      [[5., 5., 5., 5.], [5., 5., 5., 5.], [5., 5., 5., 5.]]])
    C, H, W = g.shape
    bounds = (0.0, 10.0, 3.0, 12.0)
    pos = torch.tensor([[[0.0, 10.0], [1.5, 10.5], [3.0, 12.0], [-5.0, 9.0], [7.0, 30.0], [2.25, 11.0]]])
    out = orc.sample_map(g.reshape(C, H * W), H, W, bounds, pos)
    # value = x + 10 (y - 10) on cell 0 (bilinear is exact on this plane), clamped at the borders; cell 1 constant
    want0 = [0.0, 1.5 + 5.0, 23.0, 0.0, 23.0, 2.25 + 10.0]
    assert torch.allclose(out[0, :, 0], torch.tensor(want0), atol=1e-5)
    assert torch.equal(out[0, :, 1], torch.full((6,), 5.0))


def test_baked_map_format_and_geometry():
    path = mk.ensure()
    gain, H, W, bounds, meta = rm.load_radio_map(path)
    assert gain.shape == (2, 512 * 512) and (H, W) == (512, 512) and gain.dtype == torch.float32
    assert bounds == (0.0, 0.0, 255.5, 255.5)
    assert np.allclose(np.asarray(meta["gnb_xy"]), [[64.0, 128.0], [192.0, 128.0]])
    g = gain.view(2, H, W)
    # each cell is strongest near its own gNB (grid point (x_j, y_i) = (0.5 j, 0.5 i) m)
    j0, i0 = int(64 / 0.5), int(128 / 0.5)
    j1 = int(192 / 0.5)
    assert g[0, i0, j0] > g[1, i0, j0] + 10 and g[1, i0, j1] > g[0, i0, j1] + 10
    assert float(g.max()) < -60.0 and float(g.min()) > -200.0
    # baking again gives the same bytes
    d = torch.tensor(mk.bake()["gain_db"]) - g
    assert float(d.abs().max()) == 0.0


def test_cdf_table_is_the_sorted_unit_marginal():
    t = orc.cdf_table(8)
    assert t.shape == (65536,) and t.dtype == torch.float32
    assert bool((t[1:] >= t[:-1]).all())
    assert abs(float(t.double().mean())) < 0.02 and abs(float(t.double().var()) - 1.0) < 0.02
    assert torch.equal(t, rm.cdf_table(8))          # the product's table is the oracle's, bit for bit
    # uniform_from_field: (#{table < z} + 0.5) / (n + 1)
    z = torch.tensor([-10.0, 10.0, float(t[1000])])
    u = (torch.searchsorted(t, z).float() + 0.5) / (t.numel() + 1)
    assert float(u[0]) == pytest.approx(0.5 / 65537) and float(u[1]) == pytest.approx(65536.5 / 65537)
    assert int(torch.searchsorted(t, z)[2]) <= 1000


def test_angle_f_sign_and_window_terms():
    lam, r = 3e8 / 3.5e9, 2.0
    d = torch.tensor([0.0, 10.0, -10.0, 89.9, 120.0])
    fin = orc._angle_f(d, torch.ones(5, dtype=torch.bool), r, lam)
    fout = orc._angle_f(d, torch.zeros(5, dtype=torch.bool), r, lam)
    assert float(fin[0]) == 0.0 and torch.allclose(fin, -fout)
    assert bool((fin[1:] > 0).all()) and bool((fin < 0.5).all())
    assert float(fin[3]) == float(fin[4])            # |delta| clamped at 89.9 deg
    a = (math.pi / 2) * math.sqrt((math.pi / lam) * r * (1 / math.cos(math.radians(10.0)) - 1))
    assert float(fin[1]) == pytest.approx(math.atan(a) / math.pi, rel=1e-5)


def test_loader_refusals(tmp_path):
    with pytest.raises(ValueError):
        rm.load_radio_map(None)
    with pytest.raises(ValueError):
        rm.load_radio_map("synthetic")
    bad = tmp_path / "bad.npz"
    np.savez(bad, gain_db=np.zeros((2, 1, 5), np.float32), bounds=np.array([0.0, 0.0, 1.0, 1.0]))
    with pytest.raises(ValueError):
        rm.load_radio_map(str(bad))
    flipped = tmp_path / "flipped.npz"
    np.savez(flipped, gain_db=np.zeros((2, 4, 4), np.float32), bounds=np.array([1.0, 0.0, 0.0, 1.0]))
    with pytest.raises(ValueError):
        rm.load_radio_map(str(flipped))


def test_config_refusals_for_obstacles():
    cfgmod = importlib.import_module("isaac-net_b200.config")
    presets = importlib.import_module("isaac-net_b200.presets")
    assert presets.workload(5).config().refusals() == []
    c = presets.workload(5).config(blockage_model="sphere")
    assert any("blockage_model" in f for f, _ in c.refusals())
    c = cfgmod.NRConfig(blockage=True, blockage_model="stochastic")
    assert c.refusals() == []
