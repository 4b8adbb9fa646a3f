"""Known answers that pin the path's building blocks: the counter-RNG hash (isaac-net tests/test_rng_levels.py:296-311,
tests/test_nr_fast.py:108-124), TS 38.214 TBS / segmentation examples (tests/test_nr_phy.py:23-60) and the NRConfig
carrier quantities (test_nr_phy.py:53-60), for the product's host code and the oracle alike."""
import importlib

import torch

from oracle import nr_oracle as O

eng = importlib.import_module("isaac-net_b200.engine")
phy = importlib.import_module("isaac-net_b200.phy")
NRConfig = importlib.import_module("isaac-net_b200").NRConfig

XS = (0, 1, 2, 12345, 0xDEADBEEF, 0xFFFFFFFF)
MIX = [0, 2261973619, 229111015, 2258480790, 707447538, 2578835075]


def test_mix32_pins():
    assert [O.mix32(x) for x in XS] == MIX
    assert [eng._mix32(x) for x in XS] == MIX
    assert O.mix32(torch.tensor(XS, dtype=torch.int64)).tolist() == MIX


def test_counter_uniform_pins():
    # CounterRNG(12345, 3): reset (episode 0), one STEP tick, uniform(STEP, stream 1, 4)
    s0 = O.seed_key(12345)
    assert s0 == eng.seed_key(12345)
    env = torch.arange(3)
    base = O.key_of(s0, env, torch.zeros(3, dtype=torch.long), O.STEP, torch.ones(3, dtype=torch.long), 1)
    u = O.uniforms(base, 4)
    bits = (u.double() * 2 ** 24).to(torch.int64).tolist()
    assert bits == [[10567228, 16700380, 16191287, 1599467], [268848, 15326424, 8181290, 3147942],
                    [13082027, 15096436, 9686026, 361841]]


def test_key_chain_matches_scalar_reference():
    seed, E = 2 ** 40 + 77, 3
    s0 = O.mix32(O.mix32(seed & 0xFFFFFFFF) ^ O.salt(seed >> 32))
    assert s0 == O.seed_key(seed)
    env = torch.arange(E)
    base = O.key_of(s0, env, torch.zeros(E, dtype=torch.long), O.STEP, torch.full((E,), 2), (O.BLER_UL << 16) | 5)
    u = O.uniforms(base, 7)
    for e in range(E):
        h = O.mix32(s0 ^ O.salt(e))
        h = O.mix32(h ^ O.salt(0))
        h = O.mix32(h ^ O.salt(O.STEP))
        h = O.mix32(h ^ O.salt(2))
        b = O.mix32(h ^ O.salt((O.BLER_UL << 16) | 5))
        for i in range(7):
            x = O.mix32(O.mix32((b + i * 0x9E3779B9) & 0xFFFFFFFF) ^ b)
            assert float(u[e, i]) == (x >> 8) / 16777216.0


def _tbs(mod, qm, r, n, nsym, dmrs):
    T = lambda v: torch.tensor(float(v))
    return int(mod.tbs_38214(T(qm), T(r), T(n), nsym, dmrs))


def test_tbs_spec_examples():
    for mod in (O, phy):
        assert _tbs(mod, 2, 120 / 1024, 1, 12, 12) == 24
        assert _tbs(mod, 6, 948 / 1024, 50, 12, 12) == 36896
        assert _tbs(mod, 4, 340 / 1024, 10, 12, 12) == 1800
        assert _tbs(mod, 2, 193 / 1024, 273, 13, 12) == 14856
        cb, c = mod.segment(torch.tensor(36896), torch.tensor(948 / 1024))
        assert int(cb) == 7408 and int(c) == 5


def test_config_carrier_quantities():
    c1 = NRConfig(mu=1, bandwidth_mhz=20)
    c0 = NRConfig(mu=0, bandwidth_mhz=20, tdd_pattern="DDDSU")
    c2 = NRConfig(mu=2, bandwidth_mhz=100, tdd_pattern="DDSU")
    c3 = NRConfig(mu=1, bandwidth_mhz=100, tdd_pattern="DSUUU")
    assert (c1.nprb, c1.rbg, c1.n_subbands, c1.subband_prbs[-1]) == (51, 4, 13, 3)
    assert (c0.nprb, c0.rbg) == (106, 8) and (c2.nprb, c2.rbg, c2.n_subbands) == (135, 8, 17)
    assert (c3.nprb, c3.rbg, c3.n_subbands) == (273, 16, 18)


def test_bsr_level_table_matches_the_oracle():
    """The MAC kernel's short-BSR level table (csrc/nr_bsr.cuh, TS 38.321 Table 6.1.3.1-1) equals the oracle's, which
    the BSR fixtures pin to the reference (isaac_net/core/mac_ul.py:38-42)."""
    import os
    import re
    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "isaac-net_b200", "csrc",
                            "nr_bsr.cuh")).read()
    body = re.search(r"kBsrLevels\[64\] = \{([^}]*)\}", src).group(1)
    assert [int(x) for x in body.replace("\n", " ").split(",")] == list(O.BSR_LEVELS)


def test_whole_band_power_settings():
    """ul_power="whole_band" runs, with or without a PHR cap (the whole-band PSD has none, mac_ul.py:154-168); with
    ul_amc_alloc="previous" it needs the per-RBG PF instance; 128-frame buffers run, 129 are refused; the split the
    kernel receives, float32(10 log10(nprb / snr_ref_prbs)), rounds the reference's float64 value."""
    import math
    ok = NRConfig(ul_power="whole_band", phr_cap=True)
    assert ok.refusals() == []
    lena = NRConfig(ul_power="whole_band", ul_amc_alloc="previous", pf_update="rbg", frame_buffer=128)
    assert lena.refusals() == []
    assert any("whole_band" in r[0] for r in NRConfig(ul_power="whole_band", ul_amc_alloc="previous").refusals())
    assert any("frame_buffer" in r[0] for r in NRConfig(frame_buffer=129).refusals())
    wb = 10 * math.log10(ok.nprb / ok.snr_ref_prbs)
    assert abs(float(torch.tensor(wb, dtype=torch.float32)) - wb) <= 1e-6 * abs(wb)


def test_several_cells_need_the_interference_the_kernels_add():
    """The reference adds the other cells' UL interference only with thermal noise and ul_interference on
    (nr_engine.py:220); the kernels always add it, so a multi-cell config without it is refused, and so is the
    downlink with several cells.  The oracle runs both (fixtures cfg3f, cfgd3*)."""
    import importlib
    wl3 = importlib.import_module("isaac-net_b200.presets").workload(3)
    assert wl3.config().noise_model == "thermal" and wl3.config().refusals() == []
    for over in (dict(noise_model="fixed"), dict(ul_interference=False), dict(dl=True, tdd_pattern="DDDSU")):
        assert wl3.config(**over).refusals(), over
    assert NRConfig(noise_model="fixed").refusals() == []          # one cell: no interference either way
    # a flush at handover under traffic models keeps the step's later arrivals in the reference (fixture cfg3h)
    assert wl3.config(ho_rlc="flush").refusals()
    assert wl3.config(ho_rlc="flush", traffic=None).refusals() == []
