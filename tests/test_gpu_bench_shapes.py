"""Parity at the benchmark shapes: the engine steps a workload at its full batch (config 2: 4096 envs x 32 robots,
config 5: 8192 x 48, config 4: 512 x 128 of its 8192 envs per GPU) and a strided sample of 64 envs, spread over the
grid's blocks (every 16th block of config 2 and a different env slot inside each block; every 128th / 8th block of
configs 5 and 4), is stepped by the oracle ("seq", same device) keyed by the same global env ids and fed the kernel's
own arrivals and path gains.  Every output and every state tensor of the sampled envs must be bitwise equal: this
covers the large-E index arithmetic, many-block grids and the multi-block paths the small golden cases never reach.
The whole-batch MAC counters are checked for conservation (every transmitted TB decodes or fails).  "2x" is config 2's
cell at 1024 envs with the switches of the reference's ul_v2l case that this engine builds (the 5G-LENA MAC switches,
the SR / BSR grant pipeline, fading off, the whole-band PSD, 128-frame buffers): the frame compaction over 128 slots
and the whole-band link adaptation at scale."""
import importlib

import pytest
import torch

from oracle.nr_oracle import OracleEngine

ib = importlib.import_module("isaac-net_b200")
presets = importlib.import_module("isaac-net_b200.presets")
ARR = ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")

pytestmark = pytest.mark.gpu


def _eq_t(a, b):
    if a.dtype.is_floating_point:
        return torch.equal(torch.nan_to_num(a, nan=12345.0), torch.nan_to_num(b, nan=12345.0)) and \
            torch.equal(torch.isnan(a), torch.isnan(b))
    return torch.equal(a, b)


def oracle_for_envs(cfg, ids, R, dev, seed):
    """An oracle over the envs with global ids `ids` (any set, not only a contiguous shard): its counter-RNG rows are
    keyed by those ids and its initial reset is redone under them with the episode counters rewound, as
    set_env_offset does for a contiguous shard (isaac_net/core/sharded.py:61-77)."""
    o = OracleEngine(cfg, len(ids), R, dev, seed=seed, reduce="seq")
    o.rng.env = ids.to(dev, torch.long).clone()
    o.rng.episode = o.rng.episode - 1
    o.reset(None)
    return o


def _rows(x, ids, E):
    """Rows `ids` of a per-env tensor (first axis E); other tensors (scalars) unchanged."""
    return x.index_select(0, ids) if torch.is_tensor(x) and x.dim() > 0 and x.shape[0] == E else x


SHAPES = {   # name: (envs, env ids of the sample, steps[, workload id, config overrides])
    "2": (4096, torch.arange(64) * 64 + torch.arange(64) % 4, 5),
    "5": (8192, torch.arange(64) * 128 + 127, 4),
    "4": (512, torch.arange(64) * 8 + 3, 4),
    "2x": (1024, torch.arange(64) * 16 + torch.arange(64) % 4, 6, 2,
           dict(pf_update="rbg", pf_avg_idle="freeze", ul_retx_sched="tdma", ul_amc_alloc="previous",
                ul_grant_model="bsr", tb_overhead_bytes=8, fading=False, ul_power="whole_band", gnb_nf_db=6.99697,
                frame_buffer=128, ue_tx_dbm=-6.0)),
}


@pytest.mark.parametrize("wl_i", sorted(SHAPES))
def test_full_batch_sample_equals_oracle(wl_i):
    E, ids, steps = SHAPES[wl_i][:3]
    wid, over = (SHAPES[wl_i][3], SHAPES[wl_i][4]) if len(SHAPES[wl_i]) > 3 else (int(wl_i), {})
    wl = presets.workload(wid)
    cfg = wl.config(**over)
    R = wl.R
    dev = torch.device("cuda:0")
    ids = ids.to(dev)
    eng = ib.make_engine("L2", E, R, dev, cfg, seed=wl.seed)
    orc = oracle_for_envs(cfg, ids, R, dev, wl.seed)
    st_k, st_o = eng.reference_state(), orc.reference_state()
    for k, v in st_o.items():
        assert _eq_t(_rows(st_k[k], ids, E), v), f"initial state {k}"
    mo = presets.Motion(wid, E, R, seed=11, step_ms=cfg.control_step_ms)
    pos = mo.current()
    reset_env = int(ids[5])
    for s in range(steps):
        if s == 2:                       # a partial reset of one sampled env and one env outside the sample
            eng.reset([reset_env, reset_env + 1])
            orc.reset([5])
        out = eng.step(None, pos.to(dev))
        a = eng.last_arrivals
        arr = {k: _rows(getattr(a, k), ids, E) for k in ARR}
        ref = orc.step(None, arr, pathgain=_rows(eng.pathgain, ids, E).clone())
        for k in ref:
            assert _eq_t(_rows(out[k], ids, E), ref[k]), f"step {s} output {k}"
        st_k, st_o = eng.reference_state(), orc.reference_state()
        for k, v in st_o.items():
            assert _eq_t(_rows(st_k[k], ids, E), v), f"step {s} state {k}"
        pos = mo.advance()
    c = eng.counters()["ul"]
    assert c["tb_new"] > 0
    assert c["tb_ok"] + c["tb_fail"] == c["tb_new"] + c["tb_retx"]
    assert 0 < c["prb_used"] <= c["prb_avail"]
