"""The fused kernel against the reference's own op sequence on the same CUDA device: the oracle in "aten" mode runs
every reduction as the reference calls it (torch.logsumexp, sum, mean, argsort: isaac_net/core/phy.py:311-328,
mac.py:276-300), so on cuda:0 it is the reference's arithmetic on the GPU, the primary oracle for bit-exact integers.
The kernel sums the RBG axis left to right (the "seq" mode it equals bitwise, test_gpu_parity.py); these tests
measure what that order changes against torch's CUDA reductions.

Measured on a B200 over every golden case (free-running with the kernel's arrivals and path gains fed to the oracle,
and teacher-forced by loading the oracle's state into the engine before every step): no integer output and no
integer state ever differs.  What does differ, and the bound each test writes down:
  * h_comb (the chase-combining sum, float state): an ulp of the EESM logsumexp moves 10^(eff/10) by an ulp in a few
    HARQ processes per case (relative 1e-5 bound).  With the whole-band PSD (ul_power="whole_band") the per-RBG SINRs
    of a grant are low, so the EESM's lse - lnw is a small difference of two ~log(S) terms and one ulp of either is a
    larger share of it: relative 1e-4 bound there (the CPU's logsumexp order against the left-to-right sum: 9.6e-6);
  * sinr_db with several cells: the serving SINR subtracts 10 log10(mean over RBGs of the N+I) from terms of ~100 dB,
    and torch's CUDA mean adds the RBGs in its own order, so the result moves by a few ulps of a 100 dB term (bound:
    1e-5 relative + 3.1e-5 dB, 4 ulps of a 128 dB value), which for SINRs near 0 dB is more than 1e-5 relative.
Every other float output is bitwise equal.  With the kernel's own radio against the oracle's radio on CUDA (configs
1, 3, 5 and the blockage / TTT variants) the path gains differ by at most 5e-3 dB (the kernel rounds the plane-wave
phases as the reference's CPU einsum does, torch's CUDA einsum rounds them its own way; the radio-map bilinear
weights take the same ulps) and the integer outputs are still equal."""
import importlib

import pytest
import torch

from golden_io import CASES, DL_CASES, Golden
from oracle.nr_oracle import OracleEngine

ib = importlib.import_module("isaac-net_b200")
ARR = ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")
SINR_ATOL = 3.1e-5          # dB: 4 ulps of a 128 dB term
RADIO_ATOL = 5e-3           # dB: path-gain difference of the two radio evaluations

pytestmark = pytest.mark.gpu


def _arr(eng):
    return {k: getattr(eng.last_arrivals, k) for k in ARR}


def _dl_arr(eng):
    """The DL arrivals the engine's DL traffic models made this step (None without the downlink)."""
    if eng.dl is None or getattr(eng.dl, "last_arrivals", None) is None:
        return None
    return {k: getattr(eng.dl.last_arrivals, k) for k in ARR}


def _snap(orc):
    """The oracle's state under the reference names, with the clock and the last schedule key the engine loads."""
    s = dict(orc.reference_state())
    s["eng.T"] = torch.tensor(orc.T)
    s["net.last_g"] = torch.tensor(-1 if orc.last_g is None else orc.last_g)
    return s


def _check_outputs(out, ref, s, sinr_atol):
    for k, v in ref.items():
        a = out[k]
        if not v.dtype.is_floating_point:
            n = int((a != v).sum())
            assert n == 0, f"step {s}: {n} elements of integer output {k} differ"
        elif k == "sinr_db":
            d = (a.double() - v.double()).abs()
            assert bool((d <= 1e-5 * v.double().abs() + sinr_atol).all()), (s, k, float(d.max()))
        else:
            assert torch.equal(torch.isnan(a), torch.isnan(v)), (s, k)
            assert torch.equal(torch.nan_to_num(a, 0.0), torch.nan_to_num(v, 0.0)), (s, k)


def _check_state(eng, orc, s, radio):
    st_k, st_o = eng.reference_state(), orc.reference_state()
    comb_rtol = 1e-4 if eng.config.ul_power == "whole_band" else 1e-5
    for k, v in st_o.items():
        a = st_k[k]
        if not v.dtype.is_floating_point:
            assert torch.equal(a, v), f"step {s} integer state {k}"
        elif radio and k == "net.pg":
            assert bool(((a - v).abs() <= RADIO_ATOL).all()), (s, k)
        elif radio:     # 5e-3 dB of path gain is 0.12 % in linear terms (N+I, combining sums)
            assert torch.allclose(a, v, rtol=2e-3, atol=0.0, equal_nan=True), f"step {s} float state {k}"
        else:
            rtol = comb_rtol if k.endswith("h_comb") else 1e-5
            assert torch.allclose(a, v, rtol=rtol, atol=0.0, equal_nan=True), f"step {s} float state {k}"


def _run(case, teacher_forced, radio=False):
    g = Golden(case)
    cfg, wl = g.config(), g.workload()
    dev = torch.device("cuda:0")
    eng = ib.make_engine("L2", g.E, g.R, dev, cfg, seed=wl.seed)
    orc = OracleEngine(cfg, g.E, g.R, dev, seed=wl.seed, reduce="aten")
    for s in range(g.steps):
        ids = g.reset_ids(s)
        if ids:
            eng.reset(ids)
            orc.reset(ids)
        if teacher_forced:
            eng.load_reference_state(_snap(orc))
        pos = torch.as_tensor(g.pos(s)).to(dev)
        out = eng.step(None, pos)
        if radio:
            ref = orc.step(pos, _arr(eng), dl_arrivals=_dl_arr(eng))
            d = (eng.pathgain.reshape(orc.pathgain.shape) - orc.pathgain).abs().max().item()
            assert d <= RADIO_ATOL, (s, d)
        else:
            ref = orc.step(None, _arr(eng), pathgain=eng.pathgain.clone(), dl_arrivals=_dl_arr(eng))
        _check_outputs(out, ref, s, RADIO_ATOL if radio else SINR_ATOL)
        _check_state(eng, orc, s, radio)


@pytest.mark.parametrize("case", CASES + DL_CASES)
def test_kernel_equals_aten_cuda_free_running(case):
    """Every step of every golden case, the oracle fed the kernel's arrivals and path gains: integer outputs and
    integer state bitwise, floats as the module docstring bounds them."""
    _run(case, teacher_forced=False)


@pytest.mark.parametrize("case", CASES + DL_CASES)
def test_kernel_equals_aten_cuda_teacher_forced(case):
    """As above with the engine loaded with the oracle's state before every step (no carry-over of any difference)."""
    _run(case, teacher_forced=True)


@pytest.mark.parametrize("case", ("1", "3", "3t", "5", "5s", "1b"))
def test_kernel_radio_free_running_vs_aten_cuda(case):
    """Poses through both radios (the kernel's and the oracle's torch evaluation on CUDA), free-running: path gains
    within 5e-3 dB, integer outputs bitwise equal over the whole case."""
    _run(case, teacher_forced=False, radio=True)
