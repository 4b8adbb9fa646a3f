"""inb_nr_step_noalloc (gain rows in the library's own device array) against inb_nr_step (gain rows in a caller buffer).

Two engines with the same seed step the same poses, one through each entry point; every output and every state
tensor must be bitwise equal after each of two consecutive steps (the second step reuses the array the first one
wrote); the three-cell case uses the multi-cell row layout (one row per UL slot holding every link's gain).  The
size check refuses a step whose gain rows exceed the array, before anything is launched, and only for calls that run
the fading or MAC launch.
This file is collected last and needs nothing from the other test files.
"""
import ctypes
import importlib

import pytest
import torch

ib = importlib.import_module("isaac-net_b200")
nat = importlib.import_module("isaac-net_b200._native")

pytestmark = pytest.mark.gpu


class _NoAllocLib:
    """The shared library with the step entry point swapped for inb_nr_step_noalloc."""

    def __init__(self, lib):
        self._lib = lib

    def __getattr__(self, name):
        return getattr(self._lib, name)

    @property
    def inb_nr_step(self):
        return self._lib.inb_nr_step_noalloc


def _same(a, b):
    if a.dtype.is_floating_point:
        return torch.equal(torch.isnan(a), torch.isnan(b)) and torch.equal(a.nan_to_num(nan=0.0), b.nan_to_num(nan=0.0))
    return torch.equal(a, b)


@pytest.mark.parametrize("wl_i,E,R", [(1, 64, 16), (2, 256, 32), (3, 32, 64)])
def test_noalloc_step_equals_step_on_two_consecutive_calls(wl_i, E, R):
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(wl_i)
    cfg = wl.config()
    engs = []
    for noalloc in (False, True):
        eng = ib.make_engine("L2", E, R, "cuda:0", cfg, seed=wl.seed)
        eng.graphs = False
        if noalloc:
            eng.L = _NoAllocLib(eng.L)
        engs.append(eng)
    mo = presets.Motion(wl_i, E, R, seed=3, step_ms=cfg.control_step_ms)
    for step in range(2):
        x = mo.current().to("cuda:0")
        mo.advance()
        out_a, out_b = (e.step(None, x) for e in engs)
        for k, v in out_a.items():
            if torch.is_tensor(v):
                assert _same(v, out_b[k]), f"step {step}: output {k}"
        st_a, st_b = (e.reference_state() for e in engs)
        for k, v in st_a.items():
            if torch.is_tensor(v):
                assert _same(v.to("cuda:0"), st_b[k].to("cuda:0")), f"step {step}: state {k}"
        assert int(engs[1].status.item()) == 0


def test_noalloc_refuses_oversize_gain_rows():
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(1)
    eng = ib.make_engine("L2", 8, 16, "cuda:0", wl.config(), seed=1)
    a = nat.InbStepArgs.from_buffer_copy(eng._args)
    a.pathgain_in = eng.st["olla"].data_ptr()      # any device pointer: the call returns before reading it
    a.p.K_rows = 1
    a.p.rows[0][1] = 12                           # one UL row
    a.p.E = nat.NOALLOC_GAIN_MAX // (2 * a.p.S * a.p.R) + 1
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert eng.L.inb_nr_step_noalloc(ctypes.byref(a), stream) == -10


def test_noalloc_size_check_only_for_the_gain_phases():
    """A call whose phases launch neither the fading nor the MAC kernel (phases = 1 with no radio launch configured:
    nothing runs) is not refused by the gain-row limit."""
    presets = importlib.import_module("isaac-net_b200.presets")
    wl = presets.workload(1)
    eng = ib.make_engine("L2", 8, 16, "cuda:0", wl.config(), seed=1)
    a = nat.InbStepArgs.from_buffer_copy(eng._args)
    a.pathgain_in = eng.st["olla"].data_ptr()
    a.p.K_rows = 1
    a.p.rows[0][1] = 12
    a.p.E = nat.NOALLOC_GAIN_MAX // (2 * a.p.S * a.p.R) + 1
    a.rm.on = 0
    a.phases = 1
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert eng.L.inb_nr_step_noalloc(ctypes.byref(a), stream) == 0
    a.phases = 2
    assert eng.L.inb_nr_step_noalloc(ctypes.byref(a), stream) == -10
