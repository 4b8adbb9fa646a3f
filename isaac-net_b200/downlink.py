"""The engine's downlink (NRConfig.dl = True, one cell): the gNB-to-robot MacLink of isaac-net (DlMac,
isaac_net/core/mac_dl.py:1-49) next to the uplink.

The DL link has its own per-robot MAC / HARQ state and frame queue (the reference's net.dl and net.dl.q), its own
counters, its DL traffic models (direction="dl", their own generator seeded as NREngine does, engine.py:369-380) and
the policy's add_dl_frames.  Its slots run in the same fused MAC kernel (the DL instance) and the same finish kernel,
launched inside inb_nr_step through InbStepArgs.dl right after the fading: the kernel finds the DL data rows, the CQI
reports and the HARQ-ACK slots of the schedule in InbParams.rows_dl and the gain of those rows in the step's gain
buffer.  This module builds the DL launch arguments from the uplink's each step and keeps the host-side state
(reset, add_dl_frames, counters, outputs)."""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _native as nat
from .traffic import DeviceTrafficGen, TrafficGen, generates

# per-robot state of a MacLink and its queue (mac.py:67-81, queues.py:45-61): name -> (dtype, initial value, dims)
_SCALARS = {"sent": 0, "floor_": 0, "bsr": 0, "sr_t": -1, "last_tx": -1, "enq": 0}
_HARQ = ("h_state", "h_lo", "h_hi", "h_ready", "h_ntx", "h_mcs", "h_tbs", "h_nsb")
_QUEUE_L = {"cap": -1, "start": 0, "end_": 0, "cls": 0, "hid": 0, "tag": 0, "prio": 0}
# reference names of the DL state (the reference's net.dl.<f>, net.dl.q.<f>) -> this module's buffers
REF = {**{"dl." + n: n for n in ("sent", "olla", "avg", "bsr", "sr_t", "last_tx", "csi", "h_state", "h_lo", "h_hi",
                                 "h_ready", "h_ntx", "h_mcs", "h_tbs", "h_nsb", "h_comb")},
       "dl.floor": "floor_", "dq.cap": "cap", "dq.start": "start", "dq.end": "end_", "dq.lost": "lost",
       "dq.fin": "fin", "dq.enq": "enq", "dq.cls": "cls", "dq.off": "off", "dq.tag": "tag", "dq.prio": "prio",
       "dq.dline": "dline"}


def _f32(x):
    return float(np.float32(x))


class Downlink:
    def __init__(self, eng):
        cfg, E, R, S, P, F, dev = eng.config, eng.E, eng.R, eng.S, eng.P, eng.F, eng.dev
        self.eng = eng
        full = lambda shape, dt, v: torch.full(shape, v, dtype=dt, device=dev)   # noqa: E731
        L, b = torch.long, torch.bool
        st = {n: full((E, R), L, v) for n, v in _SCALARS.items()}
        st["olla"], st["avg"] = full((E, R), torch.float32, 0.0), full((E, R), torch.float32, 100.0)
        st["csi"] = full((E, R, S), torch.float32, 0.0)
        for n in _HARQ:
            st[n] = full((E, R, P), L, 0)
        st["h_comb"] = full((E, R, P), torch.float32, 0.0)
        for n, v in _QUEUE_L.items():
            st[n] = full((E, R, F), L, v)
        st["lost"], st["det"] = full((E, R, F), b, False), full((E, R, F), b, False)
        st["fin"] = full((E, R, F), torch.float64, math.inf)
        st["off"] = full((E, R, F), torch.float64, 0.0)
        st["dline"] = full((E, R, F), torch.float64, math.inf)
        self.st = st
        self.ctr = torch.zeros(E, nat.NCTR, dtype=torch.long, device=dev)
        self.prb_avail = 0.0
        # the DL MCS cap and whether the thresholds below it are non-decreasing (the kernel's binary search)
        tab = eng.tab
        cap = tab.M - 1 if cfg.dl_mcs_max is None else min(int(cfg.dl_mcs_max), tab.M - 1)
        self.mcs_max = cap
        thr = tab.thr_ref[: cap + 1].cpu()
        self.thr_mono = int(bool((thr[1:] >= thr[:-1]).all()))
        # the reference SINR of a DL PRB: gNB power spread over the carrier, the UE's noise (NRNet.step_rx,
        # nr_engine.py:624-631)
        self.ref0 = _f32(cfg.gnb_tx_dbm - 10 * math.log10(cfg.nprb))
        self.noise = _f32(cfg.noise_dbm_per_prb("ue"))
        # link-adaptation tables of every DL data-symbol count of the pattern (a D slot's, an S slot's), stacked
        nsyms = sorted({cfg.slot_symbols(g)[0] for g in range(len(cfg.tdd_pattern))} - {0})
        self.nsym_tab = [0] * 16
        sets = [tab.la_tables(n) for n in nsyms]
        for j, n in enumerate(nsyms):
            self.nsym_tab[n] = j
        self.la_sets = max(1, len(sets))
        self.la = [torch.cat([s_[i] for s_ in sets]).contiguous() for i in range(4)] if sets else \
            [tab.la_tbs, tab.la_i0, tab.la_wi, tab.la_ncb]
        self.traffic = self.dtraffic = None
        if generates(cfg.traffic, "dl"):
            dseed = (int(eng.seed) * 2862933555777941757 + 3037000493) % 2 ** 62
            self.traffic = TrafficGen(cfg.traffic, E, R, dev, cfg.control_step_ms, eng.N, seed=dseed, direction="dl")
            self.dtraffic = DeviceTrafficGen(self.traffic, eng.L) if DeviceTrafficGen.supports(self.traffic) else None
        self._keep = None

    # ------------------------------------------------------------------ state
    def state_struct(self):
        s = nat.InbState()
        for n in nat.STATE_FIELDS:
            t = self.st.get(n)
            setattr(s, n, t.data_ptr() if t is not None else None)
        return s

    def reset(self, m=None):
        """Every DL state tensor of the envs of mask m [E] (None: all) back to its initial value (MacLink.reset,
        mac.py:176-189); the DL traffic models reset their streams; a full reset also clears the counters."""
        if self.traffic is not None:
            self.traffic.reset(m)
        init = dict(_SCALARS, olla=0.0, avg=100.0, csi=0.0, h_comb=0.0, lost=False, det=False, fin=math.inf, off=0.0,
                    dline=math.inf, **{n: 0 for n in _HARQ}, **_QUEUE_L)
        for n, t in self.st.items():
            if m is None:
                t.fill_(init[n])
            else:
                t.masked_fill_(m.view(-1, *([1] * (t.dim() - 1))).expand_as(t), init[n])
        if m is None:
            self.ctr.zero_()
            self.prb_avail = 0.0

    def add_frames(self, T, nbytes, cls=None):
        """NRNet.add_dl_frames (nr_engine.py:489-495): one DL frame of nbytes [E,R] per robot (0 = none) at control
        step T; cls [E,R] tags it.  Returns accepted [E,R]."""
        st, F, dev = self.st, self.eng.F, self.eng.dev
        nb_f = nbytes.to(dev, torch.float32)
        cnt = (st["cap"] >= 0).sum(-1)
        acc = (nb_f > 0) & (cnt < F)
        i = cnt.clamp(max=F - 1)
        oh = (i[..., None] == torch.arange(F, device=dev)) & acc[..., None]
        nb = nb_f.round().long()
        put = lambda n, v: st[n].copy_(torch.where(oh, v[..., None].to(st[n].dtype) if torch.is_tensor(v)  # noqa: E731
                                                   else torch.full_like(st[n], v), st[n]))
        put("cap", T)
        put("start", st["enq"])
        put("end_", st["enq"] + nb)
        put("lost", False)
        put("fin", math.inf)
        put("off", 0.0)
        put("tag", 0)
        put("prio", 0)
        put("dline", math.inf)
        if cls is not None:
            put("cls", cls.to(dev, torch.long))
        st["enq"].add_(nb * acc)
        return acc

    # ------------------------------------------------------------------ one step
    # DL outputs: always, and with DL traffic models; (name, dtype, shape) and the InbOutputs field each goes to
    OUT_BASE = (("dl_newest", torch.long, "ER", "newest"), ("dl_queue_len", torch.long, "ER", "queue_len"))
    OUT_TRAFFIC = (("dl_delivered", torch.bool, "ERF", "delivered"), ("dl_lost", torch.bool, "ERF", "lost_any"),
                   ("dl_delay", torch.float32, "ERF", "delay"), ("dl_tag", torch.long, "ERF", "tag"),
                   ("dl_generated", torch.bool, "ERF", "generated"), ("dl_bytes", torch.long, "ERF", "bytes"),
                   ("dl_deadline_miss", torch.bool, "ERF", "deadline_miss"),
                   ("gen_dl_accepted", torch.long, "ER", "gen_accepted"), ("gen_dl_bytes", torch.long, "ER", "gen_bytes"))

    def out_spec(self):
        """(name, dtype, shape, InbOutputs field) of this link's step outputs."""
        E, R, F = self.eng.E, self.eng.R, self.eng.F
        dims = {"ER": (E, R), "ERF": (E, R, F)}
        outs = self.OUT_BASE + (self.OUT_TRAFFIC if self.traffic is not None else ())
        return [(n, dt, dims[d], f) for n, dt, d, f in outs]

    def _base_args(self, a):
        """The DL launch arguments from the uplink's `a` (already filled): the DL parameters, state and counters."""
        d = nat.InbStepArgs.from_buffer_copy(a)
        p = d.p
        p.mcs_max, p.thr_mono = self.mcs_max, self.thr_mono
        p.phr_cap = p.tdma = p.amc_prev = p.bsr_on = p.whole_band = 0   # uplink-only switches
        p.ul_ref0, p.noise_prb = self.ref0, self.noise
        p.la_sets = self.la_sets
        for n in range(16):
            p.dl_nsym_tab[n] = self.nsym_tab[n]
        d.t.la_tbs, d.t.la_i0, d.t.la_wi, d.t.la_ncb = (x.data_ptr() for x in self.la)
        d.s = self.state_struct()
        d.ctr = self.ctr.data_ptr()
        d.trace = d.det_hid = d.dl = None
        return d

    def _set_arrivals(self, d, arr, keep):
        p = d.p
        if arr is None:
            p.M = 0
            for n in nat.ARR_FIELDS:
                setattr(d.a, n, None)
            return
        for n in nat.ARR_FIELDS:
            v = getattr(arr, n).contiguous()
            keep.append(v)
            setattr(d.a, n, v.data_ptr())
        p.M = arr.valid.shape[-1]
        if p.M > 64:
            raise ValueError(f"{p.M} DL traffic arrivals per robot per step (at most 64)")

    def graph_args(self, a, arr, offsets, bias):
        """The DL launch arguments of a step captured in a CUDA graph (pose input, no SNR input): as launch_args, with
        the arrivals `arr` of the DL traffic models (produced inside the graph) and every output as its byte offset
        plus `bias` from the output block whose address the graph's kernels read (InbStepArgs.o_base)."""
        d = self._base_args(a)
        keep = []
        self._set_arrivals(d, arr if self.traffic is not None else None, keep)
        o = nat.InbOutputs()
        for n, dt, shape, f in self.out_spec():
            setattr(o, f, bias + offsets[n])
        d.o = o
        self._graph_keep = getattr(self, "_graph_keep", []) + [d, keep]
        return d

    def launch_args(self, a, snr=None, dl_snr=None, arrivals=None):
        """The DL launch arguments of this step from the uplink's `a` (already filled): the DL parameters, state,
        counters, arrivals and a fresh set of DL outputs.  snr / dl_snr: the step's SNR input (the DL reference is
        dl_snr, else snr + dl_snr_offset_db, NRNet.step, nr_engine.py:651-653); arrivals: given DL arrivals in place
        of the DL traffic models' (tests feed the reference's).  Returns (args, outputs)."""
        eng, cfg, E, R, S, F, dev = self.eng, self.eng.config, self.eng.E, self.eng.R, self.eng.S, self.eng.F, \
            self.eng.dev
        d = self._base_args(a)
        p = d.p
        keep = []
        if snr is not None:
            dref = dl_snr.to(dev, torch.float32) if dl_snr is not None else snr.to(dev, torch.float32) + \
                cfg.dl_snr_offset_db
            ref = (dref if dref.dim() == 3 else dref[..., None].expand(E, R, S)).contiguous()
            keep.append(ref)
            d.ul_ref_in = ref.data_ptr()
        arr = None
        if self.traffic is not None:
            if arrivals is not None:
                arr = arrivals
            else:
                arr = self.dtraffic.step() if self.dtraffic is not None else self.traffic.step(eng.clock, None)
            self.last_arrivals = arr
        self._set_arrivals(d, arr, keep)
        out = {}
        o = nat.InbOutputs()
        for n, dt, shape, f in self.out_spec():
            out[n] = torch.empty(shape, dtype=dt, device=dev)
            setattr(o, f, out[n].data_ptr())
        d.o = o
        self._keep = (d, keep, out)          # the launch reads them (and `d` lives in host memory)
        return d, out

    def counters(self):
        return self.eng.fold_counters(self.ctr.sum(0), self.prb_avail)["ul"]
