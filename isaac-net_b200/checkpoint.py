"""Checkpoints in the reference's own format: the flat state dict that isaac-net's engine.state_dict() writes
(isaac_net/core/checkpoint.py:1-60, keys are the dotted attribute paths of the reference engine's object graph, e.g.
"net.ul.q.cap", "net.ul.ctr[tb_ok]", "net.rng.ctr[2]", "T") read into the B200 engine, and the B200 engine's state
written under those keys.

What moves, by reference key (the state a control step reads or writes):
  net.ul.<f>, net.ul.q.<f>          MAC / HARQ / BSR state and the frame queue
  net.h, net.spec, net.k_lin        fading state (Rician phasor and K)
  net.last_g, net.rng.episode, net.rng.ctr[2], T, epoch, _last_snr, _last_hid   clocks and counter-RNG counters
  net.assoc.<f>, net.ni_ul, net._pg  several cells: association, the gNBs' N+I, the last path gains
  radio.k / radio.phi, radio.ch.sf_los.*, radio.blk_a.field.*, radio.blk_a.{t,xk,yk,vel}   radio fields, blockage
  traffic.streams[i].<f>            the traffic models' per-robot state
  net.ul.ctr[<name>], net.ul.ntx_hist, net.ul.rv_tx, net.ul.rv_fail, net.ul.prb_used_env   counters
What does not: constants and scratch of the reference's object graph (tables, sizes, hooks, static buffers) and the
torch.Generator states of its traffic models and engine: the B200 engine's traffic stream is its own device stream
(the CUDA Philox replay or the counter-keyed stream), so a loaded engine continues with its own draws from there.
Counter totals the reference keeps as scalars (net.ul.ctr[...]) are placed in the first env's counter words, so
counters() returns the same totals."""
from __future__ import annotations

import re

import numpy as np
import torch

from . import _native as nat

# reference key -> the B200 engine's reference-state name (NRB200Engine.reference_state / load_reference_state)
_EXACT = {"T": "eng.T", "epoch": "eng.epoch", "_last_snr": "eng.last_snr", "_last_hid": "eng.last_hid",
          "net.h": "net.h", "net.spec": "net.spec", "net.k_lin": "net.k_lin", "net.last_g": "net.last_g",
          "net.ni_ul": "net.ni_ul", "net._pg": "net.pg", "net.rng.episode": "rng.episode",
          "net.rng.ctr[2]": "rng.ctr_step", "radio.k": "radio.k", "radio.phi": "radio.phi",
          "radio.ch.sf_los.k": "radio.sf_los.k", "radio.ch.sf_los.phi": "radio.sf_los.phi",
          "radio.blk_a.field.k": "radio.blk.k", "radio.blk_a.field.phi": "radio.blk.phi",
          "radio.blk_a.t": "radio.blk.t", "radio.blk_a.xk": "radio.blk.xk", "radio.blk_a.yk": "radio.blk.yk",
          "radio.blk_a.vel": "radio.blk.vel"}
_PREFIX = (("net.ul.q.", "q."), ("net.ul.", "ul."), ("net.assoc.", "assoc."))
_CTR = re.compile(r"^net\.ul\.ctr\[(\w+)\]$")
_SRC = re.compile(r"^traffic\.streams\[(\d+)\]\.(\w+)$")


def short_name(key):
    """The engine's reference-state name of a reference checkpoint key (None: not a state name of that kind)."""
    if key in _EXACT:
        return _EXACT[key]
    for a, b in _PREFIX:
        if key.startswith(a):
            return b + key[len(a):]
    return None


def _long_names():
    inv = {v: k for k, v in _EXACT.items()}

    def long(name):
        if name in inv:
            return inv[name]
        for a, b in _PREFIX:
            if name.startswith(b):
                return a + name[len(b):]
        return None
    return long


def _t(v):
    return v if torch.is_tensor(v) else torch.as_tensor(np.asarray(v))


def load(eng, sd, strict=False):
    """Load a reference state dict into `eng` (an NRB200Engine) in place; returns the keys it did not use.  strict:
    raise when a key that names engine state (MAC, queue, fading, clocks, RNG, association, radio, traffic model,
    counter) could not be placed."""
    known = set(eng._REF) | {"net.last_g", "rng.episode", "rng.ctr_step", "eng.T", "eng.epoch", "eng.last_snr",
                             "eng.last_hid", "net.pg"} | set(eng._FIELD_KEYS.get(eng.config.channel, ()))
    if eng.config.blockage:
        known |= {"radio.blk." + n for n in ("k", "phi", "t", "xk", "yk", "vel")}
    snap, unused, missed = {}, [], []
    ctr = {}
    src = {}
    for k, v in sd.items():
        m = _CTR.match(k)
        if m:
            ctr[m.group(1)] = v
            continue
        if k in ("net.ul.ntx_hist", "net.ul.rv_tx", "net.ul.rv_fail", "net.ul.prb_used_env"):
            ctr[k.rsplit(".", 1)[1]] = v
            continue
        m = _SRC.match(k)
        if m:
            src[(int(m.group(1)), m.group(2))] = v
            continue
        n = short_name(k)
        if n is not None and n in known and (torch.is_tensor(v) or isinstance(v, (int, float, np.ndarray))):
            if n in eng._REF and eng._REF[n] not in eng.st:
                missed.append(k)
                continue
            snap[n] = v
        else:
            unused.append(k)
    if "net.pg" in snap and eng.C == 1:
        snap.pop("net.pg")
    eng.load_reference_state({k: _t(v) for k, v in snap.items()})
    if eng.C > 1 and "net.pg" in snap:
        eng.pathgain = _t(snap["net.pg"]).to(eng.dev, torch.float32).clone()
    # traffic models' per-robot state
    tg = eng.traffic
    for (i, n), v in src.items():
        if tg is not None and i < len(tg.sources) and n in tg.sources[i].names + ("deferred",):
            getattr(tg.sources[i], n).copy_(_t(v).to(eng.dev))
        elif n in ("rob", "E", "R", "M", "tag", "step_ms", "slot_ms", "state", "gen", "rgen"):
            unused.append(f"traffic.streams[{i}].{n}")
        else:
            missed.append(f"traffic.streams[{i}].{n}")
    # counters: totals into env 0's words, per-env vectors into every env's
    if ctr:
        c = torch.zeros_like(eng.ctr)
        names = list(nat.CTR_NAMES) + (list(nat.LENA_CTR_NAMES) if eng.config.lena_mac_switches() else [])
        for i, n in enumerate(names):
            if n in ctr and n != "prb_used":
                c[0, i] = int(round(float(_t(ctr[n]))))
        if "prb_used_env" in ctr:
            c[:, nat.CTR_NAMES.index("prb_used")] = _t(ctr["prb_used_env"]).to(eng.dev).round().long()
        elif "prb_used" in ctr:
            c[0, nat.CTR_NAMES.index("prb_used")] = int(round(float(_t(ctr["prb_used"]))))
        H = eng.config.max_harq_tx + 1
        if "ntx_hist" in ctr:
            c[0, nat.CTR_NTX_HIST:nat.CTR_NTX_HIST + H] = _t(ctr["ntx_hist"]).to(eng.dev).round().long()[:H]
        for n, w in (("rv_tx", nat.CTR_RV_TX), ("rv_fail", nat.CTR_RV_FAIL)):
            if n in ctr:
                x = _t(ctr[n]).to(eng.dev).round().long()
                c[:, w:w + H] = x[:, :H] if x.dim() == 2 else x[None, :H]
        eng.ctr.copy_(c)
        if "prb_avail" in ctr:
            eng.prb_avail = float(_t(ctr["prb_avail"]))
    if strict and missed:
        raise KeyError(f"reference checkpoint keys this engine holds no state for: {missed}")
    return sorted(unused + missed)


def save(eng):
    """The engine's state under the reference's checkpoint keys (tensors cloned to the CPU, reference dtypes)."""
    long = _long_names()
    out = {}
    for n, v in eng.reference_state().items():
        k = long(n)
        if k is None:
            continue
        if n in ("eng.T", "net.last_g"):
            out[k] = int(v)
        else:
            out[k] = v.detach().clone().cpu()
    if eng.C == 1:
        out.pop("net._pg", None)
    tg = eng.traffic
    if tg is not None:
        for i, s in enumerate(tg.sources):
            for n in s.names + ("deferred",):
                out[f"traffic.streams[{i}].{n}"] = getattr(s, n).detach().clone().cpu()
    cu = eng.counters()["ul"]
    for n in list(nat.CTR_NAMES) + (list(nat.LENA_CTR_NAMES) if eng.config.lena_mac_switches() else []) + \
            ["prb_avail"]:
        out[f"net.ul.ctr[{n}]"] = torch.tensor(cu[n], dtype=torch.float32)
    c = eng.ctr.cpu()
    H = eng.config.max_harq_tx + 1
    out["net.ul.ntx_hist"] = torch.tensor(cu["ntx_hist"], dtype=torch.float32)
    out["net.ul.rv_tx"] = c[:, nat.CTR_RV_TX:nat.CTR_RV_TX + H].float()
    out["net.ul.rv_fail"] = c[:, nat.CTR_RV_FAIL:nat.CTR_RV_FAIL + H].float()
    out["net.ul.prb_used_env"] = c[:, nat.CTR_NAMES.index("prb_used")].float()
    return out
