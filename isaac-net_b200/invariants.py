"""Host-side invariant checks of the engine state and of a step's outputs (debug / test mode: they synchronize).

There is no sanitizer on the path (the reference has none, and a device-side one is not available on every GPU
pool), so correctness of a run can be checked from the outside after any step:

  state_violations(engine)                  the per-robot state is well formed: 0 <= floor <= sent <= enq; bsr >= 0;
                                            HARQ states in {0, 1} with h_lo <= h_hi; the frame FIFO compacted
                                            (valid frames a prefix, at most F), every valid frame's bytes > 0 and
                                            frames in stream order (start non-decreasing, end = next start or less)
  step_violations(q_before, accepted, out)  conservation of messages over the step, per robot: frames queued when
                                            the step starts (policy submits included) + frames the traffic models
                                            add in the step = frames queued after + frames that left (delivered,
                                            timed out or dropped)

NRB200Engine.debug_invariants = True runs both after every step and raises on the first violation.
"""
from __future__ import annotations

import torch


def state_violations(engine):
    st, F = engine.st, engine.F
    bad = []
    floor_, sent, enq = st["floor_"], st["sent"], st["enq"]
    if bool(((floor_ < 0) | (floor_ > sent) | (sent > enq)).any()):
        bad.append("0 <= floor <= sent <= enq")
    if bool((st["bsr"] < 0).any()):
        bad.append("bsr >= 0")
    hs = st["h_state"]
    if bool(((hs != 0) & (hs != 1)).any()):
        bad.append("HARQ state in {0, 1}")
    if bool(((hs == 1) & (st["h_lo"] > st["h_hi"])).any()):
        bad.append("h_lo <= h_hi of a pending process")
    valid = st["cap"] >= 0
    if F > 1 and bool((valid[..., 1:] & ~valid[..., :-1]).any()):
        bad.append("valid frames form a prefix of the FIFO")
    if bool((valid & (st["end_"] <= st["start"])).any()):
        bad.append("a queued frame has bytes")
    if F > 1:
        both = valid[..., 1:] & valid[..., :-1]
        if bool((both & (st["start"][..., 1:] < st["end_"][..., :-1])).any()):
            bad.append("frames in stream order")
    if bool((valid & (st["end_"] > enq[..., None])).any()):
        bad.append("a queued frame ends at or before enq")
    return bad


def step_violations(q_before, accepted, out):
    gone = (out["delivered"] | out["timed_out"] | out["dropped"]).sum(-1)
    if bool((q_before + accepted != out["queue_len"] + gone).any()):
        return ["queued before + accepted = queued after + delivered + timed out + dropped"]
    return []


__all__ = ["state_violations", "step_violations"]
