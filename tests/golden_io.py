"""Reading the golden fixtures (tests/golden/*.npz, written by tests/golden/make_golden.py)."""
import ast
import importlib
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ("1", "2", "4", "1s", "2s", "3", "3s", "3t", "5", "5s", "1b", "2r", "3r", "2v", "3v", "1v", "2g", "3g", "2w",
         "3w", "2x", "1m", "2m", "3m")
BSR_CASES = ("2g", "3g", "2x")   # the SR / BSR grant pipeline (ul_grant_model = "bsr") on one and three cells
# fixtures the oracle is pinned to but the kernels refuse: several cells with the reference's default fixed noise (no
# same-slot interference), the downlink with several cells, and the lena_like switches (wideband PF rate, PDCP
# arrival discard, per-packet overhead; "2V" the ul_v2l config with the shipped tables), ho_rlc="flush" with traffic
# models ("3h": the step's later arrivals survive a flush)
ORACLE_ONLY_CASES = ("3f", "2L", "3L", "2V", "3h")
ORACLE_ONLY_DL_CASES = ("d3", "d3s", "d3n", "d2L")
ORACLE_ONLY_POLICY_CASES = ("1pL",)
DL_CASES = ("d1", "d2", "d2s")   # the downlink MAC with CQI and DL traffic models (TDD patterns with D, S, U slots)
POLICY_CASES = ("1p",)   # policy submits + SNR input (tests/golden/make_golden.py POLICY_CASES)


class Golden:
    def __init__(self, case):
        self.case = case
        self.d = np.load(os.path.join(GOLDEN, f"cfg{case}.npz"))
        self.E, self.R, self.steps = int(self.d["E"]), int(self.d["R"]), int(self.d["steps"])
        self.workload_id = int(self.d["workload"])
        self.overrides = ast.literal_eval(str(self.d["overrides"]))
        self.resets = self.d["resets"]

    def workload(self):
        return importlib.import_module("isaac-net_b200.presets").workload(self.workload_id)

    def config(self):
        over = dict(self.overrides)
        if "dl_traffic" in self.d.files:     # the DL cases' traffic models (make_golden.dl_traffic)
            import sys
            sys.path.insert(0, GOLDEN)
            from make_golden import dl_traffic
            over["traffic"] = dl_traffic(self.workload_id, self.R)
        return self.workload().config(**over)

    def dl_arrivals(self, s):
        """The DL traffic arrivals of step s (DL cases), else None."""
        if f"s{s}/dlarr.valid" not in self.d.files:
            return None
        return {n: self.d[f"s{s}/dlarr.{n}"] for n in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")}

    def pos(self, s):
        return self.d[f"s{s}/pos"]

    def arrivals(self, s):
        return {n: self.d[f"s{s}/arr.{n}"] for n in ("valid", "nbytes", "slot", "tag", "prio", "dline", "det")}

    def outputs(self, s):
        pre = f"s{s}/out."
        return {k[len(pre):]: self.d[k] for k in self.d.files if k.startswith(pre)}

    def has_state(self, s):
        return f"s{s}/st.eng.T" in self.d.files

    def state(self, s):
        pre = "init/" if s < 0 else f"s{s}/st."
        return {k[len(pre):]: self.d[k] for k in self.d.files if k.startswith(pre)}

    def reset_ids(self, s):
        return np.nonzero(self.resets[s])[0].tolist()

    @property
    def legacy_step(self):
        return int(self.d["legacy_step"]) if "legacy_step" in self.d.files else -1

    def policy(self, s):
        """The policy case's inputs of step s: send, det, hid, tag, prio, dline, snr, cur_hid (numpy)."""
        pre = f"s{s}/in."
        return {k[len(pre):]: self.d[k] for k in self.d.files if k.startswith(pre)}
