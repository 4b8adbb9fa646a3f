"""Link-abstraction tables of the B200 NR engine, built once per engine on its device.

The tables restate isaac-net's PHY (isaac_net/core/phy.py): the 38.214 MCS tables (phy.py:20-30), the exact TBS of
TS 38.214 5.1.3.2 (phy.py:77-106), LDPC segmentation (phy.py:109-119), the SINR-to-BLER curves and the 10 % BLER
thresholds (phy.py:234-243, 263-295).  They are computed with torch operations on the engine's device, so the
values (float32 / float64 rounding included) are the ones the reference's own torch code computes on that device.
Link adaptation then reads TBS, code-block index / weight and code-block count per (PRBs, MCS) from
[NPRB + 1, M] tables instead of recomputing them per robot.
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

MCS_T1 = [(2, 120), (2, 157), (2, 193), (2, 251), (2, 308), (2, 379), (2, 449), (2, 526), (2, 602), (2, 679),
          (4, 340), (4, 378), (4, 434), (4, 490), (4, 553), (4, 616), (4, 658), (6, 438), (6, 466), (6, 517),
          (6, 567), (6, 616), (6, 666), (6, 719), (6, 772), (6, 822), (6, 873), (6, 910), (6, 948)]
MCS_T2 = [(2, 120), (2, 193), (2, 308), (2, 449), (2, 602), (4, 378), (4, 434), (4, 490), (4, 553), (4, 616),
          (4, 658), (6, 466), (6, 517), (6, 567), (6, 616), (6, 666), (6, 719), (6, 772), (6, 822), (6, 873),
          (8, 682.5), (8, 711), (8, 754), (8, 797), (8, 841), (8, 885), (8, 916.5), (8, 948)]
# TS 38.214 Table 5.1.3.2-1 (TBS for N_info <= 3824)
TBS_TABLE = (24, 32, 40, 48, 56, 64, 72, 80, 88, 96, 104, 112, 120, 128, 136, 144, 152, 160, 168, 176, 184, 192,
             208, 224, 240, 256, 272, 288, 304, 320, 336, 352, 368, 384, 408, 432, 456, 480, 504, 528, 552, 576,
             608, 640, 672, 704, 736, 768, 808, 848, 888, 928, 984, 1032, 1064, 1128, 1160, 1192, 1224, 1256, 1288,
             1320, 1352, 1416, 1480, 1544, 1608, 1672, 1736, 1800, 1864, 1928, 2024, 2088, 2152, 2216, 2280, 2408,
             2472, 2536, 2600, 2664, 2728, 2792, 2856, 2976, 3104, 3240, 3368, 3496, 3624, 3752, 3824)
DATA = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data", "phy_tables.npz")


def tbs_38214(qm, r, n_prb, nsym, dmrs=12, oh=0):
    """TBS in bits (int64) of TS 38.214 5.1.3.2 steps 1-4, elementwise in float64."""
    dev = n_prb.device
    f64 = lambda x: (x.to(torch.float64) if torch.is_tensor(x)
                     else torch.full((), float(x), dtype=torch.float64, device=dev))
    qm, r, n_prb, nsym = f64(qm), f64(r), f64(n_prb), f64(nsym)
    n_re = torch.clamp(12 * nsym - f64(dmrs) - f64(oh), max=156) * n_prb
    n_info = n_re * r * qm
    n = torch.clamp(torch.floor(torch.log2(n_info.clamp(min=1.0))) - 6, min=3)
    q_small = torch.clamp(2 ** n * torch.floor(n_info / 2 ** n), min=24)
    table = torch.tensor(TBS_TABLE, dtype=torch.float64, device=dev)
    small = table[torch.searchsorted(table, q_small.contiguous(), right=False).clamp(max=len(TBS_TABLE) - 1)]
    n4 = torch.floor(torch.log2((n_info - 24).clamp(min=1.0))) - 5
    q4 = torch.clamp(2 ** n4 * torch.floor((n_info - 24) / 2 ** n4 + 0.5), min=3840)
    c_lo = torch.ceil((q4 + 24) / 3816)
    tb_lo = 8 * c_lo * torch.ceil((q4 + 24) / (8 * c_lo)) - 24
    c_hi = torch.ceil((q4 + 24) / 8424)
    tb_hi = 8 * c_hi * torch.ceil((q4 + 24) / (8 * c_hi)) - 24
    tb_mid = 8 * torch.ceil((q4 + 24) / 8) - 24
    large = torch.where(r <= 0.25, tb_lo, torch.where(q4 > 8424, tb_hi, tb_mid))
    tbs = torch.where(n_info <= 3824, small, large)
    return torch.where(n_re > 0, tbs, torch.zeros_like(tbs)).long()


def segment(tbs, r):
    """LDPC base graph and code-block segmentation (TS 38.212 5.2.2 / 7.2.2): (code-block size, blocks), float64."""
    tbs = tbs.double()
    r = r.to(torch.float64)
    bg2 = (tbs <= 292) | ((tbs <= 3824) & (r <= 0.67)) | (r <= 0.25)
    kcb = torch.where(bg2, torch.full_like(tbs, 3840.0), torch.full_like(tbs, 8448.0))
    b = tbs + torch.where(tbs > 3824, torch.full_like(tbs, 24.0), torch.full_like(tbs, 16.0))
    c = torch.where(b <= kcb, torch.ones_like(b), torch.ceil(b / (kcb - 24)))
    bp = torch.where(c > 1, b + 24 * c, b)
    return bp / c, c


class PhyTables:
    """Every table inb_nr_step reads, on `device`, for one config."""

    def __init__(self, cfg, S_prbs, device):
        dev = torch.device(device)
        mcs = MCS_T1 if cfg.mcs_table == 1 else MCS_T2
        self.M = M = len(mcs)
        self.qm = torch.tensor([q for q, _ in mcs], dtype=torch.float32, device=dev)
        self.r = torch.tensor([c / 1024 for _, c in mcs], dtype=torch.float32, device=dev)
        self.se = (self.qm * self.r).contiguous()
        d = np.load(DATA)
        bler = torch.tensor(d[f"bler_t{cfg.mcs_table}"], device=dev)[None]
        self.bler = bler.reshape(-1).contiguous()
        grid = torch.tensor(d["snr_grid"], device=dev)
        axis = torch.tensor(d["cbs_axis"], device=dev)
        self.beta = torch.tensor(d[f"beta_t{cfg.mcs_table}"], device=dev).contiguous()
        _, _, self.C, self.G = bler.shape
        self.s0 = float(grid[0]); self.ds = float(grid[1] - grid[0])
        self.c0 = float(axis[0]); self.dc = float(axis[1] - axis[0])
        cap = cfg.ul_mcs_max
        self.mcs_max = M - 1 if cap is None else min(int(cap), M - 1)
        # 10 % BLER threshold of every MCS for one 10-PRB RBG (PHY.set_target, phy.py:234-243)
        ok = bler <= cfg.bler_target
        first = torch.where(ok.any(-1), ok.float().argmax(-1), torch.full(ok.shape[:-1], self.G - 1, device=dev))
        thr = grid[first]
        tb = tbs_38214(self.qm, self.r, torch.tensor(10.0, device=dev), 12, 12)
        k, _ = segment(tb, self.r)
        i0, wi = self._cidx(k.float())
        m = torch.arange(M, device=dev)
        self.thr_ref = (thr[0, m, i0] * (1 - wi) + thr[0, m, i0 + 1] * wi).contiguous()
        # per-RBG constants
        self.w = torch.tensor([float(x) for x in S_prbs], dtype=torch.float32, device=dev)
        self.lw = torch.log(self.w.float()).contiguous()
        self.lw10 = (10 * torch.log10(self.w / cfg.snr_ref_prbs)).contiguous()
        # link adaptation tables over (PRBs 0..NPRB, MCS) at the UL data-slot symbols
        self.nprb, self.cfg = int(sum(S_prbs)), cfg
        self.la_tbs, self.la_i0, self.la_wi, self.la_ncb = self.la_tables(cfg.ul_data_symbols)
        self.rate = self.r.contiguous()

    def la_tables(self, nsym):
        """TBS (bits), BLER-table code-block index and weight, code blocks over (PRBs 0..NPRB, MCS) of a data slot of
        nsym symbols (PHY.tbs_all + segment, phy.py:77-119): int32, int32, float32, float32 [NPRB+1, M]."""
        cfg = self.cfg
        n = torch.arange(self.nprb + 1, device=self.qm.device, dtype=torch.float32)
        tbs = tbs_38214(self.qm, self.r, n[:, None], nsym, cfg.dmrs_re_per_prb, cfg.overhead_re_per_prb)
        cbs, c = segment(tbs, self.r)
        i0, wi = self._cidx(cbs.float())
        return (tbs.to(torch.int32).contiguous(), i0.to(torch.int32).contiguous(), wi.float().contiguous(),
                c.float().contiguous())

    def _cidx(self, cbs):
        x = ((cbs - self.c0) / self.dc).clamp(0, self.C - 1)
        i0 = x.floor().clamp(max=self.C - 2).long()
        return i0, x - i0


__all__ = ["PhyTables", "tbs_38214", "segment", "MCS_T1", "MCS_T2"]
