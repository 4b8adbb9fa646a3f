"""Host-side inputs of the radio launch: radio-map files and the blockage CDF table.

``load_radio_map`` reads the reference's radio-map format (isaac_net/core/channels/radio_map.py:1-16, 68-79):
``gain_db`` [C, H, W] (or [H, W] for one cell), ``bounds`` (x0, y0, x1, y1) and scalar metadata.  The grid goes to
the device as float32 [C, H*W]; the kernel samples it (RadioMap._bilinear, radio_map.py:101-115).

``cdf_table`` is the sorted sample of the unit sum-of-cosines marginal that maps a blockage field value to a uniform
(channels/fields.py:93-106).  The table is part of the model's definition: it must be the very samples the reference
draws (a CPU torch.Generator seeded 0, float64 uniforms, sorted, rounded to float32), so it is drawn the same way.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def load_radio_map(path):
    """(gain [C, H*W] float32 CPU tensor, H, W, bounds tuple, metadata dict) of a .npz / .pt radio-map file."""
    if not path:
        raise ValueError("channel='radio_map' needs NRConfig.radio_map_path")
    if path == "synthetic":
        raise ValueError("radio_map_path='synthetic' (the reference's shipped test map) is not bundled; bake a map "
                         "file (isaac-net_b200/data/make_radio_map.py shows the format)")
    if str(path).endswith(".pt"):
        d = torch.load(path, map_location="cpu")
        d = {k: (v.numpy() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
    else:
        with np.load(path, allow_pickle=False) as z:
            d = {k: z[k] for k in z.files}
    g = torch.as_tensor(np.asarray(d["gain_db"], dtype=np.float32))
    if g.dim() == 2:
        g = g[None]
    if g.dim() != 3 or g.shape[1] < 2 or g.shape[2] < 2:
        raise ValueError("gain_db must be [C, H, W] with H, W >= 2")
    C, H, W = g.shape
    x0, y0, x1, y1 = (float(b) for b in np.asarray(d["bounds"]).reshape(4))
    if not (x1 > x0 and y1 > y0):
        raise ValueError("bounds = (x0, y0, x1, y1) with x1 > x0, y1 > y0")
    meta = {k: (v.item() if hasattr(v, "item") and np.ndim(v) == 0 else v) for k, v in d.items()
            if k not in ("gain_db", "bounds", "los_prob", "obstacle_z")}
    return g.reshape(C, H * W).contiguous(), H, W, (x0, y0, x1, y1), meta


def cdf_table(K, n=1 << 16, seed=0):
    """Sorted float32 samples [n] of sqrt(2/K) sum_k cos(U_k), U_k ~ U(0, 2 pi) (CPU)."""
    g = torch.Generator().manual_seed(seed)
    z = math.sqrt(2 / K) * torch.cos(torch.rand(n, K, generator=g, dtype=torch.float64) * 2 * math.pi).sum(-1)
    return z.sort().values.float()
