"""The Isaac-side network module on the B200 engine: NetModule, IsaacNetCfg, TrafficRequest (isaac_net/isaac/
net_module.py, isaac/config.py, isaac/obs.py of isaac-net v0.2.0), for the engine's own radio.

    net = NetModule("L2", E, R, "cuda", NRConfig(...), backend="b200",
                    isaac=IsaacNetCfg(radio="engine", obs_features=("aoi", "sinr", "delay_history")))
    net.reset(env_ids)
    net.submit(None, TrafficRequest(send[E,R], tag[E,R]))
    out = net.step(None, poses_end[E,R,3], cur_tag[E])
    x = net.obs()                                          # [E, R, net.obs_dim]

Each step is the engine's captured control step followed by ONE launch of inb_net_obs (csrc/net_obs.cu), which
derives NetModule.step's outputs from the engine's step dict (freshness last_cap, age of information, delays in
seconds, RSRP, blocked / los, tag_delivered; net_module.py:340-374) and packs the selected observation features,
normalised, with the delay history (NetObs.update, obs.py:48-87).  Every output is a fresh tensor of one output
block per step, as the reference returns new tensors.  The Isaac radio (IsaacNetCfg.radio = "isaac": per-env radio
parameters, pose chunks, Isaac blockage) and domain randomization of its radio keys are not part of this path and
are refused; with the engine's radio the reference honors no dr_ranges key at level L2 either (it warns, or raises
with dr_strict), and so does this module.
"""
from __future__ import annotations

import ctypes
import math
import warnings
from dataclasses import dataclass, field, replace
from typing import Optional, Sequence

import numpy as np
import torch

from . import _native as nat
from .config import NRConfig
from .engine import B200Unsupported

OBS_FEATURES = ("delivered_mask", "msg_delay", "aoi", "queue_len", "queue_bytes", "sinr", "rsrp", "serving_cell",
                "last_delivered", "delay_history", "blocked", "los")       # isaac/config.py:56-57
DEFAULT_OBS = ("aoi", "sinr", "queue_len", "last_delivered")
_OBS_ALIASES = {"delivered": "last_delivered", "snr": "sinr", "delay": "msg_delay", "queue": "queue_len"}
DB_SCALE = 40.0
TIME_SCALE_STEPS = 50
DR_KEYS = ("p_tx_dbm", "noise_dbm", "pl_const_db", "pl_exp", "shadow_sigma_db", "blockage_db", "gnb_offset_m",
           "delay_median_steps", "delay_log_sigma", "loss")


def canonical_features(features: Sequence[str]) -> tuple:
    """Feature names with the reference's aliases resolved, unknown or repeated names refused (isaac/config.py:
    90-99)."""
    out = []
    for f in features:
        f = _OBS_ALIASES.get(f, f)
        if f not in OBS_FEATURES:
            raise ValueError(f"unknown observation feature {f!r}; one of {OBS_FEATURES}")
        if f in out:
            raise ValueError(f"observation feature {f!r} listed twice")
        out.append(f)
    return tuple(out)


def feature_dims(features: Sequence[str], frame_buffer: int = 16, n_cells: int = 1, history: int = 4) -> dict:
    """{feature: width} in the order of `features` (isaac/config.py:102-106)."""
    width = {"delivered_mask": frame_buffer, "msg_delay": frame_buffer, "serving_cell": n_cells,
             "delay_history": history}
    return {f: width.get(f, 1) for f in canonical_features(features)}


@dataclass
class IsaacNetCfg:
    """Isaac-specific settings (isaac/config.py:109-160), the reference's fields and defaults.  This module runs
    radio="engine"; the Isaac radio's own fields are accepted and unused, as the reference leaves them unused on the
    engine's radio."""
    radio: str = "isaac"
    pose_asset: Optional[str] = None
    pose_body_ids: Optional[Sequence[int]] = None
    pose_offset_m: Sequence[float] = (0.0, 0.0, 0.0)
    gnb_pos: Optional[Sequence[Sequence[float]]] = None
    gnb_height_m: float = 0.0
    pose_chunks: int = 4
    scene_map: Optional[object] = None
    net_decimation: int = 1
    net_substeps: int = 1
    blockage: bool = True
    robot_blockers: bool = False
    blocker_radius_m: float = 0.3
    blockage_db: float = 20.0
    dr_ranges: dict = field(default_factory=dict)
    dr_mode: str = "reset"
    dr_interval_steps: tuple = (50, 100)
    dr_strict: bool = False
    obs_features: Sequence[str] = DEFAULT_OBS
    obs_history: int = 4
    obs_time_scale_s: Optional[float] = None
    nr: dict = field(default_factory=dict)
    log_kpis: bool = True
    log_every: int = 1

    def __post_init__(self):
        if self.radio not in ("isaac", "engine"):
            raise ValueError(f"radio must be 'isaac' or 'engine', got {self.radio!r}")
        if self.dr_mode not in ("reset", "interval", "off"):
            raise ValueError(self.dr_mode)
        if self.net_decimation < 1 or self.net_substeps < 1 or (self.net_decimation > 1 and self.net_substeps > 1):
            raise ValueError("net_decimation and net_substeps are >= 1, and only one of them > 1")
        if self.pose_chunks < 1 or self.obs_history < 1:
            raise ValueError("pose_chunks and obs_history are >= 1")
        for k, v in self.dr_ranges.items():
            if k not in DR_KEYS:
                raise KeyError(f"{k!r} is not a randomization key; one of {DR_KEYS}")
            if v[0] > v[1]:
                raise ValueError(f"dr_ranges[{k!r}] = {v}: lo > hi")
        self.obs_features = canonical_features(self.obs_features)

    def with_(self, **kw) -> "IsaacNetCfg":
        return replace(self, **kw)

    def time_scale_s(self, config: NRConfig) -> float:
        if self.obs_time_scale_s is not None:
            return float(self.obs_time_scale_s)
        return TIME_SCALE_STEPS * config.control_step_ms / 1000.0

    def n_gnb(self, config: NRConfig) -> int:
        return len(self.gnb_pos) if self.gnb_pos is not None else config.n_cells

    def obs_dims(self, config: NRConfig) -> dict:
        return feature_dims(self.obs_features, config.frame_buffer, self.n_gnb(config), self.obs_history)

    def obs_dim(self, config: NRConfig) -> int:
        return sum(self.obs_dims(config).values())


@dataclass
class TrafficRequest:
    """Messages each robot enqueues this control step: send [E,R] long (0 = nothing, c >= 1 = one message of class
    c), tag [E,R] long (-1 = none) or None (net_module.py:79-88)."""
    send: torch.Tensor
    tag: Optional[torch.Tensor] = None


def _f32(x):
    return float(np.float32(x))


def _inv32(x):
    """1 / x as torch's CUDA division by a python scalar computes it: float32(1) / float32(x)."""
    return float(np.float32(1.0) / np.float32(x))


class ObsPacker:
    """The device observation packing of E x R robots: its state (last_cap [E,R], the delay history [E,R,K]) and one
    inb_net_obs launch per step on the current stream.  `features` in order (canonical names), G one-hot width,
    K history length, step_dt (s), noise_db (the config's subband noise, dBm), time_scale (s), q_bytes
    (frame_buffer x the largest message size)."""

    def __init__(self, features, E, R, F, G, K, step_dt, noise_db, time_scale, q_bytes, device):
        self.E, self.R, self.F, self.G, self.K = int(E), int(R), int(F), int(G), int(K)
        self.dev = torch.device(device)
        self.dims = feature_dims(features, self.F, self.G, self.K)
        self.dim = sum(self.dims.values())
        self.last_cap = torch.zeros(self.E, self.R, dtype=torch.long, device=self.dev)
        self.hist = torch.zeros(self.E, self.R, self.K, device=self.dev)
        self.L = nat.lib()
        a = self.args = nat.InbObsArgs()
        a.E, a.R, a.F, a.G, a.K, a.dim = self.E, self.R, self.F, self.G, self.K, self.dim
        offs, col = {n: -1 for n in nat.OBS_OFFS}, 0
        for f, w in self.dims.items():
            offs[nat.OBS_OFFS[OBS_FEATURES.index(f)]] = col
            col += w
        for n, v in offs.items():
            setattr(a, n, v)
        a.step_dt, a.noise_db = _f32(step_dt), _f32(noise_db)
        a.inv_ts, a.inv_F, a.inv_qbytes, a.inv_db = _inv32(time_scale), _inv32(self.F), _inv32(q_bytes), \
            _inv32(DB_SCALE)
        a.last_cap, a.hist = self.last_cap.data_ptr(), self.hist.data_ptr()
        self._lay = None

    def reset(self, ids):
        """Zero the freshness state and the delay history of env ids (None = all)."""
        for buf in (self.last_cap, self.hist):
            if ids is None:
                buf.zero_()
            else:
                buf.index_fill_(0, ids, 0)

    def _block(self):
        """One output block per step: a fresh tensor per output, 256-byte aligned slices of one allocation."""
        if self._lay is None:
            E, R = self.E, self.R
            spec = [("last_cap_out", torch.long, (E, R)), ("aoi_s", torch.float32, (E, R)),
                    ("delay_s", torch.float32, (E, R, self.F)), ("rsrp_dbm", torch.float32, (E, R)),
                    ("x", torch.float32, (E, R, self.dim)), ("delivered_any", torch.bool, (E, R)),
                    ("blocked_out", torch.bool, (E, R)), ("los_out", torch.bool, (E, R)),
                    ("tag_delivered", torch.bool, (E,))]
            lay, off = [], 0
            for n, dt, shape in spec:
                nb = math.prod(shape) * torch.empty((), dtype=dt).element_size()
                lay.append((n, dt, shape, off, nb))
                off += (nb + 255) // 256 * 256
            self._lay = (lay, max(off, 256))
        lay, total = self._lay
        blk = torch.empty(total, dtype=torch.uint8, device=self.dev)
        return {n: blk[off:off + nb].view(dt).view(shape) for n, dt, shape, off, nb in lay}

    def step(self, o: dict, cur_tag: Optional[torch.Tensor] = None) -> dict:
        """Launch the packing of one engine step dict `o` (device tensors); returns the new output tensors
        (last_cap_out, aoi_s, delay_s, rsrp_dbm, x, delivered_any, blocked_out, los_out[, tag_delivered])."""
        b = self._block()
        a = self.args
        a.newest, a.t, a.queue_len, a.serving = (o["newest"].data_ptr(), o["t"].data_ptr(),
                                                 o["queue_len"].data_ptr(), o["serving_cell"].data_ptr())
        a.queue_bytes, a.sinr_db, a.delay = (o["queue_bytes"].data_ptr(), o["sinr_db"].data_ptr(),
                                             o["delay"].data_ptr())
        a.delivered, a.cap, a.det_env = o["delivered"].data_ptr(), o["cap"].data_ptr(), o["det_env"].data_ptr()
        a.blocked = o["blocked"].data_ptr() if "blocked" in o else None
        a.los = o["los"].data_ptr() if "los" in o else None
        ct = None
        if cur_tag is not None:
            ct = cur_tag.to(self.dev, torch.long).contiguous()
        a.cur_tag = ct.data_ptr() if ct is not None else None
        a.tag_delivered = b["tag_delivered"].data_ptr() if ct is not None else None
        for n in ("last_cap_out", "aoi_s", "delay_s", "rsrp_dbm", "x", "delivered_any", "blocked_out", "los_out"):
            setattr(a, n, b[n].data_ptr())
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        nat.check(self.L.inb_net_obs(ctypes.byref(a), stream), "inb_net_obs")
        self._keep = (o, ct)          # the launch is asynchronous: keep its inputs alive
        if ct is None:
            b.pop("tag_delivered")
        return b


class NetModule:
    """Network in the loop of E envs x R robots on the B200 engine (isaac/net_module.py:89-176, 221-376)."""

    def __init__(self, level="L2", num_envs: int = None, num_robots: int = None, device="cuda",
                 config: Optional[NRConfig] = None, backend: str = "b200", *, isaac: Optional[IsaacNetCfg] = None,
                 seed: Optional[int] = None, strict: bool = False, **isaac_overrides):
        from . import make_engine
        if level != "L2":
            raise B200Unsupported(f"level {level!r}: the B200 backend runs the NR engine (level 'L2')")
        isc = isaac if isaac is not None else IsaacNetCfg()
        if isaac_overrides:
            isc = replace(isc, **isaac_overrides)
        if isc.radio != "engine":
            raise B200Unsupported("IsaacNetCfg(radio='isaac'): the Isaac radio (per-env radio parameters, pose chunks) "
                                  "is not part of the B200 path; pass radio='engine'")
        if isc.nr:
            raise B200Unsupported("IsaacNetCfg.nr overrides: pass the resolved NRConfig as config")
        if isc.gnb_pos is not None:
            raise B200Unsupported("IsaacNetCfg.gnb_pos: with radio='engine' the cells are NRConfig's")
        cfg = config if config is not None else NRConfig()
        if cfg.frame_buffer > 64:
            raise B200Unsupported(f"frame_buffer={cfg.frame_buffer}: the observation packing handles at most 64 frame "
                                  "slots per robot")
        if isc.dr_ranges and isc.dr_mode != "off":      # none is honored at level L2 on the engine's radio
            msg = (f"level L2 does not honor these dr_ranges keys with radio='engine': {sorted(isc.dr_ranges)}")
            if isc.dr_strict:
                raise ValueError(msg)
            warnings.warn(msg, stacklevel=2)
        self.level, self.backend, self.isaac, self.config = level, backend, isc, cfg
        self.E, self.R = int(num_envs), int(num_robots)
        self.eng = make_engine("L2", self.E, self.R, device, cfg, backend, seed=seed, strict=strict)
        self.dev = self.eng.dev
        self.F, self.G = cfg.frame_buffer, isc.n_gnb(cfg)
        self.K = int(isc.obs_history)
        self.step_dt = cfg.control_step_ms / 1000.0
        self.dims = isc.obs_dims(cfg)
        self.obs_dim = sum(self.dims.values())
        self.features = tuple(self.dims)
        self.packer = ObsPacker(self.features, self.E, self.R, self.F, self.G, self.K, self.step_dt,
                                cfg.subband_noise_dbm, isc.time_scale_s(cfg), self.F * max(cfg.msg_sizes), self.dev)
        self.x = torch.zeros(self.E, self.R, self.obs_dim, device=self.dev)
        self._zero_hid = torch.zeros(self.E, dtype=torch.long, device=self.dev)
        self._submitted = False

    @property
    def last_cap(self) -> torch.Tensor:
        """[E,R] newest capture step delivered this episode (0 = the state at reset)."""
        return self.packer.last_cap

    # ------------------------------------------------------------------ properties
    @property
    def clock(self) -> torch.Tensor:
        """[E] per-env episode clock (control steps since that env's reset)."""
        return self.eng.clock

    # ------------------------------------------------------------------ contract API
    def reset(self, env_ids=None):
        """Partial reset of env_ids (index tensor, bool mask, list or None = all): the engine, the freshness state
        and the observation features (net_module.py:221-235, obs.py:43-46).  Other envs are bitwise unaffected."""
        if env_ids is None:
            ids = None
        else:
            t = torch.as_tensor(env_ids, device=self.dev)
            ids = t.nonzero().flatten() if t.dtype == torch.bool else t.long().flatten()
            if ids.numel() == 0:
                return
        self.eng.reset(ids)
        self.packer.reset(ids)
        if ids is None:
            self.x.zero_()
        else:
            self.x.index_fill_(0, ids, 0)

    def submit(self, t, req: TrafficRequest):
        """Messages captured at the start of this control step (t is ignored: per-env clocks); call before step
        (net_module.py:237-247)."""
        from .traffic import Requests
        tag = req.tag
        if tag is None:
            det, hid = None, None
        else:
            det = tag >= 0
            hid = tag.max(-1).values.clamp(min=0)
        self._submitted = True
        return self.eng.submit(None, Requests(req.send, det, hid))

    def step(self, t, poses: torch.Tensor, cur_tag: Optional[torch.Tensor] = None, blocked_fn=None,
             blockers: Optional[torch.Tensor] = None) -> dict:
        """Advance every env by one control step (net_module.py:287-375); poses [E,R,3] or [E,R,2] at the END of
        the step, cur_tag [E] long (-1 = none) for tag_delivered.  Returns the reference's dict: delivered,
        newest_cap, last_cap, aoi_s, queue_len, queue_bytes, sinr_db, rsrp_dbm, serving, blocked, los,
        msg_delivered, timed_out, cap, cls, delay_s, t (+ tag_delivered)."""
        if blocked_fn is not None or blockers is not None:
            raise B200Unsupported("blocked_fn / blockers: LOS callbacks and TR 38.901 screens are not part of the "
                                  "B200 path")
        if not self._submitted:
            self.submit(None, TrafficRequest(torch.zeros(self.E, self.R, dtype=torch.long, device=self.dev)))
        self._submitted = False
        # det_env of the engine compares queued messages with the hid of the step: the env's current tag
        self.eng._last_hid.copy_(cur_tag.clamp(min=0) if cur_tag is not None else self._zero_hid)
        o = self.eng.step(None, poses)
        b = self.packer.step(o, cur_tag)
        self.x = b["x"]
        out = dict(delivered=b["delivered_any"], newest_cap=o["newest"], last_cap=b["last_cap_out"], aoi_s=b["aoi_s"],
                   queue_len=o["queue_len"], queue_bytes=o["queue_bytes"], sinr_db=o["sinr_db"],
                   rsrp_dbm=b["rsrp_dbm"], serving=o["serving_cell"], blocked=b["blocked_out"], los=b["los_out"],
                   msg_delivered=o["delivered"], timed_out=o["timed_out"], cap=o["cap"], cls=o["cls"],
                   delay_s=b["delay_s"], t=o["t"])
        if cur_tag is not None:
            out["tag_delivered"] = b["tag_delivered"]
        return out

    def obs(self) -> torch.Tensor:
        """[E,R,obs_dim] the selected observation features of the last step (zeros after a reset)."""
        return self.x

    def queued(self) -> torch.Tensor:
        return self.eng.queued()

    # ------------------------------------------------------------------ checkpoints
    def state_dict(self) -> dict:
        """The engine's state and the module's own (freshness, delay history, last observation)."""
        sd = {"eng." + k: v for k, v in self.eng.state_dict().items()}
        sd.update({"net.last_cap": self.packer.last_cap.clone(), "net.hist": self.packer.hist.clone(),
                   "net.x": self.x.clone()})
        return sd

    def load_state_dict(self, sd: dict, strict: bool = True):
        self.eng.load_state_dict({k[4:]: v for k, v in sd.items() if k.startswith("eng.")}, strict=strict)
        self.packer.last_cap.copy_(sd["net.last_cap"])
        self.packer.hist.copy_(sd["net.hist"])
        self.x = sd["net.x"].to(self.dev).clone()
