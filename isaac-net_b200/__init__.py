"""isaac_net_b200: a B200-native (sm_100a) implementation of isaac-net's NR uplink control-step engine.

The package directory is named ``isaac-net_b200``; it registers itself as ``isaac_net_b200`` on first import, so both
``importlib.import_module("isaac-net_b200")`` and, after that, ``import isaac_net_b200`` work.

Public API (a drop-in for ``isaac_net.make_engine("L2", ...)`` on the uplink path):
    make_engine(level, E, R, device, config, backend="b200", *, seed=None) -> NRB200Engine
    NRConfig, TrafficModel, Requests
    NetModule, IsaacNetCfg, TrafficRequest  (the Isaac-side module on the engine's radio, net_module.py)
    ShardedEngine, shard_invariant  (one batch split over several GPUs in one process, sharded.py)
"""
import importlib as _importlib
import importlib.abc as _abc
import importlib.util as _util
import sys as _sys

_ALIAS, _REAL = "isaac_net_b200", __name__


class _SubmoduleAlias(_abc.MetaPathFinder, _abc.Loader):
    """Resolves ``isaac_net_b200.<sub>`` to the one ``isaac-net_b200.<sub>`` module object (never a second copy)."""

    def find_spec(self, name, path=None, target=None):
        if name.startswith(_ALIAS + ".") and _REAL != _ALIAS:
            return _util.spec_from_loader(name, self)
        return None

    def create_module(self, spec):
        return _importlib.import_module(_REAL + spec.name[len(_ALIAS):])

    def exec_module(self, module):
        pass


_sys.modules.setdefault(_ALIAS, _sys.modules[__name__])
if not any(isinstance(f, _SubmoduleAlias) for f in _sys.meta_path):
    _sys.meta_path.insert(0, _SubmoduleAlias())

from .config import NRConfig  # noqa: E402
from .traffic import Requests, TrafficModel  # noqa: E402


def make_engine(level, E, R, device="cuda", config=None, backend="b200", *, sizes=None, seed=None, strict=False,
                traffic_rng="generator"):
    """Build the B200 NR engine (level "L2") for E envs x R robots (isaac_net/core/engine.py:232-293 signature).
    traffic_rng="counter" opts into the shard-invariant counter-keyed traffic stream (see NRB200Engine)."""
    from .engine import make_engine as _make
    return _make(level, E, R, device, config, backend, sizes=sizes, seed=seed, strict=strict,
                 traffic_rng=traffic_rng)


def __getattr__(name):
    """The Isaac-side module (net_module.py) on first use: NetModule, IsaacNetCfg, TrafficRequest."""
    if name in ("NetModule", "IsaacNetCfg", "TrafficRequest"):
        return getattr(_importlib.import_module(__name__ + ".net_module"), name)
    if name in ("ShardedEngine", "shard_invariant"):
        return getattr(_importlib.import_module(__name__ + ".sharded"), name)
    raise AttributeError(name)


__all__ = ["make_engine", "NRConfig", "TrafficModel", "Requests", "NetModule", "IsaacNetCfg", "TrafficRequest",
           "ShardedEngine", "shard_invariant"]
