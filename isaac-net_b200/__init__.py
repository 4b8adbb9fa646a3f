"""isaac_net_b200: a B200-native (sm_100a) implementation of isaac-net's NR uplink control-step engine.

The package directory is named ``isaac-net_b200``; it registers itself as ``isaac_net_b200`` on first import, so both
``importlib.import_module("isaac-net_b200")`` and, after that, ``import isaac_net_b200`` work.

Public API (a drop-in for ``isaac_net.make_engine("L2", ...)`` on the uplink path):
    make_engine(level, E, R, device, config, backend="b200", *, seed=None) -> NRB200Engine
    NRConfig, TrafficModel, Requests
"""
import sys as _sys

_sys.modules.setdefault("isaac_net_b200", _sys.modules[__name__])

from .config import NRConfig  # noqa: E402
from .traffic import Requests, TrafficModel  # noqa: E402


def make_engine(level, E, R, device="cuda", config=None, backend="b200", *, sizes=None, seed=None, strict=False):
    """Build the B200 NR engine (level "L2") for E envs x R robots (isaac_net/core/engine.py:232-293 signature)."""
    from .engine import make_engine as _make
    return _make(level, E, R, device, config, backend, sizes=sizes, seed=seed, strict=strict)


__all__ = ["make_engine", "NRConfig", "TrafficModel", "Requests"]
