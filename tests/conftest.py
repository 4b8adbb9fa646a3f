import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
importlib.import_module("isaac-net_b200")
# the config-5 radio map is a build product (isaac-net_b200/data/make_radio_map.py); bake it if this tree has none
importlib.import_module("isaac-net_b200.data.make_radio_map").ensure()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs CUDA")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
