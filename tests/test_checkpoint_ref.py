"""Reference-format checkpoints on the host: every state tensor the reference's golden state snapshot holds (the
names the engine's reference_state uses) is found in the reference's own engine.state_dict() (fixtures cfgk*.npz,
written by tests/golden/make_golden.py from isaac_net/core/checkpoint.py's collect) under the key the mapping of
isaac-net_b200/checkpoint.py gives it, with the same values."""
import importlib

import numpy as np
import pytest

from golden_io import GOLDEN

ck = importlib.import_module("isaac-net_b200.checkpoint")
CKPT = ("k2", "k3", "k5")
NOT_STATE = ("ctr.", "radio.sf_nlos.", "radio.los_field.")   # counters are mapped separately; fields of the LOS
# draws the forced-LOS channel never reads


@pytest.mark.parametrize("case", CKPT)
def test_reference_keys_map_to_the_engine_state_names(case):
    d = np.load(f"{GOLDEN}/cfg{case}.npz")
    ckpt = {k[5:]: d[k] for k in d.files if k.startswith("ckpt/")}
    by_short = {}
    for k, v in ckpt.items():
        n = ck.short_name(k)
        if n is not None:
            by_short[n] = v
    want = [k[5:] for k in d.files if k.startswith("ckst/") and not k[5:].startswith(NOT_STATE)]
    assert want
    for n in want:
        assert n in by_short, n
        assert np.array_equal(np.asarray(by_short[n]), d["ckst/" + n], equal_nan=True), n
