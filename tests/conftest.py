"""Shared pytest setup: the `gpu` marker, import paths and common fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hypermoe-engine_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


_HOST_LAYERS = {}


def host_layer(cfg_name, seed):
    """Seeded synthetic layer of a named configuration, synthesized once per
    test session (the C5 arena is 2.4 GB and takes seconds to generate)."""
    import hmoe_api
    key = (cfg_name, seed)
    if key not in _HOST_LAYERS:
        if len(_HOST_LAYERS) >= 2:
            _HOST_LAYERS.clear()
        _HOST_LAYERS[key] = hmoe_api.make_host_layer(hmoe_api.CONFIGS[cfg_name], seed=seed)
    return _HOST_LAYERS[key]


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    import hmoe_api
    hmoe_api.lib()  # raises if libhmoe.so is missing: no silent fallback
    return torch.device("cuda:0")
