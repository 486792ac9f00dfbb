import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "slo-aware-llm-serving-engine_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np
    here = os.path.join(ROOT, "tests", "golden")
    with open(os.path.join(here, "golden.json")) as f:
        manifest = json.load(f)
    return manifest, dict(np.load(os.path.join(here, "golden.npz")))
