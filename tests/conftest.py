import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "input-adaptive-matrix-inference-optimization_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")

if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_pkg():
    if "iam_b200" in sys.modules:
        return sys.modules["iam_b200"]
    spec = importlib.util.spec_from_file_location("iam_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["iam_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libiamb200.so")


@pytest.fixture(scope="session")
def iam():
    return load_pkg()


@pytest.fixture(scope="session")
def ora():
    from oracle import ora as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def weights_mod(iam):
    import importlib
    return importlib.import_module("iam_b200.weights")


def golden(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


GOLDEN_CASES = ["bm_256x64.npz", "bm_128x512.npz", "bm_48x96_ties.npz", "bm_16x4096.npz"]


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device: run the gpu marker on a B200 box")
    return torch.device("cuda:0")
