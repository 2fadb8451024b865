"""Shared test setup: the `gpu` marker, import of the hyphen-named product
package, and seeded input generators (numpy default_rng, draw order x, W,
scales, as the benchmark inputs)."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "qwen3-vl-2b-inference_b200")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def import_qvl():
    """Import qwen3-vl-2b-inference_b200 as module `qvl_b200`."""
    if "qvl_b200" in sys.modules:
        return sys.modules["qvl_b200"]
    spec = importlib.util.spec_from_file_location(
        "qvl_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["qvl_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def make_linear_inputs(seed, M, N, K, g):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N * (K // g)).astype(np.float32)
    return x, w, ws


@pytest.fixture(scope="session")
def qvl():
    return import_qvl()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
