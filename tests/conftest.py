"""Shared test setup: the `gpu` marker, the CUDA package and the CPU oracle.

The package directory is ``llama.rs_b200`` (not an importable identifier), so
it is loaded by path under the module name ``llamars_b200``.
"""
import importlib.util
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "llama.rs_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


def _gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def load_package():
    if "llamars_b200" in sys.modules:
        return sys.modules["llamars_b200"]
    lib = os.path.join(PKG_DIR, "libllamars.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-s", "-C", PKG_DIR, "-j8"], check=True)
    spec = importlib.util.spec_from_file_location(
        "llamars_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llamars_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def lrs():
    return load_package()


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def backend(lrs):
    if not _gpu_available():
        pytest.fail("GPU test run without a CUDA device")
    be = lrs.CudaBackend(0)
    yield be
    be.close()


# Greedy tokens may swap only where two logits are closer than any bar can
# separate: at a step whose oracle top-1/top-2 margin is below NEAR_TIE
# (twenty times below the 2e-2 logit bar).  After such a swap the sequences
# differ by construction, so the comparison stops there.
NEAR_TIE = 1e-3


def assert_greedy(ref, toks, near_tie=NEAR_TIE):
    """ref: oracle benchmark_tokens() result (tokens, margins); toks: the
    tokens the GPU fed at each step.  Equal up to the first near-tie."""
    import numpy as np
    want = np.asarray(ref["tokens"])
    toks = np.asarray(toks)
    diff = np.nonzero(want != toks)[0]
    if not diff.size:
        return None
    i = int(diff[0])
    margin = float(ref["margins"][i])
    assert margin < near_tie, (f"greedy tokens diverge at step {i}: oracle {want[i]} gpu {toks[i]}; "
                               f"oracle top1-top2 margin there {margin:.3e}")
    return i
