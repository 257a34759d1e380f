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
