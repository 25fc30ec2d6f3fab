"""Shared pytest setup: the `gpu` marker, repo paths and the package loader.

The product package lives in the directory ``memory-aware-inference_b200`` (a
name that is not a Python identifier); it is loaded by path and registered as
``mai_b200``.
"""
import importlib.util
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
PKG_DIR = os.path.join(REPO, "memory-aware-inference_b200")


def load_package():
    if "mai_b200" in sys.modules:
        return sys.modules["mai_b200"]
    spec = importlib.util.spec_from_file_location(
        "mai_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mai_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def mai():
    return load_package()


@pytest.fixture(scope="session")
def ctx(mai):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = mai.CudaContext(0)
    yield c
    c.close()
