"""Shared fixtures.  Tests marked ``gpu`` need a B200 (sm_100a) and call the
product library through its C ABI; everything else runs on the CPU."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def O():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def q8(pkg):
    import importlib

    return importlib.import_module(__graft_entry__.PKG_NAME + ".q8")


@pytest.fixture(scope="session")
def chain_mod(pkg):
    import importlib

    return importlib.import_module(__graft_entry__.PKG_NAME + ".chain")


@pytest.fixture(scope="session")
def frame_mod(pkg):
    import importlib

    return importlib.import_module(__graft_entry__.PKG_NAME + ".frame")


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    return torch.device("cuda:0")
