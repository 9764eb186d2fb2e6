"""Shared test setup.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``) and
  the ``refgpu`` marker (the reference's own CUDA backend measured on a GPU;
  run with ``-m refgpu``);
* imports the package directory ``distributed-recommendation-model-training-system_b200``
  (its name is not a Python identifier) under the module name ``eps_b200``;
* makes the CPU checkers (oracle/) importable as ``oracle_lib``.
"""
from __future__ import annotations

import importlib.util
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "distributed-recommendation-model-training-system_b200")
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU")
    config.addinivalue_line("markers", "refgpu: measures the reference's own CUDA backend on a "
                            "GPU (run explicitly with -m refgpu; skipped without a GPU)")


def import_package():
    if "eps_b200" in sys.modules:
        return sys.modules["eps_b200"]
    spec = importlib.util.spec_from_file_location(
        "eps_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["eps_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def import_workloads():
    if "eps_b200_workloads" in sys.modules:
        return sys.modules["eps_b200_workloads"]
    spec = importlib.util.spec_from_file_location("eps_b200_workloads",
                                                  os.path.join(PKG_DIR, "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["eps_b200_workloads"] = mod
    spec.loader.exec_module(mod)
    return mod


def _ensure_oracle():
    so = os.path.join(ROOT, "oracle", "_build", "libeps_oracle.so")
    src = os.path.join(ROOT, "oracle", "eps_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"])


_ensure_oracle()


@pytest.fixture(scope="session")
def eps():
    return import_package()


@pytest.fixture(scope="session")
def workloads():
    return import_workloads()


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
