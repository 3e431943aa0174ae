"""Shared test set-up.

Markers: ``gpu`` -- needs a B200 (sm_100a) and the built CUDA library; everything else runs on
CPU. The CPU oracle (oracle/) is the checker for every parity test; the products under test go
through the C ABI of librt_b200.so.
"""
from __future__ import annotations

import importlib.util
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "intel-phi-apl_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")

sys.path.insert(0, ORACLE)
sys.path.insert(0, PKG)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def _ensure_oracle_built() -> None:
    lib = os.path.join(ORACLE, "libq8oracle.so")
    srcs = [os.path.join(ORACLE, f) for f in ("q8_oracle.c", "prims_oracle.c", "q8_oracle.h")]
    if not os.path.exists(lib) or any(os.path.exists(f) and os.path.getmtime(f) > os.path.getmtime(lib) for f in srcs):
        subprocess.run(["make", "-C", ORACLE, "port"], check=True, capture_output=True)


_ensure_oracle_built()


def load_module(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    return O


@pytest.fixture(scope="session")
def rtb():
    import rtb200
    return rtb200


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="session")
def runtime(cuda, rtb):
    rt = rtb.Runtime()
    yield rt
    rt.close()
