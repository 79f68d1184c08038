"""Shared pytest setup: the `gpu` marker, import paths for the binding and the oracle, and helpers."""
from __future__ import annotations

import os
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
# the emugemm-cdna source tree: present where the oracle is built, absent on a GPU box (tests that read it skip)
REF_ROOT = pathlib.Path(os.environ.get("EMUGEMM_REF_ROOT", "/root/reference"))
for p in (ROOT / "emugemm-cdna_b200", ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libemugemm.so")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"device is sm_{major}{minor}, the library is built for sm_100a")
    return torch


@pytest.fixture(scope="session")
def handle(cuda):
    import emugemm

    h = emugemm.Handle()
    yield h
    h.close()


@pytest.fixture(autouse=True)
def _restore_kernel_choices(request):
    """A test that changes the session handle's kernel choices (emugemm_set_attr) leaves them as it found them."""
    yield
    if "handle" in request.fixturenames:
        request.getfixturevalue("handle").reset_kernels()
