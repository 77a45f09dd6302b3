"""Test configuration: import paths for the drop-in modules and the `gpu` marker.

The drop-in modules (flash_atten, tuner, mma, exceptions, ttft) live flat in
flash-attn-economical-gpu_b200/, the way the reference's modules live flat in
its checkout, so that directory goes on sys.path.  Tests marked `gpu` need a
CUDA device; the CPU suite runs with `-m "not gpu"`.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "flash-attn-economical-gpu_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs an sm_100 device, found sm_{major}{minor}")
    return torch.device("cuda:0")


@pytest.fixture
def fake_limits(monkeypatch):
    """B200 per-block limits for host-logic tests that run without a GPU."""
    limits = {
        "available_shared_memory_bytes_per_sm": 232448,
        "available_registers_per_sm": 65536,
        "available_register_file_size_bytes_per_sm": 65536 * 4,
        "warp_size": 32,
        "max_threads_per_block": 1024,
        "max_warps_per_block": 32,
        "multiprocessor_count": 148,
    }
    import tuner

    monkeypatch.setattr(tuner, "get_sm_resource_limits", lambda: dict(limits))
    return limits
