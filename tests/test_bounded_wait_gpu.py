"""A bounded wait that runs out ends the kernel with an error status, not a hang.

Every wait in the attention kernels gives up after a time limit, records a
code in the device error word and unwinds (waits for its own copies and
products, frees TMEM, returns).  Here the limit is cut to 2 ms and the
producer is told to skip one K/V load, so one barrier is starved for real;
nothing faults, traps or spins without end.  The test checks that the kernel
returns, that the host reads a K/V-pipeline wait code and the Python layer raises,
and that the next normal call on the same device is correct.  This mirrors
the reference turning a failed launch into a status instead of a crash
(test_flash_atten.py:574-583).
"""
from __future__ import annotations

import pytest
import torch

import _native
import flash_atten

pytestmark = pytest.mark.gpu

# The starved tile stops the K/V pipeline from both ends: the MMA thread's wait for the tile (kDevTimeoutKV,
# 2) and the producer's wait for the ring slot that tile would have freed (kDevTimeoutEmpty, 6) start within
# microseconds of each other, and the first to run out records its code (csrc/ptx.cuh).
KV_PIPELINE_CODES = (2, 6)


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(77)
    q = torch.randn(1, 2, 256, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(1, 2, 1024, 128, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(1, 2, 1024, 128, generator=g, device=dev, dtype=torch.bfloat16)
    return q, k, v


def _run(q, k, v, variant):
    o = torch.empty_like(q)
    flash_atten._launch_attention(q, k, v, o, None, causal=False, sm_scale=128 ** -0.5, what="test", variant=variant)
    return o


@pytest.mark.parametrize("variant", [0, 1], ids=["two_tiles_one_s_buffer", "one_tile_two_s_buffers"])
def test_starved_load_gives_up_and_device_recovers(variant, cuda_device):
    q, k, v = _inputs(cuda_device)
    plan = flash_atten.attention_plan(q, k, v, variant=variant)
    assert plan["s_buffers"] == (1 if variant == 0 else 2)  # 2 CTAs < 1.5 per SM: the two-buffer tile
    want = _run(q, k, v, variant)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    try:
        _native.set_wait_limit_ns(2_000_000)
        _native.starve_kv_load(2)  # ring tile 2: K_1 with one S buffer, V_0 with two
        _run(q, k, v, variant)
        torch.cuda.synchronize()  # the kernel returned: no hang
        assert _native.device_error() in KV_PIPELINE_CODES
        # the same failure seen through the Python layer
        _run(q, k, v, variant)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="bounded wait"):
            _native.raise_on_device_error()
    finally:
        _native.starve_kv_load(-1)
        _native.set_wait_limit_ns(0)
    # the context is still usable and the next call is right
    got = _run(q, k, v, variant)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert torch.equal(got, want)
