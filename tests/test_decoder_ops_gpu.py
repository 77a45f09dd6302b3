"""The decoder's fused memory-bound ops (fab_rmsnorm, fab_bias_rope, fab_silu_mul) against the PyTorch
expressions of the TTFT model they replace, on the same bf16 inputs.

bias + RoPE and SwiGLU round exactly where the PyTorch expressions do and must match them bit for bit.
RMSNorm sums squares in a different order than torch's reduction, so its scale may differ in the last fp32
bits and an element may land one bf16 step away (rtol 1e-2, and at most 1 % of elements differing).
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import _native
import ttft
from mma import split_gate_up

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0


@pytest.mark.parametrize("rows, cols, with_residual", [(2048, 3584, True), (333, 3584, False), (5, 896, True)])
def test_rmsnorm_matches_torch(rows, cols, with_residual, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g, device=cuda_device).to(torch.bfloat16)
    res = torch.randn(rows, cols, generator=g, device=cuda_device).to(torch.bfloat16) if with_residual else None
    w = (1 + 0.1 * torch.randn(cols, generator=g, device=cuda_device)).to(torch.bfloat16)
    xr = x + res if with_residual else x
    ref = ttft._rms_norm(xr, w, 1e-6)
    xn = x.clone()
    h = ttft._native_rmsnorm(xn, w, 1e-6, residual=res)
    if with_residual:
        assert torch.equal(xn, xr)  # the residual add is exact
    torch.testing.assert_close(h.float(), ref.float(), rtol=1e-2, atol=1e-2)
    assert (h != ref).float().mean().item() < 0.01


@pytest.mark.parametrize("with_bias", [True, False])
def test_bias_rope_matches_torch_bit_for_bit(with_bias, cuda_device):
    arch = ttft.KNOWN_ARCHS["Qwen/Qwen2.5-7B"]
    S, nq, nkv, D = 300, 28, 4, arch.head_dim
    g = torch.Generator(device=cuda_device).manual_seed(7)
    qkv = torch.randn(S, (nq + 2 * nkv) * D, generator=g, device=cuda_device).to(torch.bfloat16)
    bias = torch.randn((nq + 2 * nkv) * D, generator=g, device=cuda_device).to(torch.bfloat16) if with_bias else None
    cos, sin = ttft.rope_tables(arch, S, cuda_device)
    ref = qkv.clone()
    if bias is not None:
        ref += bias
    q = ref[:, : nq * D].view(S, nq, D)
    k = ref[:, nq * D:(nq + nkv) * D].view(S, nkv, D)
    q_ref = q * cos[:, None, :] + ttft._rotate_half(q) * sin[:, None, :]
    k_ref = k * cos[:, None, :] + ttft._rotate_half(k) * sin[:, None, :]
    out = qkv.clone()
    ttft._native_bias_rope(out, bias, cos, sin, nq + 2 * nkv, nq + nkv, D)
    assert torch.equal(out[:, : nq * D].view(S, nq, D), q_ref)
    assert torch.equal(out[:, nq * D:(nq + nkv) * D].view(S, nkv, D), k_ref)
    assert torch.equal(out[:, (nq + nkv) * D:], ref[:, (nq + nkv) * D:])


def test_silu_mul_matches_torch_bit_for_bit(cuda_device):
    """The interleaved gate/up layout the decoder's weights use."""
    g = torch.Generator(device=cuda_device).manual_seed(8)
    gu = (3 * torch.randn(777, 2 * 2368, generator=g, device=cuda_device)).to(torch.bfloat16)
    gate, up = split_gate_up(gu)
    ref = F.silu(gate) * up
    out = ttft._native_silu_mul(gu)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_silu_mul_concatenated_halves(dtype, cuda_device):
    """interleave 0: gate in the first m columns, up in the last m (through the C ABI)."""
    import ctypes

    g = torch.Generator(device=cuda_device).manual_seed(9)
    gu = (3 * torch.randn(300, 2 * 520, generator=g, device=cuda_device)).to(dtype)
    m = gu.shape[1] // 2
    out = torch.empty(300, m, device=cuda_device, dtype=dtype)
    rc = _native.lib.fab_silu_mul(gu.data_ptr(), out.data_ptr(), 300, m, gu.stride(0), out.stride(0), 0,
                                  _native.dtype_code(dtype),
                                  ctypes.c_void_p(_native.current_stream_handle(gu.device)))
    _native.check(rc, "fab_silu_mul")
    assert torch.equal(out, F.silu(gu[:, :m]) * gu[:, m:])
