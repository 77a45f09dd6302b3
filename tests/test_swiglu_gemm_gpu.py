"""The GEMM's SwiGLU epilogue (mma.matmul_swiglu) on the GPU.

The epilogue reads the same fp32 accumulators the plain GEMM stores, so it must equal, bit for bit, the
plain GEMM's rounded product followed by PyTorch's silu(gate) * up on the de-interleaved halves.  Against an
fp32 PyTorch reference the tolerance is the north star's (max-abs 2e-2, rtol 1e-2) on inputs scaled so the
products are O(1).
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import _native
from mma import interleave_gate_up, matmul, matmul_swiglu, split_gate_up

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0


SHAPES = [
    # M, K, m (gate/up width)
    (2048, 3584, 2368),   # Qwen2.5-7B MLP at TP8
    (777, 256, 192),      # ragged rows; 2m = 384 leaves a half-filled last tile
    (128, 64, 64),        # a single tile, a single K block
    (1, 512, 128),        # one row
]


def _operands(M, K, m, dtype, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn(M, K, generator=g, device=device).to(dtype)
    wg = (torch.randn(K, m, generator=g, device=device) * K ** -0.5).to(dtype)
    wu = (torch.randn(K, m, generator=g, device=device) * K ** -0.5).to(dtype)
    return a, wg, wu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_swiglu_epilogue_equals_gemm_then_torch(shape, dtype, cuda_device):
    M, K, m = shape
    a, wg, wu = _operands(M, K, m, dtype, cuda_device, seed=M + K + m)
    w = interleave_gate_up(wg, wu)
    out = matmul_swiglu(a, w)
    gate, up = split_gate_up(matmul(a, w, stream_k=False))
    assert out.shape == (M, m) and out.dtype == dtype
    assert torch.equal(out, F.silu(gate) * up)


@pytest.mark.parametrize("shape", SHAPES[:2], ids=lambda s: "x".join(map(str, s)))
def test_swiglu_epilogue_against_fp32_reference(shape, cuda_device):
    M, K, m = shape
    a, wg, wu = _operands(M, K, m, torch.bfloat16, cuda_device, seed=3 * M + K)
    ref = F.silu(a.float() @ wg.float()) * (a.float() @ wu.float())
    out = matmul_swiglu(a, interleave_gate_up(wg, wu)).float()
    torch.testing.assert_close(out, ref, rtol=1e-2, atol=2e-2)


def test_swiglu_writes_into_a_strided_output(cuda_device):
    M, K, m = 256, 128, 256
    a, wg, wu = _operands(M, K, m, torch.bfloat16, cuda_device, seed=77)
    big = torch.full((M, m + 64), 7.0, device=cuda_device, dtype=torch.bfloat16)
    out = big[:, :m]
    matmul_swiglu(a, interleave_gate_up(wg, wu), out=out)
    gate, up = split_gate_up(matmul(a, interleave_gate_up(wg, wu), stream_k=False))
    assert torch.equal(out, F.silu(gate) * up)
    assert torch.all(big[:, m:] == 7.0)


def test_swiglu_empty_contraction_is_zero(cuda_device):
    a = torch.empty(64, 0, device=cuda_device, dtype=torch.bfloat16)
    w = torch.empty(0, 256, device=cuda_device, dtype=torch.bfloat16)
    out = torch.full((64, 128), 3.0, device=cuda_device, dtype=torch.bfloat16)
    matmul_swiglu(a, w, out=out)
    assert torch.all(out == 0)
