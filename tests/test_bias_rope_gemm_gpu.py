"""QKV projection with the bias add and rotate-half RoPE in the GEMM epilogue (FAB_GEMM_EPILOGUE_BIAS_ROPE).

The fused kernel must equal, bit for bit, the two-pass path it replaces in the TTFT decoder: the GEMM's 16-bit
output followed by fab_bias_rope.  That path in turn equals the PyTorch expressions `qkv + b` and
`q*cos + rotate_half(q)*sin` bit for bit (test_decoder_ops_gpu.py); one case here checks PyTorch directly too.
Shapes cover the CTA-pair kernel (the decoder's 2048 x 3584 -> 4608 projection) and the single-CTA kernel
(ragged rows, a partial last tile of whole heads), head_dim 64 and 128, with and without a bias, and K = 0.
The TTFT decoder tests (test_ttft_gpu.py) run the fused path inside whole prefills, TP shards included.
"""
from __future__ import annotations

import pytest
import torch

import _native
import mma
import ttft
from mma import matmul, matmul_bias_rope

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _tables(S, D, device, dtype):
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    freqs = torch.outer(torch.arange(S, device=device, dtype=torch.float32), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _case(S, K, heads, rot_heads, D, dtype, with_bias, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    N = heads * D
    a = (torch.randn(S, K, generator=g, device=device) / K ** 0.5).to(dtype)
    w = (torch.randn(K, N, generator=g, device=device)).to(dtype)
    bias = torch.randn(N, generator=g, device=device).to(dtype) if with_bias else None
    cos, sin = _tables(S, D, device, dtype)
    return a, w, bias, cos, sin


def _two_pass(a, w, bias, cos, sin, heads, rot_heads, D):
    y = matmul(a, w, stream_k=False)  # whole tiles: the fused kernel's summation order
    ttft._native_bias_rope(y, bias, cos, sin, heads, rot_heads, D)
    return y


CASES = [
    # S, K, heads, rot_heads, head_dim, dtype, bias
    (2048, 3584, 36, 32, 128, torch.bfloat16, True),   # the decoder's QKV projection at TP 1 (CTA pairs)
    (300, 512, 5, 3, 128, torch.bfloat16, True),       # single-CTA kernel, ragged rows, last tile half full
    (300, 512, 5, 3, 128, torch.float16, False),       # fp16, no bias
    (129, 256, 8, 6, 64, torch.bfloat16, True),        # head_dim 64: four heads per tile
    (64, 128, 4, 0, 128, torch.bfloat16, True),        # bias only
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "S{}K{}H{}R{}D{}-{}-{}".format(
    c[0], c[1], c[2], c[3], c[4], str(c[5])[6:], "bias" if c[6] else "nobias"))
def test_fused_equals_two_pass(case, cuda_device):
    S, K, heads, rot_heads, D, dtype, with_bias = case
    a, w, bias, cos, sin = _case(S, K, heads, rot_heads, D, dtype, with_bias, cuda_device, seed=S + K + D)
    fused = matmul_bias_rope(a, w, bias, cos, sin, rope_cols=rot_heads * D, head_dim=D)
    assert torch.equal(fused, _two_pass(a, w, bias, cos, sin, heads, rot_heads, D))


def test_fused_equals_pytorch_expression(cuda_device):
    S, K, nq, nkv, D = 257, 640, 6, 2, 128
    a, w, bias, cos, sin = _case(S, K, nq + 2 * nkv, nq + nkv, D, torch.bfloat16, True, cuda_device, seed=3)
    ref = matmul(a, w, stream_k=False) + bias
    q = ref[:, : nq * D].view(S, nq, D)
    k = ref[:, nq * D:(nq + nkv) * D].view(S, nkv, D)
    q_ref = q * cos[:, None, :] + ttft._rotate_half(q) * sin[:, None, :]
    k_ref = k * cos[:, None, :] + ttft._rotate_half(k) * sin[:, None, :]
    out = matmul_bias_rope(a, w, bias, cos, sin, rope_cols=(nq + nkv) * D, head_dim=D)
    assert torch.equal(out[:, : nq * D].view(S, nq, D), q_ref)
    assert torch.equal(out[:, nq * D:(nq + nkv) * D].view(S, nkv, D), k_ref)
    assert torch.equal(out[:, (nq + nkv) * D:], ref[:, (nq + nkv) * D:])


def test_empty_contraction_gives_rope_of_bias(cuda_device):
    S, N, D = 40, 384, 128
    g = torch.Generator(device=cuda_device).manual_seed(4)
    bias = torch.randn(N, generator=g, device=cuda_device).to(torch.bfloat16)
    cos, sin = _tables(S, D, cuda_device, torch.bfloat16)
    a = torch.empty(S, 0, device=cuda_device, dtype=torch.bfloat16)
    w = torch.empty(0, N, device=cuda_device, dtype=torch.bfloat16)
    c = torch.full((S, N), 7.0, device=cuda_device, dtype=torch.bfloat16)
    mma._gemm(a, w, c, S, N, 0, lda=1, ldb=N, ldc=N, round_f16=False, epilogue=_native.FAB_GEMM_EPILOGUE_BIAS_ROPE,
              rope=(bias, cos, sin, 2 * D, D))
    ref = torch.zeros(S, N, device=cuda_device, dtype=torch.bfloat16)
    ttft._native_bias_rope(ref, bias, cos, sin, N // D, 2, D)
    assert torch.equal(c, ref)
