"""Split-K matmul (a cluster of CTAs shares each 128x256 tile's K; partial sums meet in distributed shared
memory) against the oracle.

16-bit inputs take this kernel when the output has at most a quarter as many 128x256 tiles as there are SMs and K
has at least 48 64-deep blocks; `mma.kernel_plan` reports the choice and every shape here asserts it.  Tolerance
(the acceptance bar for 16-bit outputs): max-abs 2e-2 and rtol 1e-2 of the fp32 oracle on inputs ~ N(0,1)/sqrt(K).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _native
from mma import _gemm, kernel_plan, matmul
from oracle.mma_oracle import tiled_matmul

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
NAME = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _inputs(M, N, K, dtype, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    a = (torch.randn(M, K, generator=g, device=device) / K ** 0.5).to(dtype)
    b = (torch.randn(K, N, generator=g, device=device) / K ** 0.5).to(dtype)
    return a, b


def _check(a, b, c, round_f16=False):
    ref = tiled_matmul(a.float().cpu().numpy(), b.float().cpu().numpy(), round_f16=round_f16,
                       out_dtype=NAME[c.dtype])
    torch.testing.assert_close(c.float().cpu(), torch.from_numpy(np.asarray(ref, np.float32)), rtol=RTOL, atol=ATOL)


SHAPES = [
    # M, N, K, splits the plan may take (the largest whose clusters all fit at once; a cluster of 8 needs 8 SMs
    # of one GPC, so how many fit depends on the part)
    (16, 3584, 3584, {4, 8}),    # one row block, 14 tiles (decode-like)
    (300, 1000, 3080, {4, 8}),   # ragged M, N and K: 12 tiles, 49 K blocks (the last one partial)
    (1024, 1024, 4096, {2, 4}),  # 32 tiles
    (512, 512, 4096, {8}),       # 8 tiles
    (130, 200, 4000, {8}),       # 2 tiles
    (1, 64, 8192, {8}),          # one row, one ragged tile
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "M{}N{}K{}".format(*s[:3]))
@pytest.mark.parametrize("dtype, out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                              (torch.bfloat16, torch.float32), (torch.float16, torch.bfloat16)],
                         ids=lambda d: NAME[d])
def test_splitk_matches_oracle(shape, dtype, out_dtype, cuda_device):
    M, N, K, splits = shape
    kernel, split, _ = kernel_plan(M, N, K, dtype, out_dtype)
    assert kernel == "splitk" and split in splits
    a, b = _inputs(M, N, K, dtype, cuda_device, seed=M + N + K)
    _check(a, b, matmul(a, b, out_dtype=out_dtype))


def test_splitk_round_f16(cuda_device):
    a, b = _inputs(300, 1000, 3080, torch.bfloat16, cuda_device, seed=3)
    assert kernel_plan(300, 1000, 3080)[0] == "splitk"
    _check(a, b, matmul(a, b, round_f16=True), round_f16=True)


def test_splitk_leading_dimensions(cuda_device):
    """Row-major views with padded leading dimensions, and a strided output whose padding stays untouched."""
    a_full, b_full = _inputs(700, 1200, 3200, torch.float16, cuda_device, seed=13)
    a = a_full[:, :3136]
    b = b_full[:3136, 64:1064]
    c_full = torch.full((700, 1088), 5.0, device=cuda_device, dtype=torch.float16)
    c = c_full[:, :1000]
    assert kernel_plan(700, 1000, 3136, torch.float16)[0] == "splitk"
    _gemm(a, b, c, 700, 1000, 3136, lda=a.stride(0), ldb=b.stride(0), ldc=c.stride(0), round_f16=False)
    _check(a, b, c)
    assert torch.all(c_full[:, 1000:] == 5.0)


def test_splitk_deterministic_and_close_to_single_pass(cuda_device):
    a, b = _inputs(512, 512, 4096, torch.bfloat16, cuda_device, seed=21)
    c1, c2 = matmul(a, b), matmul(a, b)
    assert torch.equal(c1, c2)
    ref = (a.float() @ b.float())
    torch.testing.assert_close(c1.float(), ref, rtol=RTOL, atol=ATOL)


def test_large_problems_do_not_split(cuda_device):
    assert kernel_plan(2048, 2048, 2048)[0] == "single"
    assert kernel_plan(8192, 8192, 8192)[0] == "pair"
    assert kernel_plan(1024, 1024, 1024, torch.float32)[0] == "single"  # tf32 keeps the single-CTA kernel
    assert kernel_plan(1024, 1024, 1024)[0] == "single"                # 16 K blocks: the exchange costs more
    assert kernel_plan(16, 18944, 3584)[0] == "pair"                   # 74 tiles: enough to spread the loads
