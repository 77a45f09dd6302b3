"""Matmul on the GPU, through the C ABI, against the reference's outputs and the oracle.

Tolerance (the acceptance bar for 16-bit outputs): within max-abs 2e-2 and rtol 1e-2 of the
fp32 oracle on the same inputs (inputs ~ N(0,1)/sqrt(K) keep |C| ~ 1).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import _native
import mma
from mma import _matmul_contiguous_kernel, _select_2d_contiguous_config, matmul
from oracle.mma_oracle import tiled_matmul

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = [c for c in json.loads((GOLDEN / "golden.json").read_text())["cases"] if c["kind"] == "matmul"]
ARRAYS = np.load(GOLDEN / "golden.npz")
NAME = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _close(actual, expected, rtol=RTOL, atol=ATOL):
    torch.testing.assert_close(actual.detach().float().cpu(), torch.as_tensor(np.asarray(expected, np.float32)),
                               rtol=rtol, atol=atol)


def _inputs(M, N, K, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g) / K ** 0.5).to(dtype)
    b = (torch.randn(K, N, generator=g) / K ** 0.5).to(dtype)
    return a, b


def _launch_like_reference(a, b, c):
    """The reference test's call sequence (test_mma.py:304-333)."""
    M, K = a.shape
    N = b.shape[1]
    bm, bn, bk, gm, nw, ns = _select_2d_contiguous_config(M, N, K)
    grid = (-(-M // bm) * -(-N // bn),)
    _matmul_contiguous_kernel[grid](a, b, c, M, N, K, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk, GROUP_M=gm,
                                    USE_CACHE_EVICTION_HINTS=mma._supports_contiguous_cache_eviction_hints(a.device),
                                    num_warps=nw, num_stages=ns)
    return c


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_reference_golden(case, cuda_device):
    a = torch.from_numpy(ARRAYS[f"{case['name']}.a"]).to(cuda_device)
    b = torch.from_numpy(ARRAYS[f"{case['name']}.b"]).to(cuda_device)
    c = torch.empty(a.shape[0], b.shape[1], dtype=a.dtype, device=cuda_device)
    _launch_like_reference(a, b, c)
    ref = ARRAYS[f"{case['name']}.c"].astype(np.float32)
    _close(c, ref)
    # Same fp32 sums in another order, same fp16 rounding: at most an ulp or so apart.
    _close(c, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("mkn", [(1024, 256, 1024), (8192, 256, 8192), (2048, 2048, 2048)],
                         ids=lambda s: "M{}K{}N{}".format(*s))
def test_reference_test_shapes(mkn, dtype, cuda_device):
    """The reference test's (M, K, N) cases (test_mma.py:42-46) and a square size, through its call sequence."""
    M, K, N = mkn
    a, b = _inputs(M, N, K, dtype, seed=1)
    c = torch.empty(M, N, dtype=dtype, device=cuda_device)
    _launch_like_reference(a.to(cuda_device), b.to(cuda_device), c)
    rows = torch.arange(M) if M <= 2048 else torch.tensor([0, 129, M // 2, M - 1])
    ref = tiled_matmul(a[rows].float().numpy(), b.float().numpy(), block_k=K, round_f16=True, out_dtype=NAME[dtype])
    _close(c[rows.to(cuda_device)], ref)


@pytest.mark.parametrize("dtype, out_dtype", [
    (torch.float16, torch.float16), (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32),
    (torch.float16, torch.bfloat16), (torch.float32, torch.float32), (torch.float32, torch.float16),
], ids=lambda d: NAME.get(d, str(d)))
@pytest.mark.parametrize("shape", [(128, 256, 64), (129, 72, 40), (1000, 520, 264), (1, 8, 8), (300, 264, 96),
                                   (640, 1024, 1000)], ids=lambda s: "M{}N{}K{}".format(*s))
@pytest.mark.parametrize("round_f16", [False, True], ids=["no_round", "round_f16"])
def test_oracle_parity(shape, dtype, out_dtype, round_f16, cuda_device):
    M, N, K = shape
    per16 = 16 // torch.empty((), dtype=dtype).element_size()
    if K % per16 or N % per16 or N % (16 // torch.empty((), dtype=out_dtype).element_size()):
        pytest.skip("row length not a multiple of 16 bytes")
    a, b = _inputs(M, N, K, dtype, seed=M * 7 + N + K)
    c = matmul(a.to(cuda_device), b.to(cuda_device), out_dtype=out_dtype, round_f16=round_f16)
    assert c.dtype == out_dtype
    _close(c, tiled_matmul(a.float().numpy(), b.float().numpy(), round_f16=round_f16, out_dtype=NAME[out_dtype]))


def test_leading_dimensions(cuda_device):
    """Row-major views with padded leading dimensions (the TTFT model's fused projections use these)."""
    a_full, b_full = _inputs(300, 512, 384, torch.bfloat16, seed=4)
    a = a_full.to(cuda_device)[:, :320]
    b = b_full.to(cuda_device)[:320, 64:448]
    c = matmul(a, b)
    _close(c, tiled_matmul(a.float().cpu().numpy(), b.float().cpu().numpy(), round_f16=False, out_dtype="bf16"))


def test_empty_contraction_gives_zero(cuda_device):
    a = torch.empty(64, 0, dtype=torch.bfloat16, device=cuda_device)
    b = torch.empty(0, 128, dtype=torch.bfloat16, device=cuda_device)
    c = matmul(a, b)
    assert torch.count_nonzero(c) == 0


def test_deterministic(cuda_device):
    a, b = _inputs(1536, 1792, 2048, torch.bfloat16, seed=5)
    a, b = a.to(cuda_device), b.to(cuda_device)
    assert torch.equal(matmul(a, b), matmul(a, b))


@pytest.mark.parametrize("n", [4096, 8192, 16384])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
def test_config4_full_size(n, dtype, cuda_device):
    """Benchmark matmul sizes: sampled rows against the oracle plus a column-sum identity over all of C."""
    g = torch.Generator(device=cuda_device).manual_seed(n)
    a = (torch.randn(n, n, generator=g, device=cuda_device) / n ** 0.5).to(dtype)
    b = (torch.randn(n, n, generator=g, device=cuda_device) / n ** 0.5).to(dtype)
    c = torch.empty(n, n, dtype=dtype, device=cuda_device)
    _launch_like_reference(a, b, c)
    rows = torch.tensor([0, 1, n // 3, n // 2 + 5, n - 1])
    ref = tiled_matmul(a[rows].float().cpu().numpy(), b.float().cpu().numpy(), block_k=4096, round_f16=True,
                       out_dtype=NAME[dtype])
    _close(c[rows.to(cuda_device)], ref)
    # 1^T C == (1^T A) B up to the output rounding of each element (linearity over every row).
    lhs = c.sum(dim=0, dtype=torch.float64)
    rhs = a.sum(dim=0, dtype=torch.float64) @ b.double()
    err = (lhs - rhs).abs().max().item()
    assert err < 2e-3 * n ** 0.5 * 8, err
    del a, b, c
    torch.cuda.empty_cache()


# ------------------------------------------------------ narrow tiles for small problems
NARROW = [
    # M, N, K, tile width the plan takes: 256-wide tiles would leave over a quarter of the 148 SMs idle
    (1024, 1024, 1024, 64),   # 32 tiles of 256, 128 of 64
    (1536, 1536, 512, 128),   # 72 tiles of 256, 144 of 128
    (300, 1000, 520, 64),     # ragged M, N and K
    (129, 200, 72, 64),       # one partial K block past the first, ragged everywhere
    (1, 64, 256, 64),         # one row, one tile
]


@pytest.mark.parametrize("shape", NARROW, ids=lambda s: "M{}N{}K{}".format(*s[:3]))
@pytest.mark.parametrize("dtype, out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                              (torch.bfloat16, torch.float32), (torch.float16, torch.bfloat16)],
                         ids=lambda d: NAME[d])
def test_narrow_tiles_match_oracle(shape, dtype, out_dtype, cuda_device):
    M, N, K, width = shape
    assert mma.kernel_plan(M, N, K, dtype, out_dtype) == ("single", 1, width)
    g = torch.Generator(device=cuda_device).manual_seed(M * 7 + N + K)
    a = (torch.randn(M, K, generator=g, device=cuda_device) / K ** 0.5).to(dtype)
    b = (torch.randn(K, N, generator=g, device=cuda_device) / K ** 0.5).to(dtype)
    c = matmul(a, b, out_dtype=out_dtype)
    ref = tiled_matmul(a.float().cpu().numpy(), b.float().cpu().numpy(), round_f16=False, out_dtype=NAME[out_dtype])
    _close(c, ref)


def test_narrow_tiles_round_f16_strided_and_deterministic(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(5)
    a_full = (torch.randn(700, 1104, generator=g, device=cuda_device) / 1000 ** 0.5).to(torch.bfloat16)
    b_full = (torch.randn(1104, 1200, generator=g, device=cuda_device) / 1000 ** 0.5).to(torch.bfloat16)
    a, b = a_full[:, :1000], b_full[:1000, 64:1064]
    assert mma.kernel_plan(700, 1000, 1000)[2] == 64
    c_full = torch.full((700, 1088), 5.0, device=cuda_device, dtype=torch.bfloat16)
    c = c_full[:, :1000]
    mma._gemm(a, b, c, 700, 1000, 1000, lda=a.stride(0), ldb=b.stride(0), ldc=c.stride(0), round_f16=True)
    ref = tiled_matmul(a.float().cpu().numpy(), b.float().cpu().numpy(), round_f16=True, out_dtype="bf16")
    _close(c, ref)
    assert torch.all(c_full[:, 1000:] == 5.0)
    c2 = torch.empty_like(c_full)
    mma._gemm(a, b, c2, 700, 1000, 1000, lda=a.stride(0), ldb=b.stride(0), ldc=c2.stride(0), round_f16=True)
    assert torch.equal(c2[:, :1000], c)


def test_wide_tiles_where_they_fill_the_gpu(cuda_device):
    assert mma.kernel_plan(2048, 2048, 2048) == ("single", 1, 256)
    assert mma.kernel_plan(1024, 1024, 1024, torch.float32) == ("single", 1, 256)  # tf32 keeps 256
