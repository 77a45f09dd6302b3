"""Stream-K schedule of the CTA-pair matmul: the tiles past the full waves of SM pairs are cut along K.

With T tiles on P pairs, whole tiles leave T % P pairs busy in the last wave (the TTFT model's down_proj at
2048 tokens: 112 tiles on 74 pairs).  Stream-K runs the full waves whole and splits the K blocks of the
remaining tiles evenly over all pairs; the pair holding a tile's last K block adds the other pairs' fp32
pieces from the workspace.  Checked here: the plan takes it where it is chosen, results against the fp32
oracle at the acceptance tolerance (max-abs 2e-2, rtol 1e-2 on N(0,1)/sqrt(K) inputs), bitwise determinism,
the workspace's flag words back at zero after every call (the precondition of the next), CUDA-graph replay,
the folded-norm row scale, and the whole-tile layout when no workspace is given.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _native
import mma
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
    M = a.shape[0]
    rows = torch.tensor(sorted({0, 1, 127, 128, 255, 256, M // 2 + 3, M - 129, M - 1}))
    ref = tiled_matmul(a[rows].float().cpu().numpy(), b.float().cpu().numpy(), round_f16=round_f16,
                       out_dtype=NAME[c.dtype])
    torch.testing.assert_close(c[rows.to(c.device)].float().cpu(), torch.from_numpy(np.asarray(ref, np.float32)),
                               rtol=RTOL, atol=ATOL)
    full = a.float() @ b.float()  # every element against an fp32 product
    if round_f16:
        full = full.half().float()
    torch.testing.assert_close(c.float(), full.to(c.dtype).float(), rtol=RTOL, atol=ATOL)


def _flags_zero(device):
    grid = mma.kernel_grid(2048, 3584, 18944)  # the pair count of a stream-K launch: 2 CTAs per pair
    flags = mma.gemm_workspace(device, 0)[: (grid // 2) * 8 * 4].view(torch.int32)
    return bool((flags == 0).all())


SHAPES = [
    # M, K, N, dtype -- all take the stream-K schedule (asserted)
    (2048, 18944, 3584, torch.bfloat16),  # TTFT down_proj at 2048 tokens: 112 tiles on 74 pairs
    (2381, 9000, 2376, torch.float16),    # ragged in every dimension, K not a multiple of 64
    (1800, 12000, 4000, torch.bfloat16),  # ragged, 8 x 16 tiles
]


@pytest.mark.parametrize("M, K, N, dtype", SHAPES, ids=lambda x: NAME[x] if isinstance(x, torch.dtype) else str(x))
def test_matches_oracle_and_is_deterministic(M, K, N, dtype, cuda_device):
    assert mma.kernel_plan(M, N, K, dtype)[0] == "pair_streamk"
    a, b = _inputs(M, N, K, dtype, cuda_device, seed=M + N + K)
    c1 = mma.matmul(a, b)
    c2 = mma.matmul(a, b)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
    _check(a, b, c1)
    assert _flags_zero(cuda_device)


def test_down_proj_takes_stream_k(cuda_device):
    """112 tiles on 74 pairs with K = 18944: the schedule is chosen, and never with more pairs than can be
    resident.  Short K (the o_proj, K = 3584) keeps whole tiles."""
    plan = mma.kernel_plan(2048, 3584, 18944, torch.bfloat16)
    assert plan[0] == "pair_streamk", plan
    assert mma.kernel_plan(2048, 3584, 3584, torch.bfloat16)[0] == "pair"
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    assert 0 < mma.kernel_grid(2048, 3584, 18944) <= sms


def test_fp32_output_and_fp16_rounding(cuda_device):
    M, K, N = 2048, 18944, 3584
    a, b = _inputs(M, N, K, torch.float16, cuda_device, seed=7)
    c = torch.empty(M, N, device=cuda_device, dtype=torch.float32)
    mma._gemm(a, b, c, M, N, K, lda=K, ldb=N, ldc=N, round_f16=True)
    _check(a, b, c, round_f16=True)


def test_whole_tiles_without_workspace_agree(cuda_device):
    """The same product without a workspace runs whole tiles; the two differ only in fp32 summation order."""
    M, K, N = 2048, 18944, 3584
    a, b = _inputs(M, N, K, torch.bfloat16, cuda_device, seed=8)
    sk = mma.matmul(a, b)
    whole = mma.matmul(a, b, stream_k=False)
    torch.testing.assert_close(sk.float(), whole.float(), rtol=RTOL, atol=ATOL)


def test_with_row_scale(cuda_device):
    M, K, N = 2048, 18944, 3584
    a, b = _inputs(M, N, K, torch.bfloat16, cuda_device, seed=9)
    rs = torch.rand(M, device=cuda_device) + 0.5
    c = torch.empty(M, N, device=cuda_device, dtype=torch.bfloat16)
    mma._gemm(a, b, c, M, N, K, lda=K, ldb=N, ldc=N, round_f16=False, row_scale=rs)
    torch.testing.assert_close(c.float(), rs[:, None] * (a.float() @ b.float()), rtol=RTOL, atol=ATOL)


def test_inside_a_cuda_graph(cuda_device):
    """Graph replays reuse the workspace; the flags the kernel clears make every replay start clean."""
    M, K, N = 2048, 18944, 3584
    a, b = _inputs(M, N, K, torch.bfloat16, cuda_device, seed=10)
    mma.matmul(a, b)  # a first call outside the capture sizes the shared workspace
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            out = mma.matmul(a, b)
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    for seed in (11, 12):
        a2, b2 = _inputs(M, N, K, torch.bfloat16, cuda_device, seed=seed)
        a.copy_(a2)
        b.copy_(b2)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, mma.matmul(a, b))
    graph.reset()
    _check(a, b, out)
