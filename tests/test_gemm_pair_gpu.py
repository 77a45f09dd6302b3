"""The CTA-pair matmul (tcgen05 cta_group::2, 256x256 tiles per pair of SMs) against the oracle.

16-bit inputs take this kernel when the problem has at least one wave of pair tiles (one per two SMs);
every shape here does (asserted).  Tiles are 256 columns wide, or 224 where that leaves fewer pairs idle in
the last wave and K <= 8192; the shapes below exercise both.  Tolerance (the acceptance bar for 16-bit outputs): max-abs 2e-2 and rtol 1e-2 of the fp32
oracle on inputs ~ N(0,1)/sqrt(K).  Rows are sampled for the oracle (first, last, ragged edge, a few in
between); a column-sum identity checks every row.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import _native
from mma import matmul
from oracle.mma_oracle import tiled_matmul

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
NAME = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _pair_tiles(M, N):
    return -(-M // 256) * -(-N // 256)


def _inputs(M, N, K, dtype, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    a = (torch.randn(M, K, generator=g, device=device) / K ** 0.5).to(dtype)
    b = (torch.randn(K, N, generator=g, device=device) / K ** 0.5).to(dtype)
    return a, b


def _check(a, b, c, round_f16):
    M = a.shape[0]
    rows = torch.tensor(sorted({0, 1, 127, 128, 255, 256, M // 2 + 3, M - 129, M - 1}))
    ref = tiled_matmul(a[rows].float().cpu().numpy(), b.float().cpu().numpy(), round_f16=round_f16,
                       out_dtype=NAME[c.dtype])
    torch.testing.assert_close(c[rows.to(c.device)].float().cpu(), torch.from_numpy(np.asarray(ref, np.float32)),
                               rtol=RTOL, atol=ATOL)
    # Every row: 1^T C == (1^T A) B up to each element's output rounding.
    lhs = c.float().sum(dim=0, dtype=torch.float64)
    rhs = (a.double().sum(dim=0) @ b.double())
    tol = 2e-2 * M ** 0.5 + 1e-2 * rhs.abs()
    assert torch.all((lhs - rhs).abs() <= tol)


SHAPES = [
    # M, N, K: ragged in every dimension, K not a multiple of the 64-deep stage
    (2381, 2376, 1000),
    (2304, 4672, 520),
    (4097, 2304, 136),
    (2048, 3584, 18944),   # the TTFT down projection at TP=1
    (3000, 3072, 520),     # 256-wide tiles (the others pick 224: fewer idle pairs in the last wave)
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "M{}N{}K{}".format(*s))
@pytest.mark.parametrize("dtype, out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                              (torch.bfloat16, torch.float32), (torch.float16, torch.bfloat16)],
                         ids=lambda d: NAME[d])
def test_pair_matches_oracle(shape, dtype, out_dtype, cuda_device):
    M, N, K = shape
    assert _pair_tiles(M, N) >= torch.cuda.get_device_properties(cuda_device).multi_processor_count // 2
    a, b = _inputs(M, N, K, dtype, cuda_device, seed=M + N + K)
    c = matmul(a, b, out_dtype=out_dtype)
    _check(a, b, c, round_f16=False)


def test_pair_round_f16(cuda_device):
    a, b = _inputs(2381, 2376, 1000, torch.bfloat16, cuda_device, seed=9)
    _check(a, b, matmul(a, b, round_f16=True), round_f16=True)


def test_pair_leading_dimensions(cuda_device):
    """Row-major views with padded leading dimensions, and a strided output."""
    a_full, b_full = _inputs(2500, 3000, 1104, torch.bfloat16, cuda_device, seed=13)
    a = a_full[:, :1000]
    b = b_full[:1000, 64:2624]
    c_full = torch.full((2500, 2688), 5.0, device=cuda_device, dtype=torch.bfloat16)
    c = c_full[:, :2560]
    from mma import _gemm
    _gemm(a, b, c, 2500, 2560, 1000, lda=a.stride(0), ldb=b.stride(0), ldc=c.stride(0), round_f16=False)
    _check(a, b, c, round_f16=False)
    assert torch.all(c_full[:, 2560:] == 5.0)


def test_pair_deterministic(cuda_device):
    a, b = _inputs(3000, 3072, 704, torch.bfloat16, cuda_device, seed=21)
    assert torch.equal(matmul(a, b), matmul(a, b))


# ------------------------------------------------ dynamic tile order (cluster launch control)
def test_dynamic_order_launches_one_cluster_per_tile(cuda_device):
    """Whole-tile launches with more tiles than resident pairs start one two-CTA cluster per tile; running
    clusters take the tiles of clusters that have not started.  Every tile is computed exactly once."""
    import mma

    M, N, K = 4096, 4096, 1024
    assert mma.kernel_plan(M, N, K, torch.bfloat16)[0] == "pair"
    assert mma.kernel_grid(M, N, K) == 2 * _pair_tiles(M, N)
    a, b = _inputs(M, N, K, torch.bfloat16, cuda_device, seed=41)
    c = matmul(a, b)
    torch.testing.assert_close(c.float(), (a.float() @ b.float()).to(torch.bfloat16).float(), rtol=RTOL, atol=ATOL)
    assert torch.equal(c, matmul(a, b))  # the tile order never changes a tile's sums


def test_dynamic_order_on_two_streams_and_in_a_graph(cuda_device):
    """Two launches in flight at once on different streams, and graph replays: the scheduler keeps no state
    outside the launch, so neither interferes with the other."""
    shapes = [(3000, 2800, 712), (2048, 5120, 512)]  # row strides are 16-byte multiples
    ins = [_inputs(M, N, K, torch.bfloat16, cuda_device, seed=50 + i) for i, (M, N, K) in enumerate(shapes)]
    want = [matmul(a, b) for a, b in ins]
    streams = [torch.cuda.Stream(cuda_device) for _ in shapes]
    outs = [None, None]
    torch.cuda.synchronize()
    for _ in range(3):
        for i, st in enumerate(streams):
            with torch.cuda.stream(st):
                outs[i] = matmul(*ins[i])
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            assert torch.equal(o, w)
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            g_out = matmul(*ins[0])
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(g_out, want[0])
    graph.reset()
