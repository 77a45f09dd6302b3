"""Split-KV ("flash-decoding") attention on the GPU against the oracle and the single-pass kernel.

Each key range's attention goes to an fp32 workspace and a second kernel merges the ranges by their LSE.
Tolerance (the acceptance bar for 16-bit outputs): fp16/bf16 outputs within max-abs 2e-2 and rtol 1e-2 of the fp32 oracle on
the same inputs; LSE in fp32 within 2e-3.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import _native
from flash_atten import attention_forward, attention_forward_splitkv, splitkv_workspace_bytes
from oracle.fa_oracle import tiled_attention_forward

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
LSE_ATOL = 2e-3
P_DTYPE = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _inputs(shape, dtype, seed):
    B, Hq, Hkv, M, N, D = shape
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, M, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    return q, k, v


def _close(actual, expected, rtol=RTOL, atol=ATOL):
    expected = torch.as_tensor(np.asarray(expected, dtype=np.float32))
    torch.testing.assert_close(actual.detach().float().cpu(), expected, rtol=rtol, atol=atol)


CASES = [
    # (B, Hq, Hkv, M, N, D), dtype, causal, num_splits
    ((1, 28, 4, 1, 4097, 128), torch.bfloat16, False, 0),     # one decode step, Qwen2.5-7B heads, packed
    ((1, 28, 4, 1, 4097, 128), torch.bfloat16, False, 5),
    ((2, 8, 8, 3, 2000, 64), torch.float16, False, 7),         # no grouping
    ((1, 16, 4, 16, 10000, 128), torch.bfloat16, False, 0),   # 16-token block, packed rows 64
    ((1, 4, 2, 5, 3000, 256), torch.bfloat16, False, 4),
    ((1, 4, 1, 2, 1500, 64), torch.float32, False, 3),
    ((1, 2, 2, 300, 700, 128), torch.float16, True, 3),        # causal: later splits see no key for early rows
    ((1, 8, 2, 4, 1000, 128), torch.bfloat16, True, 6),        # causal, most splits empty
    ((1, 8, 2, 2, 129, 80), torch.bfloat16, False, 2),         # ragged head dim and key count
]


@pytest.mark.parametrize("shape, dtype, causal, splits", CASES,
                         ids=lambda x: "x".join(map(str, x)) if isinstance(x, tuple) else str(x))
def test_splitkv_matches_oracle(shape, dtype, causal, splits, cuda_device):
    q, k, v = _inputs(shape, dtype, seed=zlib.crc32(repr((shape, str(dtype), causal, splits)).encode()))
    o, lse = attention_forward_splitkv(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=causal,
                                       return_lse=True, num_splits=splits)
    ro, rl = tiled_attention_forward(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                                     p_dtype=P_DTYPE[dtype])
    _close(o, ro)
    _close(lse, rl, rtol=1e-4, atol=LSE_ATOL if dtype != torch.float32 else 1e-2)
    # and the single-pass kernel on the same inputs
    o1 = attention_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=causal)
    torch.testing.assert_close(o.float(), o1.float(), rtol=RTOL, atol=ATOL)


def test_split_count_reported_and_respected(cuda_device):
    need, used = splitkv_workspace_bytes((1, 28, 1, 128), (1, 4, 32768, 128), torch.bfloat16, num_splits=0)
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    assert used == sms // 4  # four packed key/value heads, at most one CTA per SM, one wave
    assert need > 0
    need1, used1 = splitkv_workspace_bytes((1, 28, 1, 128), (1, 4, 32768, 128), torch.bfloat16, num_splits=1)
    assert (need1, used1) == (0, 1)


def test_unpacked_when_heads_are_not_evenly_spaced(cuda_device):
    """q as a [B, M, H, D] buffer viewed as [B, H, M, D]: heads are D apart, positions H*D apart, so the
    query heads of a key/value head cannot share a tile; the kernel falls back to one head per tile."""
    B, Hq, Hkv, M, N, D = 1, 8, 2, 6, 3000, 128
    g = torch.Generator().manual_seed(31)
    qs = torch.randn(B, M, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16)
    qd = qs.to(cuda_device).transpose(1, 2)
    o = attention_forward_splitkv(qd, k.to(cuda_device), v.to(cuda_device), num_splits=5)
    ro, _ = tiled_attention_forward(qs.transpose(1, 2).float().numpy(), k.float().numpy(), v.float().numpy(),
                                    causal=False, p_dtype="bf16")
    _close(o, ro)


def test_caller_workspace_reused_across_calls(cuda_device):
    shape = (1, 28, 4, 1, 8192, 128)
    q, k, v = (t.to(cuda_device) for t in _inputs(shape, torch.bfloat16, seed=32))
    need, _ = splitkv_workspace_bytes(tuple(q.shape), tuple(k.shape), torch.bfloat16, num_splits=16)
    ws = torch.zeros(need, device=cuda_device, dtype=torch.uint8)
    a = attention_forward_splitkv(q, k, v, num_splits=16, workspace=ws)
    # The workspace ends with one arrival counter per row group (4 key/value heads here: one 256-byte
    # block), which every call leaves at zero; stale partials before it must not matter, since every
    # split rewrites its own.
    torch.cuda.synchronize()
    assert bool((ws[-256:] == 0).all())
    ws[:-256].fill_(0xFF)
    b = attention_forward_splitkv(q, k, v, num_splits=16, workspace=ws)
    torch.cuda.synchronize()
    assert bool((ws[-256:] == 0).all())
    assert torch.equal(a, b)


def test_no_keys_gives_nan_rows(cuda_device):
    q = torch.randn(1, 4, 2, 64, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(1, 2, 0, 64, device=cuda_device, dtype=torch.bfloat16)
    o, lse = attention_forward_splitkv(q, k, k, return_lse=True, num_splits=4)
    assert torch.isnan(o.float()).all()
    assert torch.isneginf(lse).all()
