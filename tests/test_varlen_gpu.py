"""Packed variable-length batches (cu_seqlens) on the GPU, each sequence against the oracle on its own slice.

Tolerance (the acceptance bar for 16-bit outputs): fp16/bf16 outputs within max-abs 2e-2 and rtol 1e-2 of the fp32 oracle;
LSE in fp32 within 2e-3.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import _native
from flash_atten import attention_forward, attention_forward_varlen
from oracle.fa_oracle import tiled_attention_forward

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
P_DTYPE = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _cu(lengths):
    return torch.tensor([0, *np.cumsum(lengths)], dtype=torch.int32)


CASES = [
    # q lengths, k lengths, Hq, Hkv, D, dtype, causal
    ((100, 513, 1), (100, 513, 1), 8, 2, 128, torch.bfloat16, True),
    ((100, 513, 1), (100, 513, 1), 8, 2, 128, torch.bfloat16, False),
    ((5, 300, 0, 257), (700, 20, 9, 257), 4, 4, 64, torch.float16, False),   # cross lengths, an empty query set
    ((129, 64), (129, 64), 2, 1, 256, torch.bfloat16, True),
    ((70, 33), (99, 45), 2, 2, 80, torch.bfloat16, True),                    # ragged head dim
    ((40, 200), (40, 200), 2, 2, 64, torch.float32, False),
    ((3, 4), (0, 10), 2, 2, 64, torch.bfloat16, False),                       # a sequence with no keys
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"q{c[0]}k{c[1]}H{c[2]}/{c[3]}D{c[4]}{str(c[5])[6:]}{'c' if c[6] else ''}")
def test_varlen_matches_oracle_per_sequence(case, cuda_device):
    lq, lk, Hq, Hkv, D, dtype, causal = case
    g = torch.Generator().manual_seed(zlib.crc32(repr(case).encode()))
    q = torch.randn(sum(lq), Hq, D, generator=g).to(dtype)
    k = torch.randn(sum(lk), Hkv, D, generator=g).to(dtype)
    v = torch.randn(sum(lk), Hkv, D, generator=g).to(dtype)
    cq, ck = _cu(lq), _cu(lk)
    o, lse = attention_forward_varlen(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), cq.to(cuda_device),
                                      ck.to(cuda_device), max(lq), max(lk), causal=causal, return_lse=True)
    o, lse = o.float().cpu(), lse.cpu()
    for b in range(len(lq)):
        qs, ks = slice(int(cq[b]), int(cq[b + 1])), slice(int(ck[b]), int(ck[b + 1]))
        if lq[b] == 0:
            continue
        if lk[b] == 0:
            assert torch.isnan(o[qs]).all() and torch.isneginf(lse[:, qs]).all()
            continue
        qb = q[qs].transpose(0, 1)[None].float().numpy()
        kb = k[ks].transpose(0, 1)[None].float().numpy()
        vb = v[ks].transpose(0, 1)[None].float().numpy()
        ro, rl = tiled_attention_forward(qb, kb, vb, causal=causal, p_dtype=P_DTYPE[dtype])
        torch.testing.assert_close(o[qs], torch.from_numpy(ro[0]).transpose(0, 1), rtol=RTOL, atol=ATOL)
        lse_tol = 1e-2 if dtype == torch.float32 else 2e-3
        torch.testing.assert_close(lse[:, qs], torch.from_numpy(rl[0]), rtol=1e-4, atol=lse_tol)


def test_varlen_equals_dense_for_equal_lengths(cuda_device):
    """Equal lengths: the packed path and the dense [B, H, S, D] path compute the same thing."""
    B, H, S, D = 3, 4, 300, 128
    g = torch.Generator().manual_seed(51)
    q, k, v = (torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    cu = _cu([S] * B).to(cuda_device)
    ov = attention_forward_varlen(q.reshape(B * S, H, D), k.reshape(B * S, H, D), v.reshape(B * S, H, D), cu, cu, S, S,
                                  causal=True)
    od = attention_forward(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), causal=True)
    assert torch.equal(ov.reshape(B, S, H, D), od.transpose(1, 2))
