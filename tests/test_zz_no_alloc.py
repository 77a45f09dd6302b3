"""fab_attention_fwd_splitkv_static: the split-KV path with its partials in the library's own 8 MiB device
array, for callers that cannot allocate device memory.  Checked against the workspace entry point
(fab_attention_fwd_splitkv) on the same inputs, two calls in a row.

This file is named to be collected last, and passes alone as well as after the other tests.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import _native

STATIC_SCRATCH_BYTES = 8 << 20


def _params(q, k, v, o, lse=None, causal=False):
    B, Hq, M, D = q.shape
    _, Hkv, N, _ = k.shape
    p = _native.FabAttentionParams()
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.q_stride_b, p.q_stride_h, p.q_stride_s = q.stride()[:3]
    p.k_stride_b, p.k_stride_h, p.k_stride_s = k.stride()[:3]
    p.v_stride_b, p.v_stride_h, p.v_stride_s = v.stride()[:3]
    p.o_stride_b, p.o_stride_h, p.o_stride_s = o.stride()[:3]
    if lse is not None:
        p.lse_stride_b, p.lse_stride_h, p.lse_stride_s = lse.stride()
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim = B, Hq, Hkv, M, N, D
    p.dtype = _native.dtype_code(q.dtype)
    p.sm_scale = D ** -0.5
    p.causal = 1 if causal else 0
    return p


@pytest.mark.gpu
@pytest.mark.parametrize("shape, splits", [((1, 28, 4, 1, 8192, 128), 16), ((2, 8, 2, 3, 5000, 64), 0)])
def test_static_scratch_matches_workspace_entry(shape, splits, cuda_device):
    B, Hq, Hkv, M, N, D = shape
    g = torch.Generator().manual_seed(41)
    q = torch.randn(B, Hq, M, D, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(cuda_device)
    v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(cuda_device)
    lib = _native.lib
    stream = ctypes.c_void_p(_native.current_stream_handle(cuda_device))

    o_ref = torch.empty_like(q)
    lse_ref = torch.empty(B, Hq, M, device=cuda_device, dtype=torch.float32)
    p_ref = _params(q, k, v, o_ref, lse_ref)
    need, used = ctypes.c_size_t(0), ctypes.c_int(0)
    _native.check(lib.fab_attention_fwd_splitkv_workspace(ctypes.byref(p_ref), splits, ctypes.byref(need),
                                                          ctypes.byref(used)), "workspace")
    assert used.value > 1 and 0 < need.value <= STATIC_SCRATCH_BYTES
    ws = torch.zeros(need.value, device=cuda_device, dtype=torch.uint8)
    _native.check(lib.fab_attention_fwd_splitkv(ctypes.byref(p_ref), splits, ws.data_ptr(), need.value, stream),
                  "workspace entry")

    for _ in range(2):  # two calls in a row reuse the same static array
        o = torch.full_like(q, float("nan"))
        lse = torch.full((B, Hq, M), float("nan"), device=cuda_device, dtype=torch.float32)
        _native.check(lib.fab_attention_fwd_splitkv_static(ctypes.byref(_params(q, k, v, o, lse)), splits, stream),
                      "static entry")
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref)
        assert torch.equal(lse, lse_ref)
    assert _native.device_error() == 0


def test_static_scratch_rejects_oversize_requests():
    """A plan whose partials exceed the 8 MiB array is refused before anything touches the device."""
    B, Hq, Hkv, M, N, D = 4, 32, 8, 16, 65536, 128
    p = _native.FabAttentionParams()
    p.q = p.k = p.v = p.o = 4096  # never dereferenced: the request is refused first
    p.q_stride_b, p.q_stride_h, p.q_stride_s = Hq * M * D, M * D, D
    p.k_stride_b, p.k_stride_h, p.k_stride_s = Hkv * N * D, N * D, D
    p.v_stride_b, p.v_stride_h, p.v_stride_s = Hkv * N * D, N * D, D
    p.o_stride_b, p.o_stride_h, p.o_stride_s = Hq * M * D, M * D, D
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim = B, Hq, Hkv, M, N, D
    p.dtype = _native.FAB_DTYPE_BF16
    p.sm_scale = D ** -0.5
    need = ctypes.c_size_t(0)
    assert _native.lib.fab_attention_fwd_splitkv_workspace(ctypes.byref(p), 16, ctypes.byref(need), None) == 0
    assert need.value > STATIC_SCRATCH_BYTES
    assert _native.lib.fab_attention_fwd_splitkv_static(ctypes.byref(p), 16, None) == _native.FAB_ERR_WORKSPACE
    with pytest.raises(ValueError, match="workspace"):
        _native.check(_native.FAB_ERR_WORKSPACE, "fab_attention_fwd_splitkv_static")
