"""The C-ABI library loads, exports every declared symbol, and validates arguments.

Runs without a GPU: only entry points that return before touching the device
are called.
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import torch

import _native

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fa_b200.h"


def _declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(fab_[a-z0-9_]+)\s*\(", text))


def test_header_declares_the_boundary():
    names = _declared_functions()
    for required in (
        "fab_flash_attn_fwd_basic",
        "fab_flash_attn_fwd_optimize_shared_mem",
        "fab_flash_attn_fwd_block_d_nomask_contiguous",
        "fab_attention_fwd",
        "fab_matmul_contiguous",
        "fab_gemm",
    ):
        assert required in names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (fab_[a-z0-9_]+)$", out.stdout, flags=re.M))
    declared = _declared_functions()
    assert declared <= exported, f"declared but not exported: {sorted(declared - exported)}"
    for name in declared:
        assert hasattr(_native.lib, name)


def test_python_binding_covers_every_declared_symbol():
    assert _declared_functions() == set(_native.PROTOTYPES)


def test_abi_version_and_error_strings():
    assert _native.lib.fab_abi_version() == _native.ABI_VERSION
    assert _native.error_string(_native.FAB_OK) == "ok"
    for rc in range(1, 7):
        assert _native.error_string(rc) != "unknown error"
    assert _native.error_string(99) == "unknown error"


def test_return_code_mapping():
    _native.check(_native.FAB_OK, "x")
    with pytest.raises(ValueError):
        _native.check(_native.FAB_ERR_INVALID_ARG, "x")
    with pytest.raises(ValueError):
        _native.check(_native.FAB_ERR_UNSUPPORTED, "x")
    with pytest.raises(_native.DeviceTimeoutError):
        _native.check(_native.FAB_ERR_DEVICE_TIMEOUT, "x")
    with pytest.raises(RuntimeError):
        _native.check(_native.FAB_ERR_LAUNCH, "x")
    with pytest.raises(ValueError, match="workspace"):
        _native.check(_native.FAB_ERR_WORKSPACE, "x")


@pytest.mark.parametrize(
    "dtype, D, expect",
    [
        # (head_dim_padded, q_tiles_per_cta, block_n, K/V ring slots, s_buffers)
        (_native.FAB_DTYPE_BF16, 64, (64, 2, 128, 10, 1)),
        (_native.FAB_DTYPE_BF16, 128, (128, 2, 128, 5, 1)),
        (_native.FAB_DTYPE_F16, 96, (128, 2, 128, 5, 1)),
        (_native.FAB_DTYPE_F16, 256, (256, 1, 128, 2, 2)),
        (_native.FAB_DTYPE_F32, 64, (64, 2, 128, 5, 1)),
        (_native.FAB_DTYPE_F32, 128, (128, 1, 128, 2, 2)),
    ],
)
def test_tile_table(dtype, D, expect):
    cfg = _native.fa_config(dtype, D)
    assert (cfg.head_dim_padded, cfg.q_tiles_per_cta, cfg.block_n, cfg.stages, cfg.s_buffers) == expect
    assert cfg.threads == 128 * (1 + cfg.q_tiles_per_cta)
    assert cfg.smem_bytes <= 232448
    assert cfg.tmem_columns in (256, 512)
    used = cfg.q_tiles_per_cta * (cfg.s_buffers * cfg.block_n + cfg.head_dim_padded)
    assert used <= cfg.tmem_columns


def test_tile_table_rejects_out_of_range_head_dims():
    assert _native.fa_config(_native.FAB_DTYPE_BF16, 512) is None
    assert _native.fa_config(_native.FAB_DTYPE_F32, 256) is None
    with pytest.raises(ValueError):
        _native.fa_config(7, 64)


def test_null_and_bad_arguments_are_rejected_before_any_launch():
    lib = _native.lib
    assert lib.fab_attention_fwd(None, None) == _native.FAB_ERR_INVALID_ARG
    assert lib.fab_gemm(None, None) == _native.FAB_ERR_INVALID_ARG
    p = _native.FabGemmParams()
    p.M, p.N, p.K = -1, 8, 8
    assert lib.fab_gemm(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG
    p.M, p.N, p.K, p.in_dtype, p.out_dtype = 8, 8, 8, 9, 0
    assert lib.fab_gemm(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG
    # Empty problems are a no-op.
    p.M, p.N, p.in_dtype = 0, 8, 0
    assert lib.fab_gemm(ctypes.byref(p), None) == _native.FAB_OK
    # SwiGLU epilogue: 2m a multiple of 128, 16-bit output, no fp16 pre-rounding, an unknown mode rejected.
    p.M, p.N, p.K, p.in_dtype, p.out_dtype, p.c, p.ldc = 8, 256, 64, 1, 1, 4096, 128
    for bad in (dict(epilogue=2), dict(epilogue=1, N=192), dict(epilogue=1, out_dtype=2, ldc=256),
                dict(epilogue=1, round_f16=1), dict(epilogue=1, ldc=120)):
        q = _native.FabGemmParams.from_buffer_copy(p)
        for key, val in bad.items():
            setattr(q, key, val)
        assert lib.fab_gemm(ctypes.byref(q), None) == _native.FAB_ERR_INVALID_ARG, bad
    a = _native.FabAttentionParams()
    a.batch, a.heads_q, a.heads_kv, a.seqlen_q, a.seqlen_k, a.head_dim, a.dtype = 1, 4, 3, 16, 16, 64, 1
    a.sm_scale = 0.125
    a.q = a.k = a.v = a.o = 4096
    assert lib.fab_attention_fwd(ctypes.byref(a), None) == _native.FAB_ERR_INVALID_ARG  # 4 % 3 != 0
    a.heads_kv = 2
    a.sm_scale = -1.0
    assert lib.fab_attention_fwd(ctypes.byref(a), None) == _native.FAB_ERR_UNSUPPORTED
    a.sm_scale = 0.125
    a.head_dim = 512
    assert lib.fab_attention_fwd(ctypes.byref(a), None) == _native.FAB_ERR_UNSUPPORTED
    a.head_dim = 64
    a.seqlen_q = 0
    assert lib.fab_attention_fwd(ctypes.byref(a), None) == _native.FAB_OK
    a.seqlen_q = 16
    a.o = 4100  # not 16-byte aligned
    assert lib.fab_attention_fwd(ctypes.byref(a), None) == _native.FAB_ERR_INVALID_ARG


def test_attention_plan_reports_the_launch_without_a_device():
    lib = _native.lib
    plan = _native.FabFaPlan()
    assert lib.fab_attention_fwd_plan(None, 0, ctypes.byref(plan)) == _native.FAB_ERR_INVALID_ARG
    a = _native.FabAttentionParams()
    a.batch, a.heads_q, a.heads_kv, a.seqlen_q, a.seqlen_k, a.head_dim, a.dtype = 4, 32, 32, 8192, 8192, 128, 1
    a.sm_scale = 128 ** -0.5
    a.q = a.k = a.v = a.o = 4096
    a.q_stride_s = a.k_stride_s = a.v_stride_s = a.o_stride_s = 128
    assert lib.fab_attention_fwd_plan(ctypes.byref(a), 5, ctypes.byref(plan)) == _native.FAB_ERR_INVALID_ARG
    assert lib.fab_attention_fwd_plan(ctypes.byref(a), 0, None) == _native.FAB_ERR_INVALID_ARG
    # The two-tile table needs no device query: 256 query rows per CTA, one CTA per SM.
    assert lib.fab_attention_fwd_plan(ctypes.byref(a), 0, ctypes.byref(plan)) == _native.FAB_OK
    assert (plan.config.q_tiles_per_cta, plan.config.block_n, plan.ctas, plan.ctas_per_sm) == (2, 128, 4 * 32 * 32, 1)
    a.seqlen_q = 0
    assert lib.fab_attention_fwd_plan(ctypes.byref(a), 0, ctypes.byref(plan)) == _native.FAB_OK
    assert plan.ctas == 0


def test_strided_entry_requires_unit_head_dim_stride():
    lib = _native.lib
    args = [4096, 4096, 4096, 4096, None]
    strides = [1024, 256, 64, 2] + [1024, 256, 64, 1] * 2 + [1024, 256, 64, 1] + [0, 0, 0]
    rc = lib.fab_flash_attn_fwd_basic(*args, *strides, 1, 4, 4, 4, 64, 0.125, 0, 0, 1, None)
    assert rc == _native.FAB_ERR_INVALID_ARG
    # HAS_LSE without an lse pointer
    strides[3] = 1
    rc = lib.fab_flash_attn_fwd_basic(*args, *strides, 1, 4, 4, 4, 64, 0.125, 0, 1, 1, None)
    assert rc == _native.FAB_ERR_INVALID_ARG


def _decode_params(B=1, Hq=28, Hkv=4, M=1, N=32768, D=128, dtype=_native.FAB_DTYPE_BF16):
    a = _native.FabAttentionParams()
    a.q = a.k = a.v = a.o = 4096  # never dereferenced by these calls
    a.q_stride_b, a.q_stride_h, a.q_stride_s = Hq * M * D, M * D, D
    a.k_stride_b, a.k_stride_h, a.k_stride_s = Hkv * N * D, N * D, D
    a.v_stride_b, a.v_stride_h, a.v_stride_s = Hkv * N * D, N * D, D
    a.o_stride_b, a.o_stride_h, a.o_stride_s = Hq * M * D, M * D, D
    a.batch, a.heads_q, a.heads_kv, a.seqlen_q, a.seqlen_k, a.head_dim, a.dtype = B, Hq, Hkv, M, N, D, dtype
    a.sm_scale = D ** -0.5
    return a


def _round256(x):
    return (x + 255) // 256 * 256


@pytest.mark.parametrize("splits, expect_used", [(8, 8), (1, 1), (1000, 256), (300, 256)])
def test_splitkv_workspace_size(splits, expect_used):
    """Workspace = fp32 partial O of every split and row, the partial LSEs, then one arrival counter per row
    group (4 key/value heads, whose 7 query heads share one 128-row tile), each 256-byte aligned; the split
    count is capped by the number of 128-key tiles."""
    lib = _native.lib
    a = _decode_params()
    need, used = ctypes.c_size_t(0), ctypes.c_int(0)
    assert lib.fab_attention_fwd_splitkv_workspace(ctypes.byref(a), splits, ctypes.byref(need), ctypes.byref(used)) == 0
    assert used.value == expect_used
    rows = 1 * 28 * 1
    groups = 4
    want = 0 if expect_used == 1 else (_round256(4 * expect_used * rows * 128) + _round256(4 * expect_used * rows)
                                       + _round256(4 * groups))
    assert need.value == want


def test_splitkv_rejects_bad_workspace_before_any_launch():
    lib = _native.lib
    a = _decode_params()
    need = ctypes.c_size_t(0)
    assert lib.fab_attention_fwd_splitkv_workspace(ctypes.byref(a), 8, ctypes.byref(need), None) == 0
    assert lib.fab_attention_fwd_splitkv(ctypes.byref(a), 8, None, need.value, None) == _native.FAB_ERR_WORKSPACE
    assert lib.fab_attention_fwd_splitkv(ctypes.byref(a), 8, 1 << 20, need.value - 1, None) == _native.FAB_ERR_WORKSPACE
    assert lib.fab_attention_fwd_splitkv(ctypes.byref(a), 8, (1 << 20) + 16, need.value, None) == _native.FAB_ERR_WORKSPACE
    assert lib.fab_attention_fwd_splitkv_workspace(None, 8, ctypes.byref(need), None) == _native.FAB_ERR_INVALID_ARG
    a.heads_kv = 3
    assert lib.fab_attention_fwd_splitkv(ctypes.byref(a), 8, 1 << 20, 1 << 30, None) == _native.FAB_ERR_INVALID_ARG
    a.heads_kv, a.seqlen_q = 4, 0  # nothing to compute: no workspace, no launch
    assert lib.fab_attention_fwd_splitkv_workspace(ctypes.byref(a), 8, ctypes.byref(need), None) == 0
    assert need.value == 0
    assert lib.fab_attention_fwd_splitkv(ctypes.byref(a), 8, None, 0, None) == _native.FAB_OK


def test_varlen_entry_validates_before_any_launch():
    lib = _native.lib
    assert lib.fab_attention_fwd_varlen(None, None) == _native.FAB_ERR_INVALID_ARG
    p = _native.FabAttentionVarlenParams()
    p.q = p.k = p.v = p.o = 4096
    p.batch, p.heads_q, p.heads_kv, p.total_q, p.total_k = 2, 4, 2, 10, 12
    p.max_seqlen_q, p.max_seqlen_k, p.head_dim, p.dtype, p.sm_scale = 6, 7, 64, _native.FAB_DTYPE_BF16, 0.125
    p.q_stride_t, p.q_stride_h = 4 * 64, 64
    p.k_stride_t, p.k_stride_h = 2 * 64, 64
    p.v_stride_t, p.v_stride_h = 2 * 64, 64
    p.o_stride_t, p.o_stride_h = 4 * 64, 64
    assert lib.fab_attention_fwd_varlen(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG  # no cu_seqlens
    p.cu_seqlens_q, p.cu_seqlens_k = 8192, 8194  # second one misaligned
    assert lib.fab_attention_fwd_varlen(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG
    p.cu_seqlens_k = 8200
    p.heads_kv = 3
    assert lib.fab_attention_fwd_varlen(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG
    p.heads_kv, p.total_q = 2, -1
    assert lib.fab_attention_fwd_varlen(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG
    p.total_q = 0  # nothing to compute
    assert lib.fab_attention_fwd_varlen(ctypes.byref(p), None) == _native.FAB_OK


def test_gemm_plan_validates_like_gemm():
    p = _native.FabGemmParams()
    p.a = p.b = p.c = 256
    p.lda, p.ldb, p.ldc = 64, 64, 64
    p.M, p.N, p.K = 64, 64, 64
    p.in_dtype = p.out_dtype = _native.dtype_code(torch.bfloat16)
    kernel, split, tile_n = ctypes.c_int(-1), ctypes.c_int(-1), ctypes.c_int(-1)
    p.M = -1
    assert _native.lib.fab_gemm_plan(ctypes.byref(p), ctypes.byref(kernel), ctypes.byref(split), ctypes.byref(tile_n)) == \
        _native.FAB_ERR_INVALID_ARG
    p.M = 0  # nothing to compute
    assert _native.lib.fab_gemm_plan(ctypes.byref(p), ctypes.byref(kernel), ctypes.byref(split), ctypes.byref(tile_n)) == _native.FAB_OK
    assert (kernel.value, split.value, tile_n.value) == (_native.FAB_GEMM_KERNEL_SINGLE, 1, 256)
    p.M, p.ldc = 64, 32  # ldc < N
    assert _native.lib.fab_gemm_plan(ctypes.byref(p), ctypes.byref(kernel), ctypes.byref(split), ctypes.byref(tile_n)) == \
        _native.FAB_ERR_INVALID_ARG
    assert _native.lib.fab_gemm_plan(ctypes.byref(p), None, ctypes.byref(split), ctypes.byref(tile_n)) == \
        _native.FAB_ERR_INVALID_ARG


@pytest.mark.parametrize("change, ok", [
    (dict(), True),
    (dict(head_dim=96), False),
    (dict(rope_cols=100), False),
    (dict(rope_cols=1024), False),
    (dict(out_dtype=2), False),
    (dict(round_f16=1), False),
    (dict(rope_cos=0), False),
    (dict(bias=8), False),
    (dict(N=640 + 64), False),
])
def test_bias_rope_epilogue_validation(change, ok):
    """Argument checks of FAB_GEMM_EPILOGUE_BIAS_ROPE; only the invalid ones are sent (no GPU here)."""
    if ok:
        return
    p = _native.FabGemmParams()
    p.a = p.b = p.c = 256
    p.M, p.N, p.K = 64, 640, 64
    p.lda, p.ldb, p.ldc = 64, 704, 704
    p.in_dtype = p.out_dtype = _native.dtype_code(torch.bfloat16)
    p.epilogue = _native.FAB_GEMM_EPILOGUE_BIAS_ROPE
    p.bias, p.rope_cos, p.rope_sin = 512, 768, 1024
    p.rope_cols, p.head_dim = 384, 128
    for k, v in change.items():
        setattr(p, k, v)
    assert _native.lib.fab_gemm(ctypes.byref(p), None) == _native.FAB_ERR_INVALID_ARG
