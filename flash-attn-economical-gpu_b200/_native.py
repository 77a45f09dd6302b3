"""ctypes binding of libfa_b200.so, the C ABI declared in include/fa_b200.h.

This module is the only place Python touches the native library.  It loads the
in-tree build next to this file and raises ImportError if it is missing: there
is no CPU or Triton fallback for any entry point.  Return codes are turned
into the Python exceptions the reference raises for the same conditions
(ValueError for bad shapes/arguments, RuntimeError for launch failures).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_NAME = "libfa_b200.so"
LIB_PATH = _HERE / LIB_NAME

FAB_OK = 0
FAB_ERR_INVALID_ARG = 1
FAB_ERR_UNSUPPORTED = 2
FAB_ERR_LAUNCH = 3
FAB_ERR_DEVICE_TIMEOUT = 4
FAB_ERR_CUDA = 5
FAB_ERR_WORKSPACE = 6

FAB_GEMM_EPILOGUE_STORE = 0
FAB_GEMM_EPILOGUE_SWIGLU = 1
FAB_GEMM_EPILOGUE_BIAS_ROPE = 2
FAB_GEMM_KERNEL_SINGLE = 0
FAB_GEMM_KERNEL_PAIR = 1
FAB_GEMM_KERNEL_SPLITK = 2
FAB_GEMM_KERNEL_PAIR_STREAMK = 3

FAB_DTYPE_F16 = 0
FAB_DTYPE_BF16 = 1
FAB_DTYPE_F32 = 2

FAB_FA_VARIANT_TWO_TILES = 0
FAB_FA_VARIANT_ONE_TILE = 1

FAB_KERNEL_ATTENTION = 0
FAB_KERNEL_MATMUL = 1
FAB_KERNEL_ATTENTION_ONE_TILE = 2

# Every symbol include/fa_b200.h declares, with its ctypes prototype.
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_vp = ctypes.c_void_p
_f32 = ctypes.c_float


class FabAttentionParams(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("o", _vp), ("lse", _vp),
        ("q_stride_b", _i64), ("q_stride_h", _i64), ("q_stride_s", _i64),
        ("k_stride_b", _i64), ("k_stride_h", _i64), ("k_stride_s", _i64),
        ("v_stride_b", _i64), ("v_stride_h", _i64), ("v_stride_s", _i64),
        ("o_stride_b", _i64), ("o_stride_h", _i64), ("o_stride_s", _i64),
        ("lse_stride_b", _i64), ("lse_stride_h", _i64), ("lse_stride_s", _i64),
        ("batch", _i32), ("heads_q", _i32), ("heads_kv", _i32),
        ("seqlen_q", _i32), ("seqlen_k", _i32), ("head_dim", _i32),
        ("dtype", _i32), ("sm_scale", _f32), ("causal", _i32),
    ]


class FabGemmParams(ctypes.Structure):
    _fields_ = [
        ("a", _vp), ("b", _vp), ("c", _vp),
        ("lda", _i64), ("ldb", _i64), ("ldc", _i64),
        ("M", _i32), ("N", _i32), ("K", _i32),
        ("in_dtype", _i32), ("out_dtype", _i32), ("round_f16", _i32), ("group_m", _i32), ("epilogue", _i32),
        ("bias", _vp), ("rope_cos", _vp), ("rope_sin", _vp), ("rope_cols", _i32), ("head_dim", _i32),
        ("row_scale", _vp), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class FabAttentionVarlenParams(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("o", _vp), ("lse", _vp),
        ("cu_seqlens_q", _vp), ("cu_seqlens_k", _vp),
        ("q_stride_t", _i64), ("q_stride_h", _i64),
        ("k_stride_t", _i64), ("k_stride_h", _i64),
        ("v_stride_t", _i64), ("v_stride_h", _i64),
        ("o_stride_t", _i64), ("o_stride_h", _i64),
        ("lse_stride_h", _i64), ("lse_stride_t", _i64),
        ("batch", _i32), ("heads_q", _i32), ("heads_kv", _i32), ("total_q", _i32), ("total_k", _i32),
        ("max_seqlen_q", _i32), ("max_seqlen_k", _i32), ("head_dim", _i32), ("dtype", _i32),
        ("sm_scale", _f32), ("causal", _i32),
    ]


MAX_TP_RANKS = 8


class FabGemmAllreduceParams(ctypes.Structure):
    _fields_ = [
        ("a", _vp), ("b", _vp),
        ("lda", _i64), ("ldb", _i64), ("ldo", _i64),
        ("M", _i32), ("N", _i32), ("K", _i32), ("in_dtype", _i32), ("world", _i32), ("rank", _i32),
        ("inbox", _vp * MAX_TP_RANKS), ("out", _vp * MAX_TP_RANKS), ("counters", _vp * MAX_TP_RANKS),
    ]


class FabFaConfig(ctypes.Structure):
    _fields_ = [
        ("head_dim_padded", _i32), ("q_tiles_per_cta", _i32), ("block_n", _i32), ("stages", _i32),
        ("threads", _i32), ("smem_bytes", _i32), ("tmem_columns", _i32), ("s_buffers", _i32),
    ]


class FabFaPlan(ctypes.Structure):
    _fields_ = [("config", FabFaConfig), ("ctas", ctypes.c_longlong), ("ctas_per_sm", _i32)]


class FabKernelAttrs(ctypes.Structure):
    _fields_ = [("registers_per_thread", _i32), ("shared_bytes", _i32), ("threads", _i32)]


class FabDeviceLimits(ctypes.Structure):
    _fields_ = [
        ("shared_bytes_per_sm", _i32), ("shared_bytes_per_block_optin", _i32), ("registers_per_sm", _i32),
        ("warp_size", _i32), ("max_threads_per_block", _i32), ("multiprocessor_count", _i32),
        ("cc_major", _i32), ("cc_minor", _i32),
    ]


_STRIDED_FA_ARGS = [_vp] * 4 + [ctypes.POINTER(_f32)] + [_i64] * 19 + [_i32] * 5 + [_f32] + [_i32] * 3 + [_vp]

PROTOTYPES = {
    "fab_flash_attn_fwd_basic": (_i32, _STRIDED_FA_ARGS),
    "fab_flash_attn_fwd_optimize_shared_mem": (_i32, _STRIDED_FA_ARGS),
    "fab_flash_attn_fwd_block_d_nomask_contiguous": (_i32, [_vp] * 4 + [_i32] * 5 + [_f32, _i32, _vp]),
    "fab_attention_fwd": (_i32, [ctypes.POINTER(FabAttentionParams), _vp]),
    "fab_attention_fwd_varlen": (_i32, [ctypes.POINTER(FabAttentionVarlenParams), _vp]),
    "fab_attention_fwd_variant": (_i32, [ctypes.POINTER(FabAttentionParams), _i32, _vp]),
    "fab_flash_attn_config_variant": (_i32, [_i32, _i32, _i32, ctypes.POINTER(FabFaConfig)]),
    "fab_attention_fwd_plan": (_i32, [ctypes.POINTER(FabAttentionParams), _i32, ctypes.POINTER(FabFaPlan)]),
    "fab_debug_set_wait_limit_ns": (_i32, [ctypes.c_ulonglong]),
    "fab_debug_starve_kv_load": (_i32, [_i32]),
    "fab_attention_fwd_splitkv_workspace": (
        _i32, [ctypes.POINTER(FabAttentionParams), _i32, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(_i32)]),
    "fab_attention_fwd_splitkv": (_i32, [ctypes.POINTER(FabAttentionParams), _i32, _vp, ctypes.c_size_t, _vp]),
    "fab_attention_fwd_splitkv_static": (_i32, [ctypes.POINTER(FabAttentionParams), _i32, _vp]),
    "fab_matmul_contiguous": (_i32, [_vp] * 3 + [_i32] * 6 + [_vp]),
    "fab_gemm": (_i32, [ctypes.POINTER(FabGemmParams), _vp]),
    "fab_gemm_plan": (_i32, [ctypes.POINTER(FabGemmParams), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                             ctypes.POINTER(_i32)]),
    "fab_gemm_workspace_size": (_i32, [ctypes.POINTER(FabGemmParams), ctypes.POINTER(ctypes.c_size_t)]),
    "fab_gemm_grid": (_i32, [ctypes.POINTER(FabGemmParams), ctypes.POINTER(ctypes.c_longlong)]),
    "fab_gemm_allreduce_layout": (_i32, [_i32, _i32, _i32, ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_size_t),
                                         ctypes.POINTER(ctypes.c_size_t)]),
    "fab_gemm_allreduce": (_i32, [ctypes.POINTER(FabGemmAllreduceParams), _vp]),
    "fab_ipc_export": (_i32, [_vp, _vp, ctypes.POINTER(ctypes.c_size_t)]),
    "fab_ipc_import": (_i32, [_vp, ctypes.c_size_t, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "fab_ipc_close": (_i32, [_vp]),
    "fab_rmsnorm": (_i32, [_vp] * 5 + [_i32, _i32] + [_i64] * 4 + [_f32, _i32, _vp]),
    "fab_rmsnorm_rstd": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i64, _i64, _i64, _f32, _i32, _vp]),
    "fab_bias_rope": (_i32, [_vp] * 4 + [_i32] * 4 + [_i64, _i32, _vp]),
    "fab_silu_mul": (_i32, [_vp, _vp, _i32, _i32, _i64, _i64, _i32, _i32, _vp]),
    "fab_flash_attn_config": (_i32, [_i32, _i32, ctypes.POINTER(FabFaConfig)]),
    "fab_kernel_attrs_query": (_i32, [_i32, _i32, _i32, ctypes.POINTER(FabKernelAttrs)]),
    "fab_device_limits_query": (_i32, [_i32, ctypes.POINTER(FabDeviceLimits)]),
    "fab_get_device_error": (_i32, [ctypes.POINTER(_i32)]),
    "fab_error_string": (ctypes.c_char_p, [_i32]),
    "fab_abi_version": (_i32, []),
}

ABI_VERSION = 8


def _load() -> ctypes.CDLL:
    path = os.environ.get("FAB_LIBRARY", str(LIB_PATH))
    if not Path(path).is_file():
        raise ImportError(
            f"{LIB_NAME} not found at {path}; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(there is no fallback implementation)"
        )
    lib = ctypes.CDLL(path)
    for name, (restype, argtypes) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.fab_abi_version() != ABI_VERSION:
        raise ImportError(f"{path} has ABI version {lib.fab_abi_version()}, expected {ABI_VERSION}")
    return lib


lib = _load()


class DeviceTimeoutError(RuntimeError):
    """A kernel gave up on one of its bounded waits (see fab_get_device_error)."""


def error_string(rc: int) -> str:
    return lib.fab_error_string(int(rc)).decode()


def check(rc: int, what: str) -> None:
    """Raise the Python exception matching a FAB_* return code."""
    if rc == FAB_OK:
        return
    msg = f"{what}: {error_string(rc)} (code {rc})"
    if rc in (FAB_ERR_INVALID_ARG, FAB_ERR_UNSUPPORTED, FAB_ERR_WORKSPACE):
        raise ValueError(msg)
    if rc == FAB_ERR_DEVICE_TIMEOUT:
        raise DeviceTimeoutError(msg)
    raise RuntimeError(msg)


def device_error() -> int:
    """Read and clear the device error word of the current CUDA device."""
    code = _i32(0)
    check(lib.fab_get_device_error(ctypes.byref(code)), "fab_get_device_error")
    return int(code.value)


# What each device error code's wait was waiting for (fab_get_device_error, include/fa_b200.h).
DEVICE_WAITS = {1: "a Q tile's load", 2: "a K/V tile's load", 3: "an S product", 4: "a softmax's P",
                5: "O's last product", 6: "a free K/V or stage slot", 7: "a GEMM accumulator",
                8: "the drain at teardown", 9: "a peer rank's partial tile", 10: "a peer owner's reduced tile",
                11: "a stream-K piece from another CTA pair", 12: "the CTA-pair GEMM's next tile from its scheduler",
                13: "the split-KV merge's copies"}


def raise_on_device_error() -> None:
    code = device_error()
    if code:
        what = DEVICE_WAITS.get(code, "unknown wait")
        raise DeviceTimeoutError(f"a kernel gave up on a bounded wait (device error code {code}: {what})")


def dtype_code(dtype) -> int:
    import torch

    if dtype == torch.float16:
        return FAB_DTYPE_F16
    if dtype == torch.bfloat16:
        return FAB_DTYPE_BF16
    if dtype == torch.float32:
        return FAB_DTYPE_F32
    raise ValueError(f"unsupported dtype {dtype}; expected float16, bfloat16 or float32")


def fa_config(dtype: int, head_dim: int) -> FabFaConfig | None:
    cfg = FabFaConfig()
    rc = lib.fab_flash_attn_config(int(dtype), int(head_dim), ctypes.byref(cfg))
    if rc == FAB_ERR_UNSUPPORTED:
        return None
    check(rc, "fab_flash_attn_config")
    return cfg


def fa_config_variant(dtype: int, head_dim: int, variant: int) -> FabFaConfig | None:
    """Tile of one of the two compiled families (FAB_FA_VARIANT_*), or None when head_dim is out of range."""
    cfg = FabFaConfig()
    rc = lib.fab_flash_attn_config_variant(int(dtype), int(head_dim), int(variant), ctypes.byref(cfg))
    if rc == FAB_ERR_UNSUPPORTED:
        return None
    check(rc, "fab_flash_attn_config_variant")
    return cfg


def set_wait_limit_ns(ns: int) -> None:
    """Time limit of one bounded wait in the attention kernels of the current device (0: the 2 s default)."""
    check(lib.fab_debug_set_wait_limit_ns(int(ns)), "fab_debug_set_wait_limit_ns")


def starve_kv_load(ring_tile: int) -> None:
    """Test hook: every attention CTA skips K/V ring load `ring_tile` (-1: none), so its wait runs out."""
    check(lib.fab_debug_starve_kv_load(int(ring_tile)), "fab_debug_starve_kv_load")


def kernel_attrs(which: int, dtype: int, head_dim: int = 0) -> FabKernelAttrs:
    out = FabKernelAttrs()
    check(lib.fab_kernel_attrs_query(int(which), int(dtype), int(head_dim), ctypes.byref(out)), "fab_kernel_attrs_query")
    return out


def device_limits(device: int) -> FabDeviceLimits:
    out = FabDeviceLimits()
    check(lib.fab_device_limits_query(int(device), ctypes.byref(out)), "fab_device_limits_query")
    return out


def current_stream_handle(device) -> int:
    import torch

    return int(torch.cuda.current_stream(device).cuda_stream)
