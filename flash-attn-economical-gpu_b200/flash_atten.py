"""FlashAttention forward on B200 (drop-in for the reference's flash_atten.py).

`flash_attention(launch_spec)` and `flash_attention_kernel_mapping` keep the
reference's contract (flash_atten.py:364-383): the spec's `function_name`
selects a kernel, the kernel is launched as `kernel[grid](*kernel_args,
**kernel_kwargs)`, and the call returns `kernel_args[3]` (o), or `(o, lse)`
when `kernel_args[4]` is a tensor.  The three kernel names map to launcher
objects that accept exactly the Triton kernels' argument lists
(flash_atten.py:14-51, 136-173, 261-276) and call the sm_100a tcgen05 kernel
through the C ABI (include/fa_b200.h).  There is no Triton and no CPU path:
the native library must be loaded and the tensors must live on a CUDA device.

`attention_forward` is the direct entry used by the SDPA drop-in and the
benchmarks: same maths, plus grouped-query heads mapped inside the kernel.
"""
from __future__ import annotations

import ctypes
import logging
from dataclasses import dataclass

import torch

import _native
import tune_table
from tuner import FlashAttentionLaunchSpec

logger = logging.getLogger(__name__)


def _require_cuda_tensor(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU implementation)")


def _tma_ready(t: torch.Tensor, strides: tuple[int, ...]) -> bool:
    """Unit stride on the last dim, 16-byte aligned base and outer strides."""
    es = t.element_size()
    if strides[-1] != 1:
        return False
    if t.data_ptr() % 16:
        return False
    return all((s * es) % 16 == 0 for s, n in zip(strides[:-1], t.shape[:-1]) if n > 1)


def _padded_like(t: torch.Tensor) -> torch.Tensor:
    """Uninitialised tensor shaped like `t` whose rows start on 16-byte boundaries."""
    per16 = 16 // t.element_size()
    d = t.shape[-1]
    dp = -(-d // per16) * per16
    return torch.empty((*t.shape[:-1], dp), device=t.device, dtype=t.dtype)[..., :d]


def _as_view(t: torch.Tensor, shape: tuple[int, ...], strides: tuple[int, ...]) -> torch.Tensor:
    """The tensor the reference kernel reads: `t`'s storage seen through explicit strides."""
    if tuple(t.shape) == tuple(shape) and tuple(t.stride()) == tuple(strides):
        return t
    return torch.as_strided(t, shape, strides, t.storage_offset())


def _conform(t: torch.Tensor) -> torch.Tensor:
    """A TMA-readable version of `t` (a row-padded copy only when needed)."""
    if _tma_ready(t, tuple(t.stride())):
        return t
    buf = _padded_like(t)
    buf.copy_(t)
    return buf


@dataclass
class _KernelMetadata:
    shared: int
    num_warps: int
    tmem_columns: int


class _CompiledKernelInfo:
    """What `warmup` returns: the facts the reference's tuner reads (tuner.py:355-368)."""

    def __init__(self, attrs: _native.FabKernelAttrs, tmem_columns: int = 0):
        self.n_regs = int(attrs.registers_per_thread)
        self.metadata = _KernelMetadata(int(attrs.shared_bytes), int(attrs.threads) // 32, tmem_columns)

    def _init_handles(self) -> None:
        return None


def _launch_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    lse: torch.Tensor | None,
    *,
    causal: bool,
    sm_scale: float,
    what: str,
    entry: str = "general",
    num_splits: int = 0,
    workspace: torch.Tensor | None = None,
    variant: int = 0,
) -> None:
    """Validate, conform and launch one attention forward through the C ABI.

    `entry` picks the C entry point: "basic" / "optimize_shared_mem" /
    "nomask" for the reference-named kernels, "splitkv"
    (`fab_attention_fwd_splitkv`, key splits merged by the last split CTA of
    each row group; `num_splits` 0 = as many splits as keep the grid in one wave) or "general"
    (`fab_attention_fwd`, grouped-query heads) otherwise.  `workspace` (uint8,
    CUDA, zero-filled before its first use; calls leave it zeroed) is used for
    the split partials when it is large enough, else a zeroed one is allocated.
    `variant` 1 runs the one-query-tile family (`fab_attention_fwd_variant`)
    instead of the default table, whatever `entry` names.

    q/o: [B, Hq, M, D]; k/v: [B, Hkv, N, D]; lse: [B, Hq, M] fp32 or None.
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        _require_cuda_tensor(name, t)
    if q.dtype != k.dtype or q.dtype != v.dtype or q.dtype != o.dtype:
        raise ValueError(f"{what}: q, k, v and o must share one dtype, got {q.dtype}, {k.dtype}, {v.dtype}, {o.dtype}")
    dt = _native.dtype_code(q.dtype)
    B, Hq, M, D = q.shape
    Bk, Hkv, N, Dk = k.shape
    if tuple(v.shape) != tuple(k.shape) or Bk != B or Dk != D or tuple(o.shape) != tuple(q.shape):
        raise ValueError(f"{what}: inconsistent shapes q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)} o={tuple(o.shape)}")
    if Hkv == 0 or Hq % Hkv:
        raise ValueError(f"{what}: query heads ({Hq}) must be a multiple of key/value heads ({Hkv})")
    if lse is not None:
        _require_cuda_tensor("lse", lse)
        if lse.dtype != torch.float32 or tuple(lse.shape) != (B, Hq, M):
            raise ValueError(f"{what}: lse must be float32 with shape {(B, Hq, M)}")
    if B * Hq * M == 0:
        return
    sm_scale = float(sm_scale)
    if sm_scale < 0:
        # softmax(s * c) == softmax(|c| * (-q) k^T): fold the sign into Q.
        q = -q
        sm_scale = -sm_scale
    elif sm_scale == 0:
        # Uniform weights over the visible keys; a vanishing positive scale gives the same weights.
        sm_scale = 1e-30
    qc, kc, vc = _conform(q), _conform(k), _conform(v)
    oc = o if _tma_ready(o, tuple(o.stride())) else _padded_like(o)
    lc = lse
    if lse is not None and lse.data_ptr() % 4:
        lc = torch.empty_like(lse, memory_format=torch.contiguous_format)
    with torch.cuda.device(q.device):
        stream = ctypes.c_void_p(_native.current_stream_handle(q.device))
        if variant == 0 and entry == "nomask" and all(t.is_contiguous() for t in (qc, kc, vc, oc)):
            rc = _native.lib.fab_flash_attn_fwd_block_d_nomask_contiguous(
                qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), oc.data_ptr(), B, Hq, M, N, D, sm_scale, dt, stream
            )
        elif variant == 0 and entry in ("basic", "optimize_shared_mem") and Hq == Hkv:
            fn = (
                _native.lib.fab_flash_attn_fwd_basic
                if entry == "basic"
                else _native.lib.fab_flash_attn_fwd_optimize_shared_mem
            )
            lse_ptr = ctypes.cast(ctypes.c_void_p(lc.data_ptr()), ctypes.POINTER(ctypes.c_float)) if lc is not None else None
            rc = fn(
                qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), oc.data_ptr(), lse_ptr,
                *qc.stride(), *kc.stride(), *vc.stride(), *oc.stride(),
                *(lc.stride() if lc is not None else (0, 0, 0)),
                B, Hq, M, N, D, sm_scale, 1 if causal else 0, 1 if lc is not None else 0, dt, stream,
            )
        else:
            p = _native.FabAttentionParams()
            p.q, p.k, p.v, p.o = qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), oc.data_ptr()
            p.lse = lc.data_ptr() if lc is not None else None
            p.q_stride_b, p.q_stride_h, p.q_stride_s = qc.stride()[:3]
            p.k_stride_b, p.k_stride_h, p.k_stride_s = kc.stride()[:3]
            p.v_stride_b, p.v_stride_h, p.v_stride_s = vc.stride()[:3]
            p.o_stride_b, p.o_stride_h, p.o_stride_s = oc.stride()[:3]
            if lc is not None:
                p.lse_stride_b, p.lse_stride_h, p.lse_stride_s = lc.stride()
            p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim = B, Hq, Hkv, M, N, D
            p.dtype = dt
            p.sm_scale = sm_scale
            p.causal = 1 if causal else 0
            if variant != 0:
                rc = _native.lib.fab_attention_fwd_variant(ctypes.byref(p), int(variant), stream)
            elif entry == "splitkv":
                need = ctypes.c_size_t(0)
                _native.check(_native.lib.fab_attention_fwd_splitkv_workspace(
                    ctypes.byref(p), int(num_splits), ctypes.byref(need), None), what)
                ws = workspace
                if need.value and (ws is None or ws.numel() < need.value or ws.data_ptr() % 256):
                    ws = torch.zeros(need.value, device=q.device, dtype=torch.uint8)
                rc = _native.lib.fab_attention_fwd_splitkv(
                    ctypes.byref(p), int(num_splits), ws.data_ptr() if need.value else None, need.value, stream)
            else:
                rc = _native.lib.fab_attention_fwd(ctypes.byref(p), stream)
    _native.check(rc, what)
    if oc is not o:
        o.copy_(oc)
    if lc is not None and lc is not lse:
        lse.copy_(lc)


def _compiled_info(q: torch.Tensor, D: int, variant: int) -> _CompiledKernelInfo:
    """Resource facts of the compiled kernel a launch with this dtype, head dim and tile family runs."""
    dt = _native.dtype_code(q.dtype)
    which = _native.FAB_KERNEL_ATTENTION_ONE_TILE if variant else _native.FAB_KERNEL_ATTENTION
    return _CompiledKernelInfo(_native.kernel_attrs(which, dt, D),
                               int(_native.fa_config_variant(dt, D, variant).tmem_columns))


class _StridedAttentionKernel:
    """Stands in for `_flash_attn_fwd_kernel_basic` / `_optimize_shared_mem` (Triton JITFunctions).

    Positional arguments (flash_atten.py:15-44): q, k, v, o, lse (tensor or 0),
    19 element strides, H, M, N, D, sm_scale.  Keyword arguments: causal,
    HAS_LSE and the Triton tiling knobs (BLOCK_*, num_warps, num_stages,
    debug), which the sm_100a kernel does not need and ignores, plus
    `sm100_variant` (0 or 1, the tile family a measured tuning chose).  The
    batch size is grid[1] // H, as in the Triton launch.
    """

    def __init__(self, name: str):
        self.__name__ = name
        self.fn_name = name

    def __repr__(self) -> str:
        return f"<sm_100a attention kernel {self.__name__}>"

    def __getitem__(self, grid):
        grid = tuple(grid) if isinstance(grid, (tuple, list)) else (grid,)

        def launch(*args, **kwargs):
            return self._run(grid, args, kwargs)

        return launch

    def _parse(self, grid, args, kwargs):
        if len(args) != 29:
            raise TypeError(f"{self.__name__} expects 29 positional arguments, got {len(args)}")
        q, k, v, o, lse = args[:5]
        strides = [int(s) for s in args[5:24]]
        H, M, N, D = (int(x) for x in args[24:28])
        sm_scale = float(args[28])
        causal = bool(kwargs.get("causal", False))
        has_lse = bool(kwargs.get("HAS_LSE", False))
        if H <= 0:
            raise ValueError(f"{self.__name__}: H must be positive")
        if len(grid) < 2 or int(grid[1]) % H:
            raise ValueError(f"{self.__name__}: grid[1] must be batch*H, got grid={grid} with H={H}")
        B = int(grid[1]) // H
        return q, k, v, o, lse, strides, B, H, M, N, D, sm_scale, causal, has_lse

    def _run(self, grid, args, kwargs):
        q, k, v, o, lse, st, B, H, M, N, D, sm_scale, causal, has_lse = self._parse(grid, args, kwargs)
        qv = _as_view(q, (B, H, M, D), tuple(st[0:4]))
        kv = _as_view(k, (B, H, N, D), tuple(st[4:8]))
        vv = _as_view(v, (B, H, N, D), tuple(st[8:12]))
        ov = _as_view(o, (B, H, M, D), tuple(st[12:16]))
        lv = None
        if has_lse:
            if not isinstance(lse, torch.Tensor):
                raise ValueError(f"{self.__name__}: HAS_LSE=True needs an lse tensor")
            lv = _as_view(lse, (B, H, M), tuple(st[16:19]))
        entry = "basic" if self.__name__.endswith("_basic") else "optimize_shared_mem"
        _launch_attention(qv, kv, vv, ov, lv, causal=causal, sm_scale=sm_scale, what=self.__name__, entry=entry,
                          variant=int(kwargs.get("sm100_variant", 0)))

    def warmup(self, *args, grid, **kwargs):
        return _compiled_info(args[0], int(args[27]), int(kwargs.get("sm100_variant", 0)))


class _ContiguousAttentionKernel(_StridedAttentionKernel):
    """Stands in for `_flash_attn_fwd_kernel_block_d_nomask_contiguous` (flash_atten.py:261-276).

    Positional arguments: q, k, v, o, H, M, N, D, sm_scale over contiguous
    [B, H, M|N, D] storage; non-causal, no LSE.  Unlike the Triton kernel,
    M, N and D need not be multiples of any tile size.
    """

    def _run(self, grid, args, kwargs):
        if len(args) != 9:
            raise TypeError(f"{self.__name__} expects 9 positional arguments, got {len(args)}")
        q, k, v, o = args[:4]
        H, M, N, D = (int(x) for x in args[4:8])
        sm_scale = float(args[8])
        if H <= 0 or len(grid) < 2 or int(grid[1]) % H:
            raise ValueError(f"{self.__name__}: grid[1] must be batch*H, got grid={grid} with H={H}")
        B = int(grid[1]) // H

        def contiguous_view(t, S):
            return _as_view(t, (B, H, S, D), (H * S * D, S * D, D, 1))

        _launch_attention(
            contiguous_view(q, M),
            contiguous_view(k, N),
            contiguous_view(v, N),
            contiguous_view(o, M),
            None,
            causal=False,
            sm_scale=sm_scale,
            what=self.__name__,
            entry="nomask",
            variant=int(kwargs.get("sm100_variant", 0)),
        )

    def warmup(self, *args, grid, **kwargs):
        return _compiled_info(args[0], int(args[7]), int(kwargs.get("sm100_variant", 0)))


_flash_attn_fwd_kernel_basic = _StridedAttentionKernel("_flash_attn_fwd_kernel_basic")
_flash_attn_fwd_kernel_optimize_shared_mem = _StridedAttentionKernel("_flash_attn_fwd_kernel_optimize_shared_mem")
_flash_attn_fwd_kernel_block_d_nomask_contiguous = _ContiguousAttentionKernel(
    "_flash_attn_fwd_kernel_block_d_nomask_contiguous"
)

flash_attention_kernel_mapping = {
    "_flash_attn_fwd_kernel_basic": _flash_attn_fwd_kernel_basic,
    "_flash_attn_fwd_kernel_optimize_shared_mem": _flash_attn_fwd_kernel_optimize_shared_mem,
    "_flash_attn_fwd_kernel_block_d_nomask_contiguous": _flash_attn_fwd_kernel_block_d_nomask_contiguous,
}


def flash_attention(
    launch_spec: FlashAttentionLaunchSpec,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """Launch the kernel a launch spec names; return o, or (o, lse) when the spec carries an lse buffer."""
    if launch_spec.function_name in flash_attention_kernel_mapping:
        flash_attention_kernel_mapping[launch_spec.function_name][launch_spec.grid](
            *launch_spec.kernel_args, **launch_spec.kernel_kwargs
        )
    else:
        raise NameError(f"No such kernel named {launch_spec.function_name}.")
    o = launch_spec.kernel_args[3]
    lse = launch_spec.kernel_args[4] if isinstance(launch_spec.kernel_args[4], torch.Tensor) else None
    return (o, lse) if lse is not None else o


def attention_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = False,
    sm_scale: float | None = None,
    return_lse: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """softmax(sm_scale * q k^T [causal]) v for q [B, Hq, M, D], k/v [B, Hkv, N, D].

    Query head h attends to key/value head h // (Hq // Hkv) (grouped-query
    attention without copying K/V).  Causal masking is top-left aligned, as in
    the reference (key n visible to query m iff m >= n) and torch SDPA.
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("attention_forward expects q, k, v with shape [batch, heads, seq, head_dim]")
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    o = out if out is not None else torch.empty(q.shape, device=q.device, dtype=q.dtype)
    lse = torch.empty(q.shape[:3], device=q.device, dtype=torch.float32) if return_lse else None
    variant = 0
    if q.dtype in (torch.float16, torch.bfloat16, torch.float32) and q.numel() and k.shape[2]:
        # the tile family the shipped measurements favour for this shape
        variant = tune_table.measured_variant(_native.dtype_code(q.dtype), q.shape[-1], causal,
                                              q.shape[0] * q.shape[1], q.shape[2], k.shape[2])
    _launch_attention(q, k, v, o, lse, causal=causal, sm_scale=sm_scale, what="attention_forward", variant=variant)
    return (o, lse) if return_lse else o


def attention_plan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = False,
                   variant: int | None = None) -> dict:
    """The kernel `attention_forward` (variant None: the measured tile family it picks) or the given tile
    family would launch for these tensors, without launching it: tile, grid size and CTAs per SM."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda_tensor(name, t)
    dt = _native.dtype_code(q.dtype)
    B, Hq, M, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    if variant is None:
        variant = 0
        if q.numel() and N:
            variant = tune_table.measured_variant(dt, D, causal, B * Hq, M, N)
    qc, kc, vc = _conform(q), _conform(k), _conform(v)
    o = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    p = _native.FabAttentionParams()
    p.q, p.k, p.v, p.o = qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr()
    p.q_stride_b, p.q_stride_h, p.q_stride_s = qc.stride()[:3]
    p.k_stride_b, p.k_stride_h, p.k_stride_s = kc.stride()[:3]
    p.v_stride_b, p.v_stride_h, p.v_stride_s = vc.stride()[:3]
    p.o_stride_b, p.o_stride_h, p.o_stride_s = o.stride()[:3]
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim = B, Hq, Hkv, M, N, D
    p.dtype, p.sm_scale, p.causal = dt, D ** -0.5, 1 if causal else 0
    plan = _native.FabFaPlan()
    with torch.cuda.device(q.device):
        _native.check(_native.lib.fab_attention_fwd_plan(ctypes.byref(p), int(variant), ctypes.byref(plan)),
                      "attention_plan")
    c = plan.config
    return {"variant": int(variant), "q_tiles_per_cta": c.q_tiles_per_cta, "block_n": c.block_n,
            "stages": c.stages, "s_buffers": c.s_buffers, "threads": c.threads, "smem_bytes": c.smem_bytes,
            "ctas": int(plan.ctas), "ctas_per_sm": plan.ctas_per_sm}


def attention_forward_splitkv(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = False,
    sm_scale: float | None = None,
    return_lse: bool = False,
    out: torch.Tensor | None = None,
    num_splits: int = 0,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """attention_forward with the keys cut into `num_splits` ranges (flash-decoding).

    For short query blocks (decode steps, speculative blocks) against long
    key ranges: each range is attended to by its own CTAs, and the last CTA of
    each row group to finish merges the ranges by their LSE.  `num_splits` 0
    gives as many splits as keep the grid in one wave (at most one CTA per
    SM).  A caller-supplied `workspace` must be zero-filled before its first
    use (every call leaves its counters at zero again).
    Query heads that share a key/value head are packed into one query tile
    when q is laid out [batch, head, seq, dim] contiguously (or seq == 1).
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("attention_forward_splitkv expects q, k, v with shape [batch, heads, seq, head_dim]")
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    o = out if out is not None else torch.empty(q.shape, device=q.device, dtype=q.dtype)
    lse = torch.empty(q.shape[:3], device=q.device, dtype=torch.float32) if return_lse else None
    _launch_attention(q, k, v, o, lse, causal=causal, sm_scale=sm_scale, what="attention_forward_splitkv",
                      entry="splitkv", num_splits=num_splits, workspace=workspace)
    return (o, lse) if return_lse else o


def attention_forward_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    max_seqlen_q: int,
    max_seqlen_k: int,
    *,
    causal: bool = False,
    sm_scale: float | None = None,
    return_lse: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """Attention over a packed batch of variable-length sequences.

    q: [total_q, Hq, D], k/v: [total_k, Hkv, D]; sequence b owns query rows
    cu_seqlens_q[b]:cu_seqlens_q[b+1] and key rows cu_seqlens_k[b]:cu_seqlens_k[b+1]
    (int32 CUDA tensors of batch + 1 offsets).  Returns o like q and, with
    return_lse, lse [Hq, total_q] in fp32.  Causal masking is top-left inside
    each sequence, as the reference's kernels mask a dense block.
    """
    what = "attention_forward_varlen"
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError(f"{what} expects q, k, v with shape [total_tokens, heads, head_dim]")
    for name, t in (("q", q), ("k", k), ("v", v), ("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        _require_cuda_tensor(name, t)
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(f"{what}: q, k and v must share one dtype")
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
        raise ValueError(f"{what}: cu_seqlens_q / cu_seqlens_k must be int32")
    if cu_seqlens_q.ndim != 1 or cu_seqlens_q.shape != cu_seqlens_k.shape or cu_seqlens_q.numel() < 1:
        raise ValueError(f"{what}: cu_seqlens_q and cu_seqlens_k must both have batch + 1 entries")
    total_q, Hq, D = q.shape
    total_k, Hkv, Dk = k.shape
    if tuple(v.shape) != tuple(k.shape) or Dk != D:
        raise ValueError(f"{what}: inconsistent shapes q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    if Hkv == 0 or Hq % Hkv:
        raise ValueError(f"{what}: query heads ({Hq}) must be a multiple of key/value heads ({Hkv})")
    if sm_scale is None:
        sm_scale = D ** -0.5
    o = out if out is not None else torch.empty(q.shape, device=q.device, dtype=q.dtype)
    if tuple(o.shape) != tuple(q.shape) or o.dtype != q.dtype:
        raise ValueError(f"{what}: out must match q's shape and dtype")
    lse = torch.empty(Hq, total_q, device=q.device, dtype=torch.float32) if return_lse else None
    batch = cu_seqlens_q.numel() - 1
    if batch == 0 or total_q == 0:
        return (o, lse) if return_lse else o
    sm_scale = float(sm_scale)
    if sm_scale < 0:
        q, sm_scale = -q, -sm_scale
    elif sm_scale == 0:
        sm_scale = 1e-30
    dt = _native.dtype_code(q.dtype)
    # [total, heads, D] viewed as [1, total, heads, D] -> conform as [1, heads, total, D] views.
    qc, kc, vc = (_conform(t.unsqueeze(0).transpose(1, 2)).transpose(1, 2).squeeze(0) for t in (q, k, v))
    o4 = o.unsqueeze(0).transpose(1, 2)
    oc = o if _tma_ready(o4, tuple(o4.stride())) else _padded_like(o4).transpose(1, 2).squeeze(0)
    cq, ck = cu_seqlens_q.contiguous(), cu_seqlens_k.contiguous()
    p = _native.FabAttentionVarlenParams()
    p.q, p.k, p.v, p.o = qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), oc.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.cu_seqlens_q, p.cu_seqlens_k = cq.data_ptr(), ck.data_ptr()
    p.q_stride_t, p.q_stride_h = qc.stride()[:2]
    p.k_stride_t, p.k_stride_h = kc.stride()[:2]
    p.v_stride_t, p.v_stride_h = vc.stride()[:2]
    p.o_stride_t, p.o_stride_h = oc.stride()[:2]
    if lse is not None:
        p.lse_stride_h, p.lse_stride_t = lse.stride()
    p.batch, p.heads_q, p.heads_kv = batch, Hq, Hkv
    p.total_q, p.total_k = total_q, total_k
    p.max_seqlen_q, p.max_seqlen_k = int(max_seqlen_q), int(max_seqlen_k)
    p.head_dim, p.dtype, p.sm_scale, p.causal = D, dt, sm_scale, 1 if causal else 0
    with torch.cuda.device(q.device):
        stream = ctypes.c_void_p(_native.current_stream_handle(q.device))
        rc = _native.lib.fab_attention_fwd_varlen(ctypes.byref(p), stream)
    _native.check(rc, what)
    if oc is not o:
        o.copy_(oc)
    return (o, lse) if return_lse else o


def _host_pieces(batch: int, kv_heads: int, chunks: int) -> list[tuple[int, int, int]]:
    """How attention_forward_host cuts a call: (batch entry, first kv head, end kv head) per piece.

    Every batch entry is split into the same number of runs of whole key/value-head groups (as many as make about
    `chunks` pieces in all, at most one per head), in order; together the pieces cover each unit exactly once."""
    per_b = max(1, min(kv_heads, -(-max(1, chunks) // batch)))
    pieces = []
    for b in range(batch):
        for i in range(per_b):
            h0, h1 = kv_heads * i // per_b, kv_heads * (i + 1) // per_b
            if h1 > h0:
                pieces.append((b, h0, h1))
    return pieces


def attention_forward_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = False,
    sm_scale: float | None = None,
    out: torch.Tensor | None = None,
    device=None,
    chunks: int = 16,
) -> torch.Tensor:
    """attention_forward for host tensors: q [B, Hq, M, D], k/v [B, Hkv, N, D] in CPU memory (pinned for overlap).

    Returns O in host memory (`out`, or a new pinned tensor) once it has landed there.  The call is cut into up
    to `chunks` pieces of whole (batch entry, key/value-head group) units and pipelined over three streams of
    `device` (default: the current device): piece c+1 is copied in while piece c is computed and piece c-1 is
    copied out, so both directions of the host link are busy at once and the kernel time hides behind the
    copies.  Each piece is the same kernel call as attention_forward on its units, which are independent, so
    the result equals attention_forward's bit for bit.  No counterpart in the reference (its kernels take
    device tensors).
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
            raise ValueError(f"attention_forward_host: {name} must be a CPU tensor")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("attention_forward_host expects q, k, v with shape [batch, heads, seq, head_dim]")
    B, Hq, M, D = q.shape
    Hkv = k.shape[1]
    if Hkv <= 0 or Hq % Hkv or k.shape[0] != B or v.shape != k.shape:
        raise ValueError("attention_forward_host: k and v must be [batch, kv_heads, seq, head_dim] with kv_heads "
                         "dividing q's heads")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=torch.cuda.is_available())
    elif out.device.type != "cpu" or out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("attention_forward_host: out must be a CPU tensor shaped and typed like q")
    if q.numel() == 0:
        return out
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    g = Hq // Hkv
    pieces = _host_pieces(B, Hkv, chunks)
    widest = max(h1 - h0 for _, h0, h1 in pieces)
    with torch.cuda.device(dev):
        compute = torch.cuda.current_stream(dev)
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        # Two device slots per operand, each as wide as the widest piece.
        slots = [tuple(torch.empty((1, widest * hs, t.shape[2], D), device=dev, dtype=t.dtype)
                       for t, hs in ((q, g), (k, 1), (v, 1), (q, g))) for _ in range(2)]
        # The slots come from the caching allocator on the compute stream: the first copy in waits for what is
        # already queued there (which may still be using that memory).
        h2d.wait_event(compute.record_event())
        copied, computed, drained = [], [], []
        for c, (b, h0, h1) in enumerate(pieces):
            qd, kd, vd, od = (t[:, :(h1 - h0) * hs] for t, hs in zip(slots[c % 2], (g, 1, 1, g)))
            with torch.cuda.stream(h2d):
                if c >= 2:
                    h2d.wait_event(computed[c - 2])  # this slot's inputs were read by piece c-2's kernel
                qd.copy_(q[b:b + 1, h0 * g:h1 * g], non_blocking=True)
                kd.copy_(k[b:b + 1, h0:h1], non_blocking=True)
                vd.copy_(v[b:b + 1, h0:h1], non_blocking=True)
                copied.append(h2d.record_event())
            compute.wait_event(copied[c])
            if c >= 2:
                compute.wait_event(drained[c - 2])  # this slot's output was copied out by piece c-2
            attention_forward(qd, kd, vd, causal=causal, sm_scale=sm_scale, out=od)
            computed.append(compute.record_event())
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[c])
                out[b:b + 1, h0 * g:h1 * g].copy_(od, non_blocking=True)
                drained.append(d2h.record_event())
        compute.wait_event(drained[-1])
        d2h.synchronize()
    return out


def splitkv_workspace_bytes(q_shape, k_shape, dtype, *, num_splits: int = 0, causal: bool = False) -> tuple[int, int]:
    """(workspace bytes, splits used) that attention_forward_splitkv needs for contiguous inputs of these shapes."""
    B, Hq, M, D = q_shape
    _, Hkv, N, _ = k_shape
    p = _native.FabAttentionParams()
    p.q = p.k = p.v = p.o = 256  # only shapes and strides are read
    p.q_stride_b, p.q_stride_h, p.q_stride_s = Hq * M * D, M * D, D
    p.k_stride_b, p.k_stride_h, p.k_stride_s = Hkv * N * D, N * D, D
    p.v_stride_b, p.v_stride_h, p.v_stride_s = Hkv * N * D, N * D, D
    p.o_stride_b, p.o_stride_h, p.o_stride_s = Hq * M * D, M * D, D
    p.batch, p.heads_q, p.heads_kv, p.seqlen_q, p.seqlen_k, p.head_dim = B, Hq, Hkv, M, N, D
    p.dtype = _native.dtype_code(dtype)
    p.sm_scale = 1.0
    p.causal = 1 if causal else 0
    need, used = ctypes.c_size_t(0), ctypes.c_int(0)
    _native.check(_native.lib.fab_attention_fwd_splitkv_workspace(
        ctypes.byref(p), int(num_splits), ctypes.byref(need), ctypes.byref(used)), "splitkv_workspace_bytes")
    return need.value, used.value


__all__ = [
    "flash_attention_kernel_mapping",
    "flash_attention",
    "attention_forward",
    "attention_forward_splitkv",
    "attention_forward_varlen",
    "attention_forward_host",
    "splitkv_workspace_bytes",
    "_flash_attn_fwd_kernel_basic",
    "_flash_attn_fwd_kernel_optimize_shared_mem",
    "_flash_attn_fwd_kernel_block_d_nomask_contiguous",
]
