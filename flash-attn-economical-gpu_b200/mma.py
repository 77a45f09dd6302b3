"""Matmul on B200 (drop-in for the reference's mma.py).

`_matmul_contiguous_kernel[grid](a, b, c, M, N, K, BLOCK_M=..., BLOCK_N=...,
BLOCK_K=..., GROUP_M=..., USE_CACHE_EVICTION_HINTS=..., num_warps=...,
num_stages=...)` keeps the Triton kernel's call form (mma.py:8-21) and
result: C = A B over row-major contiguous storage with fp32 accumulation,
rounded to fp16 and then stored in C's dtype (mma.py:51-52).  It runs the
sm_100a tcgen05 GEMM through the C ABI (`fab_matmul_contiguous`), which picks
the kernel: 16-bit problems of at least one wave of 256x256 tiles run on CTA
pairs (tcgen05 cta_group::2, one tile per two SMs, tiles handed out in raster
order by cluster launch control), the rest on one CTA per 128x256 tile;
the Triton tiling keywords (BLOCK_*, GROUP_M, cache hints, num_warps,
num_stages) are accepted and not needed.  `_select_2d_contiguous_config` accepts and
rejects exactly the shapes the reference accepts and rejects (mma.py:63-81)
and reports the tile the sm_100a kernel uses.
"""
from __future__ import annotations

import ctypes
import logging

import torch

import _native
from tuner import get_architecture

logger = logging.getLogger(__name__)

# Tile of the single-CTA sm_100a kernel, reported as the launch config:
# 128x256 outputs per CTA, one 128-byte swizzle atom of K per stage, 4 stages,
# 8 warps (TMA, MMA, 4 epilogue + 2 spare).  Each CTA of a pair holds the same
# 128 rows and half of a 256-wide tile's columns per stage.
SM100_BLOCK_M = 128
SM100_BLOCK_N = 256
SM100_NUM_WARPS = 8
SM100_NUM_STAGES = 4


def _sm100_block_k(element_size: int = 2) -> int:
    return 128 // element_size


def _require_cuda_tensor(name: str, t) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU implementation)")


def _gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    c: torch.Tensor,
    M: int,
    N: int,
    K: int,
    *,
    lda: int,
    ldb: int,
    ldc: int,
    round_f16: bool,
    group_m: int = 8,
    epilogue: int = _native.FAB_GEMM_EPILOGUE_STORE,
    rope: tuple | None = None,
    row_scale: torch.Tensor | None = None,
    workspace: torch.Tensor | bool | None = None,
    what: str = "gemm",
) -> None:
    """C[M,N] = A[M,K] B[K,N] over row-major storage with leading dims (elements).

    With the SwiGLU epilogue C is [M, N/2] (see `matmul_swiglu`); with the bias + RoPE epilogue `rope` is
    (bias or None, cos, sin, rope_cols, head_dim) (see `matmul_bias_rope`).  `row_scale` (fp32 [M] or None)
    multiplies row r's accumulator by row_scale[r] before the epilogue (an RMSNorm folded into the GEMM).
    `workspace`: None uses the device's shared stream-K workspace when the layout wants one (`gemm_workspace`),
    False runs whole tiles, a zero-filled uint8 CUDA tensor is used as given."""
    for name, t in (("a", a), ("b", b), ("c", c)):
        _require_cuda_tensor(name, t)
    if a.dtype != b.dtype:
        raise ValueError(f"{what}: a and b must share one dtype, got {a.dtype} and {b.dtype}")
    p = _native.FabGemmParams()
    p.a, p.b, p.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    p.lda, p.ldb, p.ldc = int(lda), int(ldb), int(ldc)
    p.M, p.N, p.K = int(M), int(N), int(K)
    p.in_dtype = _native.dtype_code(a.dtype)
    p.out_dtype = _native.dtype_code(c.dtype)
    p.round_f16 = 1 if round_f16 else 0
    p.group_m = int(group_m)
    p.epilogue = int(epilogue)
    if rope is not None:
        bias, cos, sin, rope_cols, head_dim = rope
        p.bias = bias.data_ptr() if bias is not None else None
        p.rope_cos, p.rope_sin = cos.data_ptr(), sin.data_ptr()
        p.rope_cols, p.head_dim = int(rope_cols), int(head_dim)
    if row_scale is not None:
        _require_cuda_tensor("row_scale", row_scale)
        if row_scale.dtype != torch.float32 or row_scale.numel() < M or not row_scale.is_contiguous():
            raise ValueError(f"{what}: row_scale must be a contiguous float32 tensor of at least {M} elements")
        p.row_scale = row_scale.data_ptr()
    with torch.cuda.device(a.device):
        if workspace is not False:
            need = ctypes.c_size_t(0)
            _native.check(_native.lib.fab_gemm_workspace_size(ctypes.byref(p), ctypes.byref(need)), what)
            if need.value:
                ws = gemm_workspace(a.device, need.value) if workspace is None else workspace
                p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel() * ws.element_size()
        rc = _native.lib.fab_gemm(ctypes.byref(p), ctypes.c_void_p(_native.current_stream_handle(a.device)))
    _native.check(rc, what)


_KERNEL_NAMES = {_native.FAB_GEMM_KERNEL_SINGLE: "single", _native.FAB_GEMM_KERNEL_PAIR: "pair",
                 _native.FAB_GEMM_KERNEL_SPLITK: "splitk", _native.FAB_GEMM_KERNEL_PAIR_STREAMK: "pair_streamk"}

# Stream-K workspaces, one per device, grown on demand and zero-filled when made (the kernel leaves its flag
# words zero again).  Calls on one device share it, so they must be ordered (one stream, or graph replays of
# one stream); callers that overlap GEMMs pass their own `workspace`.
_WORKSPACES: dict[int, torch.Tensor] = {}


def gemm_workspace(device, nbytes: int) -> torch.Tensor:
    """The device's shared stream-K workspace, at least `nbytes` long (uint8, 256-byte aligned, zeroed)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=torch.device("cuda", idx))
        _WORKSPACES[idx] = ws
    return ws


def kernel_plan(M: int, N: int, K: int, in_dtype: torch.dtype = torch.bfloat16,
                out_dtype: torch.dtype | None = None, device=None) -> tuple[str, int, int]:
    """(kernel, k_split, tile_n) that `matmul` runs for row-major contiguous operands of these shapes.

    kernel: "single" (one CTA per 128 x tile_n tile; tile_n 256, or 128 / 64 for small 16-bit problems), "pair"
    (CTA pairs per 256 x tile_n tile), "pair_streamk" (the same, with the K blocks of the tiles past the full
    waves split evenly over all pairs) or "splitk" (a cluster of k_split CTAs shares each 128x256 tile's K).  No
    counterpart in the reference; it reads only the shapes.
    """
    out_dtype = in_dtype if out_dtype is None else out_dtype
    p = _native.FabGemmParams()
    p.a = p.b = p.c = 256  # only shapes are read
    p.lda, p.ldb, p.ldc = max(int(K), 1), max(int(N), 1), max(int(N), 1)
    p.M, p.N, p.K = int(M), int(N), int(K)
    p.in_dtype = _native.dtype_code(in_dtype)
    p.out_dtype = _native.dtype_code(out_dtype)
    p.workspace, p.workspace_bytes = 256, 1 << 40  # what `matmul` runs: its shared workspace is large enough
    kernel, split, tile_n = ctypes.c_int(0), ctypes.c_int(1), ctypes.c_int(256)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _native.check(_native.lib.fab_gemm_plan(ctypes.byref(p), ctypes.byref(kernel), ctypes.byref(split),
                                                ctypes.byref(tile_n)), "kernel_plan")
    return _KERNEL_NAMES[kernel.value], split.value, tile_n.value


def kernel_grid(M: int, N: int, K: int, in_dtype: torch.dtype = torch.bfloat16, device=None) -> int:
    """CTAs in the grid `matmul` launches for these shapes (two per pair for the CTA-pair kernels)."""
    p = _native.FabGemmParams()
    p.a = p.b = p.c = 256
    p.lda, p.ldb, p.ldc = max(int(K), 1), max(int(N), 1), max(int(N), 1)
    p.M, p.N, p.K = int(M), int(N), int(K)
    p.in_dtype = p.out_dtype = _native.dtype_code(in_dtype)
    p.workspace, p.workspace_bytes = 256, 1 << 40
    ctas = ctypes.c_longlong(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _native.check(_native.lib.fab_gemm_grid(ctypes.byref(p), ctypes.byref(ctas)), "kernel_grid")
    return int(ctas.value)


class _MatmulKernel:
    """Stands in for the Triton JITFunction `_matmul_contiguous_kernel`."""

    __name__ = "_matmul_contiguous_kernel"

    def __repr__(self) -> str:
        return "<sm_100a matmul kernel _matmul_contiguous_kernel>"

    def __getitem__(self, grid):
        def launch(a, b, c, M, N, K, **kwargs):
            return self._run(a, b, c, int(M), int(N), int(K), kwargs)

        return launch

    def _run(self, a, b, c, M, N, K, kwargs):
        for name, t in (("a", a), ("b", b), ("c", c)):
            _require_cuda_tensor(name, t)
        if a.numel() < M * K or b.numel() < K * N or c.numel() < M * N:
            raise ValueError("_matmul_contiguous_kernel: a, b, c are smaller than M*K, K*N, M*N")
        ok = all(t.is_contiguous() and t.data_ptr() % 16 == 0 for t in (a, b, c))
        es_in, es_out = a.element_size(), c.element_size()
        ok = ok and (K * es_in) % 16 == 0 and (N * es_in) % 16 == 0 and (N * es_out) % 16 == 0
        if not ok:
            raise ValueError(
                "_matmul_contiguous_kernel needs contiguous 16-byte aligned a, b, c and rows of K and N "
                "elements that are multiples of 16 bytes"
            )
        with torch.cuda.device(a.device):
            rc = _native.lib.fab_matmul_contiguous(
                a.data_ptr(),
                b.data_ptr(),
                c.data_ptr(),
                M,
                N,
                K,
                _native.dtype_code(a.dtype),
                _native.dtype_code(c.dtype),
                1,
                ctypes.c_void_p(_native.current_stream_handle(a.device)),
            )
        _native.check(rc, "_matmul_contiguous_kernel")

    def warmup(self, *args, grid=None, **kwargs):
        a = args[0]
        attrs = _native.kernel_attrs(_native.FAB_KERNEL_MATMUL, _native.dtype_code(a.dtype))
        return attrs


_matmul_contiguous_kernel = _MatmulKernel()


def _supports_contiguous_cache_eviction_hints(device=None) -> bool:
    if not torch.cuda.is_available():
        return False
    major, _ = torch.cuda.get_device_capability(device)
    return major >= 8


def _select_2d_contiguous_config(m: int, n: int, k: int) -> tuple[int, int, int, int, int, int]:
    """(BLOCK_M, BLOCK_N, BLOCK_K, GROUP_M, num_warps, num_stages) for an accepted shape.

    Acceptance and error messages follow mma.py:63-81; the returned tile is
    the sm_100a kernel's (it has no divisibility requirement of its own).
    """
    if k % 32 != 0:
        raise ValueError("fast 2D contiguous matmul requires K % 32 == 0")
    accepted = (
        (m >= 2048 and n >= 2048 and m % 128 == 0 and n % 128 == 0)
        or (m % 128 == 0 and n % 64 == 0)
        or (m % 128 == 0 and n % 128 == 0)
        or (m % 64 == 0 and n % 256 == 0)
    )
    if not accepted:
        raise ValueError(
            "fast 2D contiguous matmul requires a supported divisible tile: "
            "(M % 128 == 0 and N % 64 == 0), "
            "(M % 128 == 0 and N % 128 == 0), or "
            "(M % 64 == 0 and N % 256 == 0), with K % 32 == 0"
        )
    return SM100_BLOCK_M, SM100_BLOCK_N, _sm100_block_k(2), 8, SM100_NUM_WARPS, SM100_NUM_STAGES


def matmul(a: torch.Tensor, b: torch.Tensor, *, out_dtype: torch.dtype | None = None, round_f16: bool = False,
           stream_k: bool = True) -> torch.Tensor:
    """C = A B for 2-D row-major a [M, K], b [K, N] (any leading dims with unit column stride).

    `stream_k` lets CTA-pair GEMMs whose tiles leave part of the last wave idle split the remaining tiles'
    K over all pairs (through the device's shared workspace, `gemm_workspace`); False runs whole tiles,
    which sum each output in the same order as the fused-epilogue GEMMs (`matmul_swiglu`,
    `matmul_bias_rope`)."""
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"matmul expects a [M, K] and b [K, N], got {tuple(a.shape)} and {tuple(b.shape)}")
    M, K = a.shape
    N = b.shape[1]
    if a.stride(1) != 1:
        a = a.contiguous()
    if b.stride(1) != 1:
        b = b.contiguous()
    c = torch.empty((M, N), device=a.device, dtype=out_dtype or a.dtype)
    _gemm(a, b, c, M, N, K, lda=a.stride(0), ldb=b.stride(0), ldc=c.stride(0), round_f16=round_f16,
          workspace=None if stream_k else False, what="matmul")
    return c


SWIGLU_BLOCK = 64  # gate/up column interleave of the SwiGLU epilogue


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """[K, 2m] weight whose columns alternate `block` gate and `block` up columns (m a multiple of block)."""
    if w_gate.shape != w_up.shape or w_gate.ndim != 2 or w_gate.shape[1] % block != 0:
        raise ValueError(f"interleave_gate_up expects two [K, m] weights with m % {block} == 0, "
                         f"got {tuple(w_gate.shape)} and {tuple(w_up.shape)}")
    K, m = w_gate.shape
    return torch.stack([w_gate.reshape(K, m // block, block), w_up.reshape(K, m // block, block)],
                       dim=2).reshape(K, 2 * m).contiguous()


def split_gate_up(gu: torch.Tensor, block: int = SWIGLU_BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    """The gate and up halves [.., m] of an interleaved [.., 2m] product (copies)."""
    *lead, two_m = gu.shape
    v = gu.reshape(*lead, two_m // (2 * block), 2, block)
    return v[..., 0, :].reshape(*lead, two_m // 2), v[..., 1, :].reshape(*lead, two_m // 2)


def matmul_bias_rope(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, cos: torch.Tensor,
                     sin: torch.Tensor, *, rope_cols: int, head_dim: int,
                     out: torch.Tensor | None = None, row_scale: torch.Tensor | None = None) -> torch.Tensor:
    """C = rope(a @ w + bias): a QKV projection with its bias and rotate-half rotary embedding in the epilogue.

    a [S, K], w [K, N] (16-bit, unit column stride), bias [N] or None, cos/sin [>=S, head_dim] contiguous tables
    (row r = position r).  Every column gets the bias; the heads of head_dim columns among the first rope_cols
    are rotated.  Equals `matmul(a, w)` followed by the bias add and `q*cos + rotate_half(q)*sin` in the
    16-bit type, bit for bit.  No counterpart in the reference (its model adds the bias and applies RoPE as
    separate PyTorch ops).  With `row_scale` (fp32 [S]) row r's product is scaled by row_scale[r] first: an
    RMSNorm folded in (see `fold_rmsnorm_weight`).
    """
    for name, t in (("a", a), ("w", w), ("cos", cos), ("sin", sin)) + ((("bias", bias),) if bias is not None else ()):
        _require_cuda_tensor(name, t)
    if a.dtype not in (torch.float16, torch.bfloat16) or w.dtype != a.dtype:
        raise ValueError("matmul_bias_rope: a and w must share one 16-bit dtype")
    for name, t in (("cos", cos), ("sin", sin)) + ((("bias", bias),) if bias is not None else ()):
        if t.dtype != a.dtype or not t.is_contiguous():
            raise ValueError(f"matmul_bias_rope: {name} must be contiguous in {a.dtype}")
    if a.ndim != 2 or w.ndim != 2 or a.shape[1] != w.shape[0]:
        raise ValueError(f"matmul_bias_rope expects a [S, K] and w [K, N], got {tuple(a.shape)} and {tuple(w.shape)}")
    M, K = a.shape
    N = w.shape[1]
    if cos.shape != sin.shape or cos.ndim != 2 or cos.shape[1] != head_dim or cos.shape[0] < M:
        raise ValueError("matmul_bias_rope: cos and sin must be [>= S, head_dim]")
    if bias is not None and bias.numel() != N:
        raise ValueError("matmul_bias_rope: bias must have N elements")
    if a.stride(1) != 1:
        a = a.contiguous()
    if w.stride(1) != 1:
        w = w.contiguous()
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=a.dtype)
    _gemm(a, w, out, M, N, K, lda=a.stride(0), ldb=w.stride(0), ldc=out.stride(0), round_f16=False,
          epilogue=_native.FAB_GEMM_EPILOGUE_BIAS_ROPE, rope=(bias, cos, sin, rope_cols, head_dim),
          row_scale=row_scale, what="matmul_bias_rope")
    return out


def matmul_swiglu(a: torch.Tensor, w_gate_up: torch.Tensor, *, out: torch.Tensor | None = None,
                  row_scale: torch.Tensor | None = None) -> torch.Tensor:
    """silu(a @ W_gate) * (a @ W_up) [M, m] in one kernel, for w_gate_up = interleave_gate_up(W_gate, W_up).

    No counterpart in the reference (its matmul has one epilogue).  The tcgen05 GEMM's epilogue warps read
    each 64-column gate block and its up block from the same accumulator tile and store only the product,
    rounding as the PyTorch expression does in a's 16-bit dtype: silu of the rounded gate product, rounded,
    times the rounded up product, rounded.  `row_scale` as in `matmul_bias_rope`."""
    if a.ndim != 2 or w_gate_up.ndim != 2 or a.shape[1] != w_gate_up.shape[0]:
        raise ValueError(f"matmul_swiglu expects a [M, K] and w [K, 2m], got {tuple(a.shape)} and "
                         f"{tuple(w_gate_up.shape)}")
    if a.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"matmul_swiglu needs float16 or bfloat16 operands, got {a.dtype}")
    M, K = a.shape
    N = w_gate_up.shape[1]
    if N % (2 * SWIGLU_BLOCK) != 0:
        raise ValueError(f"matmul_swiglu needs 2m a multiple of {2 * SWIGLU_BLOCK}, got {N}")
    if a.stride(1) != 1:
        a = a.contiguous()
    if w_gate_up.stride(1) != 1:
        w_gate_up = w_gate_up.contiguous()
    c = torch.empty((M, N // 2), device=a.device, dtype=a.dtype) if out is None else out
    _gemm(a, w_gate_up, c, M, N, K, lda=a.stride(0), ldb=w_gate_up.stride(0), ldc=c.stride(0), round_f16=False,
          epilogue=_native.FAB_GEMM_EPILOGUE_SWIGLU, row_scale=row_scale, what="matmul_swiglu")
    return c


def fold_rmsnorm_weight(norm_weight: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """B' = diag(norm_weight) B: an RMSNorm's weight folded into the [K, N] weight of the GEMM after it.

    With it, rmsnorm(x) @ B equals rstd * (x @ B') row by row, where rstd = rsqrt(mean(x^2) + eps), which
    `fab_rmsnorm_rstd` computes and the GEMM applies through `row_scale`.  The folded weight is rounded to
    B's dtype once, so results agree with the unfused PyTorch expression within rounding, not bit for bit."""
    if norm_weight.ndim != 1 or w.ndim != 2 or norm_weight.numel() != w.shape[0]:
        raise ValueError(f"fold_rmsnorm_weight expects weight [K] and B [K, N], got {tuple(norm_weight.shape)} "
                         f"and {tuple(w.shape)}")
    return (norm_weight.float()[:, None] * w.float()).to(w.dtype).contiguous()


__all__ = [
    "_select_2d_contiguous_config",
    "_supports_contiguous_cache_eviction_hints",
    "_matmul_contiguous_kernel",
    "matmul",
    "matmul_swiglu",
    "matmul_bias_rope",
    "fold_rmsnorm_weight",
    "kernel_plan",
    "kernel_grid",
    "gemm_workspace",
    "interleave_gate_up",
    "split_gate_up",
    "get_architecture",
]
