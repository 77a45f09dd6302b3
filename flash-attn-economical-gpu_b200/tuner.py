"""Launch-spec builders for the attention kernels (drop-in for the reference's tuner.py).

Public surface and behaviour follow tuner.py of the reference: the same
dataclasses (`LaunchSpec`, `FlashAttentionLaunchSpec`, `FlashAttenTuneArguments`,
tuner.py:19-108), the same tuner classes and constructor checks
(tuner.py:117-157, 593-734), the same positional kernel-argument tuples
(29 arguments for the strided kernels, tuner.py:265-295; 9 for the contiguous
one, tuner.py:640-650), the same per-key class-level cache (tuner.py:119,
159-176, 467-481) and the same `build_flash_attention_launch_spec`
allocation of `o` and fp32 `lse` (tuner.py:563-590).

What differs is the search.  The reference compiles every Triton candidate
tile and keeps the largest one that fits an SM (tuner.py:414-561).  On
sm_100a two tile families are compiled per (dtype, head_dim) into the native
library: two 128-row query tiles per CTA with one S buffer each (the default
table, `fab_flash_attn_config`) and one query tile with two S buffers
(`fab_flash_attn_config_variant`).  The candidates are those families; the
choice is by measured time -- on the caller's tensors with
`tune_by_time=True`, otherwise from the sweep shipped with the library
(`tune_table.measured_variant`).  User tune arguments are validated exactly
as the reference validates them and take part in the cache key; the tile
reported in `FlashAttentionLaunchSpec.tune_args` is the one the kernel runs.

Attribution: the blocks marked "interface kept from the reference" reproduce
the interface of josephzhong/flash-attn-economical-gpu (tuner.py: the launch-spec dataclasses, the tuners' constructor checks and ValueError texts, the kernel argument tuples and the o/lse allocation), which is
licensed under the Apache License, Version 2.0; they are kept as they are so
that callers of the reference, and code that parses its messages, work
unchanged.  Everything else in this module is this project's own.
"""
from __future__ import annotations

import math
from abc import ABC, abstractmethod
from dataclasses import dataclass

import torch

import _native
import tune_table
from exceptions import OutOfResourcesWithDetail, get_sm_resource_limits


def get_architecture():
    major, minor = torch.cuda.get_device_capability(torch.cuda.current_device())
    return major, minor


# Interface kept from the reference (tuner.py:18-108, Apache-2.0): the launch-spec
# dataclasses below, with their validation messages.
@dataclass(frozen=True)
class LaunchSpec:
    grid: tuple[int, ...]
    kernel_args: tuple[object, ...]
    kernel_kwargs: dict[str, object]
    launch_context: dict[str, object]


class Tuner(ABC):
    @abstractmethod
    def build_launch_spec(self, *data: torch.Tensor, **kwargs: object) -> LaunchSpec:
        """Build a fully materialized launch spec from runtime tensors."""

    @abstractmethod
    def build_compiling_context(self, **kwargs: object) -> dict[str, object]:
        """Build resource/compilation context for a candidate launch."""

    @abstractmethod
    def evaluate_candidate(self, *data: torch.Tensor, **kwargs: object) -> tuple[bool, LaunchSpec]:
        """Evaluate a candidate launch and return feasibility plus its launch spec."""


def _next_power_of_two(x: int) -> int:
    if x <= 0:
        raise ValueError("x must be positive")
    return 1 << (x - 1).bit_length()


def next_power_of_two(x: int) -> int:
    return _next_power_of_two(x)


def _get_max_shared_mem_bytes() -> int:
    return int(get_sm_resource_limits()["available_shared_memory_bytes_per_sm"])


@dataclass(frozen=True)
class FlashAttentionLaunchSpec(LaunchSpec):
    function_name: str
    tune_args: "FlashAttenTuneArguments"
    input_shapes: dict[str, tuple[int, ...] | None]

    def update_data(self, data):
        """Swap in new (q, k, v) for the next launch; o and lse stay the same buffers."""
        q, k, v = data
        object.__setattr__(self, "kernel_args", (q, k, v, *self.kernel_args[3:]))


def _check_positive_pow2(name: str, value: int | None, pow2: bool) -> None:
    if value is None:
        return
    if value <= 0:
        raise ValueError(f"{name} must be positive when provided")
    if pow2 and _next_power_of_two(value) != value:
        raise ValueError(f"{name} must be a power of 2 when provided")


@dataclass(frozen=True)
class FlashAttenTuneArguments:
    BLOCK_N: int | None = None
    BLOCK_M: int | None = None
    BLOCK_N_PAD: int | None = None
    BLOCK_DMODEL: int | None = None
    BLOCK_DMODEL_OUTER: int | None = None
    NUM_WARPS: int | None = None
    NUM_STAGES: int | None = None

    def __post_init__(self) -> None:
        _check_positive_pow2("BLOCK_N", self.BLOCK_N, False)
        _check_positive_pow2("BLOCK_M", self.BLOCK_M, True)
        _check_positive_pow2("BLOCK_N_PAD", self.BLOCK_N_PAD, True)
        _check_positive_pow2("BLOCK_DMODEL", self.BLOCK_DMODEL, True)
        _check_positive_pow2("BLOCK_DMODEL_OUTER", self.BLOCK_DMODEL_OUTER, True)
        _check_positive_pow2("NUM_WARPS", self.NUM_WARPS, False)
        _check_positive_pow2("NUM_STAGES", self.NUM_STAGES, False)


def _dtype_from_size(q: torch.Tensor) -> int:
    return _native.dtype_code(q.dtype)


class FlashAttentionTuner(Tuner):
    KERNEL_NAME = "_flash_attn_fwd_kernel_basic"
    _config_cache: dict[tuple[object, ...], tuple[dict[str, int | bool], dict[str, object]]] = {}

    # Interface kept from the reference (tuner.py:115-175, Apache-2.0): the
    # constructor checks and their ValueError texts.
    def __init__(
        self,
        q_shape: tuple[int, int, int, int],
        k_shape: tuple[int, int, int, int],
        v_shape: tuple[int, int, int, int],
        dtype_size: int,
        *,
        causal: bool,
        return_lse: bool,
        tune_args: FlashAttenTuneArguments | None = None,
        tune_by_time: bool = False,
    ) -> None:
        if len(q_shape) != 4 or len(k_shape) != 4 or len(v_shape) != 4:
            raise ValueError("q_shape, k_shape, and v_shape must all be 4D")
        if q_shape[:2] != k_shape[:2] or q_shape[:2] != v_shape[:2]:
            raise ValueError("Batch and head dimensions must match across q_shape, k_shape, and v_shape")
        if q_shape[3] != k_shape[3] or q_shape[3] != v_shape[3]:
            raise ValueError("Last dimension must match across q_shape, k_shape, and v_shape")
        if k_shape[2] != v_shape[2]:
            raise ValueError("k_shape and v_shape sequence lengths must match")
        self.q_shape = tuple(int(d) for d in q_shape)
        self.k_shape = tuple(int(d) for d in k_shape)
        self.v_shape = tuple(int(d) for d in v_shape)
        self.dtype_size = dtype_size
        self.causal = causal
        self.return_lse = return_lse
        self.tune_args = tune_args or FlashAttenTuneArguments()
        self.tune_by_time = bool(tune_by_time)
        self.B, self.H, self.M, self.D = self.q_shape
        _, _, self.N, _ = self.k_shape
        if (
            self.tune_args.BLOCK_DMODEL is not None
            and self.tune_args.BLOCK_DMODEL < self.D
            and not self._allow_block_dmodel_smaller_than_d()
        ):
            raise ValueError("BLOCK_DMODEL must be >= D when provided")
        if self.tune_args.BLOCK_N_PAD is not None and self.tune_args.BLOCK_N is not None:
            if self.tune_args.BLOCK_N > self.tune_args.BLOCK_N_PAD:
                raise ValueError("BLOCK_N cannot exceed BLOCK_N_PAD")
        self.sm_limits = get_sm_resource_limits()
        max_warps = max(1, int(self.sm_limits.get("max_warps_per_block", 1)))
        if self.tune_args.NUM_WARPS is not None and self.tune_args.NUM_WARPS > max_warps:
            raise ValueError(f"NUM_WARPS must be <= {max_warps} for the current device")

    # ---------------------------------------------------------------- caching
    def _cache_key(self, q: torch.Tensor) -> tuple[object, ...]:
        return (
            str(q.device),
            str(q.dtype),
            self.B,
            self.H,
            self.M,
            self.N,
            self.D,
            self.causal,
            self.return_lse,
            self.tune_args.BLOCK_N,
            self.tune_args.BLOCK_M,
            self.tune_args.BLOCK_N_PAD,
            self.tune_args.BLOCK_DMODEL,
            self.tune_args.NUM_WARPS,
            self.tune_args.NUM_STAGES,
            self.tune_by_time,
        )

    def _allow_block_dmodel_smaller_than_d(self) -> bool:
        return False

    # ------------------------------------------------------------ the table
    def _table_entry(self, dtype_code: int) -> _native.FabFaConfig | None:
        return _native.fa_config(dtype_code, self.D)

    def estimate_flash_fwd_shared_bytes(
        self,
        *,
        block_m: int,
        block_n_pad: int,
        block_dmodel: int,
        element_size: int,
    ) -> int:
        """Q tile + one K and one V tile, the reference's estimate (tuner.py:237-245)."""
        return element_size * block_dmodel * (block_m + 2 * block_n_pad)

    def _config_from_entry(self, cfg: _native.FabFaConfig, variant: int = 0) -> dict[str, int | bool]:
        return {
            "variant": int(variant),
            "BLOCK_M": 128 * int(cfg.q_tiles_per_cta),
            "BLOCK_N": int(cfg.block_n),
            "BLOCK_N_PAD": int(cfg.block_n),
            "BLOCK_DMODEL": int(cfg.head_dim_padded),
            "BLOCK_DMODEL_OUTER": int(cfg.head_dim_padded),
            "num_warps": int(cfg.threads) // 32,
            "num_stages": int(cfg.stages),
            "smem_bytes": int(cfg.smem_bytes),
            "tmem_columns": int(cfg.tmem_columns),
        }

    def _candidate_configs(self, dtype_code: int | None = None) -> list[dict[str, int | bool]]:
        """The compiled tile families that cover this head dim (default family first); empty if none does."""
        if dtype_code is None:
            dtype_code = _native.FAB_DTYPE_F16 if self.dtype_size == 2 else _native.FAB_DTYPE_F32
        if self._table_entry(dtype_code) is None:
            return []
        return [self._config_from_entry(_native.fa_config_variant(dtype_code, self.D, variant), variant)
                for variant in tune_table.candidate_variants(dtype_code, self.D)]

    def _effective_causal(self) -> bool:
        return self.causal

    def _choose(self, candidates, q, k, v, sm_scale) -> dict[str, int | bool]:
        """The candidate with the least measured time: timed here, or from the shipped sweep."""
        if len(candidates) == 1:
            return candidates[0]
        if self.tune_by_time:
            times = tune_table.time_variants(q, k, v, causal=self._effective_causal(), sm_scale=sm_scale,
                                             variants=[int(c["variant"]) for c in candidates])
            best = min(times, key=times.get)
        else:
            best = tune_table.measured_variant(_native.dtype_code(q.dtype), self.D, self._effective_causal(),
                                               self.B * self.H, self.M, self.N)
        return next((c for c in candidates if int(c["variant"]) == best), candidates[0])

    # ------------------------------------------------------- launch building
    def _kernel(self):
        import flash_atten

        return getattr(flash_atten, self.KERNEL_NAME)

    def _spec_tune_args(self, config: dict[str, int | bool]) -> FlashAttenTuneArguments:
        return FlashAttenTuneArguments(
            BLOCK_N=int(config["BLOCK_N"]),
            BLOCK_M=int(config["BLOCK_M"]),
            BLOCK_N_PAD=int(config["BLOCK_N_PAD"]),
            BLOCK_DMODEL=int(config["BLOCK_DMODEL"]),
            NUM_WARPS=int(config["num_warps"]),
            NUM_STAGES=int(config["num_stages"]),
        )

    @staticmethod
    def _shapes(q, k, v, o, lse) -> dict[str, tuple[int, ...] | None]:
        return {
            "q": tuple(int(d) for d in q.shape),
            "k": tuple(int(d) for d in k.shape),
            "v": tuple(int(d) for d in v.shape),
            "o": tuple(int(d) for d in o.shape),
            "lse": tuple(int(d) for d in lse.shape) if lse is not None else None,
        }

    def _build_candidate_launch(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        *,
        sm_scale: float,
        o: torch.Tensor,
        lse: torch.Tensor | None,
        config: dict[str, int | bool],
        launch_context: dict[str, object] | None = None,
    ) -> FlashAttentionLaunchSpec:
        grid = (math.ceil(self.M / int(config["BLOCK_M"])), self.B * self.H)
        # Interface kept from the reference (tuner.py:265-295, Apache-2.0): the
        # 29-argument kernel tuple.
        kernel_args = (
            q,
            k,
            v,
            o,
            lse if lse is not None else 0,
            *q.stride(),
            *k.stride(),
            *v.stride(),
            *o.stride(),
            *(lse.stride() if lse is not None else (0, 0, 0)),
            self.H,
            self.M,
            self.N,
            self.D,
            sm_scale,
        )
        kernel_kwargs = {
            "causal": self.causal,
            "HAS_LSE": self.return_lse,
            "BLOCK_M": int(config["BLOCK_M"]),
            "BLOCK_N": int(config["BLOCK_N"]),
            "BLOCK_N_PAD": int(config["BLOCK_N_PAD"]),
            "BLOCK_DMODEL": int(config["BLOCK_DMODEL"]),
            "num_warps": int(config["num_warps"]),
            "num_stages": int(config["num_stages"]),
            "sm100_variant": int(config.get("variant", 0)),
        }
        if launch_context is None:
            launch_context = self.build_compiling_context(
                grid=grid,
                kernel_args=kernel_args,
                kernel_kwargs=kernel_kwargs,
                attempted_shared_memory_bytes_per_block=int(config["smem_bytes"]),
            )
        return FlashAttentionLaunchSpec(
            grid=grid,
            kernel_args=kernel_args,
            kernel_kwargs=kernel_kwargs,
            launch_context=launch_context,
            function_name=self.KERNEL_NAME,
            tune_args=self._spec_tune_args(config),
            input_shapes=self._shapes(q, k, v, o, lse),
        )

    def build_compiling_context(
        self,
        *,
        grid: tuple[int, ...],
        kernel_args: tuple[object, ...],
        kernel_kwargs: dict[str, object],
        attempted_shared_memory_bytes_per_block: int,
    ) -> dict[str, object]:
        """Resource facts of the compiled kernel (replaces Triton `warmup` metadata, tuner.py:341-376)."""
        context: dict[str, object] = dict(self.sm_limits)
        num_warps = kernel_kwargs.get("num_warps")
        if num_warps is not None:
            context["threads_per_block"] = int(num_warps) * int(context["warp_size"])
        context["attempted_shared_memory_bytes_per_block"] = attempted_shared_memory_bytes_per_block
        try:
            compiled = self._kernel().warmup(*kernel_args, grid=grid, **kernel_kwargs)
            compiled._init_handles()
            context["threads_per_block"] = int(compiled.metadata.num_warps) * int(context["warp_size"])
            context["compiled_shared_memory_bytes_per_block"] = int(compiled.metadata.shared)
            context["attempted_shared_memory_bytes_per_block"] = int(compiled.metadata.shared)
            context["tmem_columns"] = int(compiled.metadata.tmem_columns)
            regs = int(compiled.n_regs)
            context["attempted_registers_per_thread"] = regs
            total = regs * int(context["threads_per_block"])
            context["attempted_registers_per_block"] = total
            context["attempted_register_file_size_bytes_per_block"] = total * 4
        except Exception as exc:  # same tolerance as the reference's introspection
            context["resource_introspection_error"] = f"{type(exc).__name__}: {exc}"
        return context

    def evaluate_candidate(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        *,
        sm_scale: float,
        o: torch.Tensor,
        lse: torch.Tensor | None,
        config: dict[str, int | bool],
    ) -> tuple[bool, FlashAttentionLaunchSpec]:
        spec = self._build_candidate_launch(q, k, v, sm_scale=sm_scale, o=o, lse=lse, config=config)
        ctx = spec.launch_context
        shared = int(ctx.get("compiled_shared_memory_bytes_per_block", ctx["attempted_shared_memory_bytes_per_block"]))
        shared_ok = shared <= int(self.sm_limits["available_shared_memory_bytes_per_sm"])
        reg_bytes = ctx.get("attempted_register_file_size_bytes_per_block")
        register_ok = reg_bytes is None or int(reg_bytes) <= int(self.sm_limits["available_register_file_size_bytes_per_sm"])
        return shared_ok and register_ok, spec

    def _validate_runtime_tensors(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        if tuple(q.shape) != self.q_shape or tuple(k.shape) != self.k_shape or tuple(v.shape) != self.v_shape:
            raise ValueError("Runtime tensor shapes do not match the tuner shapes")

    def build_launch_spec(
        self,
        *data: torch.Tensor,
        sm_scale: float,
        o: torch.Tensor,
        lse: torch.Tensor | None,
    ) -> FlashAttentionLaunchSpec:
        if len(data) != 3:
            raise ValueError("FlashAttentionTuner.build_launch_spec expects (q, k, v)")
        q, k, v = data
        self._validate_runtime_tensors(q, k, v)
        key = self._cache_key(q)
        cached = self._config_cache.get(key)
        if cached is not None:
            config, context = cached
            return self._build_candidate_launch(
                q, k, v, sm_scale=sm_scale, o=o, lse=lse, config=dict(config), launch_context=dict(context)
            )
        candidates = self._candidate_configs(_native.dtype_code(q.dtype))
        if not candidates:
            context = dict(self.sm_limits)
            context["attempted_shared_memory_bytes_per_block"] = self.estimate_flash_fwd_shared_bytes(
                block_m=128, block_n_pad=128, block_dmodel=_next_power_of_two(self.D), element_size=q.element_size()
            )
            raise OutOfResourcesWithDetail(
                int(context["attempted_shared_memory_bytes_per_block"]),
                int(self.sm_limits["available_shared_memory_bytes_per_sm"]),
                "shared memory",
                kernel_name=self.KERNEL_NAME,
                launch_context=context,
                extra_detail=f"No sm_100a attention tile covers head_dim={self.D} for dtype {q.dtype}",
            )
        config = self._choose(candidates, q, k, v, sm_scale)
        feasible, spec = self.evaluate_candidate(q, k, v, sm_scale=sm_scale, o=o, lse=lse, config=config)
        if not feasible:
            ctx = spec.launch_context
            raise OutOfResourcesWithDetail(
                int(ctx.get("attempted_shared_memory_bytes_per_block", 0)),
                int(self.sm_limits["available_shared_memory_bytes_per_sm"]),
                "shared memory",
                kernel_name=self.KERNEL_NAME,
                launch_context=ctx,
                extra_detail="The sm_100a attention tile does not fit this device",
            )
        self._config_cache[key] = (dict(config), dict(spec.launch_context))
        return spec

    # Interface kept from the reference (tuner.py:562-590, Apache-2.0): o and
    # fp32 lse allocated as the reference allocates them.
    def build_flash_attention_launch_spec(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        *,
        sm_scale: float | None = None,
    ) -> FlashAttentionLaunchSpec:
        q = q.contiguous()
        k = k.contiguous()
        v = v.contiguous()
        if sm_scale is None:
            sm_scale = q.shape[-1] ** -0.5
        o = torch.empty_like(q)
        lse = (
            torch.empty((q.shape[0], q.shape[1], q.shape[2]), device=q.device, dtype=torch.float32)
            if self.return_lse
            else None
        )
        return self.build_launch_spec(q, k, v, sm_scale=sm_scale, o=o, lse=lse)


class FlashAttentionOptimizeSharedMemTuner(FlashAttentionTuner):
    KERNEL_NAME = "_flash_attn_fwd_kernel_optimize_shared_mem"


class FlashAttentionBlockDNomaskTuner(FlashAttentionTuner):
    """Contiguous, mask-free, LSE-free variant (tuner.py:597-734).

    Like the reference's kernel it computes non-causal attention whatever
    `causal` the tuner was built with (the kernel takes no causal flag).
    """

    KERNEL_NAME = "_flash_attn_fwd_kernel_block_d_nomask_contiguous"

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.max_tile_length = 128

    def _allow_block_dmodel_smaller_than_d(self) -> bool:
        return True

    def _effective_causal(self) -> bool:
        return False  # the kernel takes no causal flag

    def _block_dmodel_outer_candidates(self) -> list[int]:
        if self.tune_args.BLOCK_DMODEL_OUTER is not None:
            return [self.tune_args.BLOCK_DMODEL_OUTER]
        return [int(self.D), int(self.D / 2), int(self.D / 4)]

    def _spec_tune_args(self, config: dict[str, int | bool]) -> FlashAttenTuneArguments:
        return FlashAttenTuneArguments(
            BLOCK_N=int(config["BLOCK_N"]),
            BLOCK_M=int(config["BLOCK_M"]),
            BLOCK_N_PAD=int(config["BLOCK_N_PAD"]),
            BLOCK_DMODEL=int(config["BLOCK_DMODEL"]),
            BLOCK_DMODEL_OUTER=int(config["BLOCK_DMODEL_OUTER"]),
            NUM_WARPS=int(config["num_warps"]),
            NUM_STAGES=int(config["num_stages"]),
        )

    def _build_candidate_launch(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        *,
        sm_scale: float,
        o: torch.Tensor,
        lse: torch.Tensor | None,
        config: dict[str, int | bool],
        launch_context: dict[str, object] | None = None,
    ) -> FlashAttentionLaunchSpec:
        grid = (math.ceil(self.M / int(config["BLOCK_M"])), self.B * self.H)
        # Interface kept from the reference (tuner.py:640-650, Apache-2.0).
        kernel_args = (q, k, v, o, self.H, self.M, self.N, self.D, sm_scale)
        kernel_kwargs = {
            "BLOCK_M": int(config["BLOCK_M"]),
            "BLOCK_N": int(config["BLOCK_N"]),
            "BLOCK_DMODEL": int(config["BLOCK_DMODEL"]),
            "BLOCK_DMODEL_OUTER": int(config["BLOCK_DMODEL_OUTER"]),
            "num_warps": int(config["num_warps"]),
            "num_stages": int(config["num_stages"]),
            "sm100_variant": int(config.get("variant", 0)),
        }
        if launch_context is None:
            launch_context = self.build_compiling_context(
                grid=grid,
                kernel_args=kernel_args,
                kernel_kwargs=kernel_kwargs,
                attempted_shared_memory_bytes_per_block=int(config["smem_bytes"]),
            )
        return FlashAttentionLaunchSpec(
            grid=grid,
            kernel_args=kernel_args,
            kernel_kwargs=kernel_kwargs,
            launch_context=launch_context,
            function_name=self.KERNEL_NAME,
            tune_args=self._spec_tune_args(config),
            input_shapes=self._shapes(q, k, v, o, lse),
        )


__all__ = [
    "FlashAttenTuneArguments",
    "FlashAttentionLaunchSpec",
    "FlashAttentionTuner",
    "FlashAttentionOptimizeSharedMemTuner",
    "FlashAttentionBlockDNomaskTuner",
    "LaunchSpec",
    "Tuner",
    "_get_max_shared_mem_bytes",
    "_next_power_of_two",
    "get_architecture",
    "next_power_of_two",
]
