"""Resource limits and the rich out-of-resources error of the drop-in API.

Same public surface as the reference's exceptions.py for the hot path:
`OutOfResourcesWithDetail` (exceptions.py:695-757), `get_sm_resource_limits`
(exceptions.py:760-775) and `_resource_usage_summary` (exceptions.py:633-685).
Device facts come from the C ABI (`fab_device_limits_query`), not from
Triton's driver.  The reference's Triton IR / PTX transfer analysis
(exceptions.py:14-631) is not reproduced: it parses compiler-written PTX, and
it is unreachable at run time in the reference (nothing stores a PTX path in
the launch context).  Register and shared-memory usage come from
`cudaFuncGetAttributes` through the C ABI instead.

Attribution: the blocks marked "interface kept from the reference" reproduce
the interface of josephzhong/flash-attn-economical-gpu (exceptions.py: the out-of-resources error class, its hint sentences and message format), which is
licensed under the Apache License, Version 2.0; they are kept as they are so
that callers of the reference, and code that parses its messages, work
unchanged.  Everything else in this module is this project's own.
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import asdict, is_dataclass
from typing import Any

import _native


class OutOfResources(Exception):
    """A launch needs more of a per-SM resource than the device has.

    Same constructor, attributes and message as Triton's OutOfResources, which
    the reference's error class derives from.
    """

    def __init__(self, required, limit, name):
        super().__init__(required, limit, name)
        self.required = required
        self.limit = limit
        self.name = name

    def __str__(self) -> str:
        return (
            f"out of resource: {self.name}, Required: {self.required}, Hardware limit: {self.limit}. "
            "Reducing block sizes or `num_stages` may help."
        )

    def __reduce__(self):
        return (type(self), (self.required, self.limit, self.name))


def _format_tune_args(tune_args: Any | None) -> str | None:
    if tune_args is None:
        return None
    if is_dataclass(tune_args):
        fields = asdict(tune_args)
    elif isinstance(tune_args, Mapping):
        fields = dict(tune_args)
    else:
        fields = {name: getattr(tune_args, name) for name in dir(tune_args) if name.isupper() and not name.startswith("_")}
    text = ", ".join(f"{k}={v}" for k, v in fields.items() if v is not None)
    return text or None


def _format_input_shapes(input_shapes: Any | None) -> str | None:
    if input_shapes is None:
        return None
    fields = dict(input_shapes) if isinstance(input_shapes, Mapping) else {"input_shapes": input_shapes}
    text = ", ".join(f"{k}={v}" for k, v in fields.items() if v is not None)
    return text or None


def _resource_usage_summary(
    name: str,
    launch_context: Mapping[str, Any] | None,
    tune_args: Any | None = None,
    input_shapes: Any | None = None,
) -> str:
    """One-block resource report in the reference's text format."""
    ctx = launch_context or {}
    shared_used = int(ctx.get("compiled_shared_memory_bytes_per_block", ctx.get("attempted_shared_memory_bytes_per_block", 0)))
    lines = [
        f"{name} tuner resources: ",
        f"shared={shared_used}/{int(ctx.get('available_shared_memory_bytes_per_sm', 0))} bytes per block/SM, ",
        f"register_file={int(ctx.get('attempted_register_file_size_bytes_per_block', 0))}/"
        f"{int(ctx.get('available_register_file_size_bytes_per_sm', 0))} bytes per block/SM, ",
        f"registers={int(ctx.get('attempted_registers_per_block', 0))}/"
        f"{int(ctx.get('available_registers_per_sm', 0))} per block/SM ",
    ]
    summary = "\n".join(lines)
    if ctx.get("tmem_columns") is not None:
        summary += f", \ntmem_columns={int(ctx['tmem_columns'])}"
    tune_text = _format_tune_args(tune_args)
    if tune_text:
        summary += f", \ntune_args={tune_text}"
    shape_text = _format_input_shapes(input_shapes)
    if shape_text:
        summary += f", \ninput_shapes={shape_text}"
    return summary


def _resource_failure_text(prefix: str, exc: "OutOfResourcesWithDetail") -> str:
    return f"{prefix}: {exc} [{_resource_usage_summary('failed', getattr(exc, 'launch_context', {}) or {})}]"


# Interface kept from the reference (exceptions.py:695-757, Apache-2.0).
class OutOfResourcesWithDetail(OutOfResources):
    """Out-of-resources error carrying the kernel name and launch context."""

    def __init__(
        self,
        required: int,
        limit: int,
        name: str,
        *,
        kernel_name: str | None = None,
        launch_context: Mapping[str, Any] | None = None,
        extra_detail: str | None = None,
        original_exception: BaseException | None = None,
    ) -> None:
        super().__init__(required, limit, name)
        self.kernel_name = kernel_name
        self.launch_context = dict(launch_context or {})
        self.extra_detail = extra_detail
        self.original_exception = original_exception

    @classmethod
    def from_out_of_resources(
        cls,
        exc: OutOfResources,
        *,
        kernel_name: str | None = None,
        launch_context: Mapping[str, Any] | None = None,
        extra_detail: str | None = None,
    ) -> "OutOfResourcesWithDetail":
        return cls(
            exc.required,
            exc.limit,
            exc.name,
            kernel_name=kernel_name,
            launch_context=launch_context,
            extra_detail=extra_detail,
            original_exception=exc,
        )

    def _resource_hint(self) -> str:
        resource = str(self.name).lower()
        if "register" in resource:
            return "The block likely needs more register file capacity per SM than the hardware can provide."
        if "shared" in resource:
            return "The block likely needs more shared memory per SM than the hardware can provide."
        return "The block likely exceeds a per-SM hardware resource limit for this launch configuration."

    def _format_context(self) -> str | None:
        if not self.launch_context:
            return None
        return "\n".join(f"{k}={v}" for k, v in self.launch_context.items())

    def __str__(self) -> str:
        parts = [super().__str__(), self._resource_hint()]
        if self.kernel_name:
            parts.append(f"Kernel: {self.kernel_name}.")
        context = self._format_context()
        if context:
            parts.append(f"Launch context: {context}.")
        if self.extra_detail:
            parts.append(self.extra_detail.rstrip(".") + ".")
        return " ".join(parts)


def get_sm_resource_limits() -> dict[str, Any]:
    """Per-block / per-SM limits of the current CUDA device (same keys as the reference)."""
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("get_sm_resource_limits() needs a CUDA device")
    lim = _native.device_limits(torch.cuda.current_device())
    warp = int(lim.warp_size)
    max_threads = int(lim.max_threads_per_block)
    return {
        "available_shared_memory_bytes_per_sm": int(lim.shared_bytes_per_block_optin),
        "available_registers_per_sm": int(lim.registers_per_sm),
        "available_register_file_size_bytes_per_sm": int(lim.registers_per_sm) * 4,
        "warp_size": warp,
        "max_threads_per_block": max_threads,
        "max_warps_per_block": max(1, max_threads // max(1, warp)),
        "multiprocessor_count": int(lim.multiprocessor_count),
    }


__all__ = [
    "OutOfResources",
    "OutOfResourcesWithDetail",
    "get_sm_resource_limits",
    "_resource_usage_summary",
    "_resource_failure_text",
    "_format_tune_args",
    "_format_input_shapes",
]
