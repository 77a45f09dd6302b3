"""Measured choice between the two compiled attention tile families.

The reference's tuner compiles every Triton candidate and keeps the largest
one that fits an SM (tuner.py:503-517).  On sm_100a two tile families are
compiled for each (dtype, head_dim): two 128-row query tiles per CTA with one
S buffer each (`FAB_FA_VARIANT_TWO_TILES`, the default table) and one query
tile with two S buffers (`FAB_FA_VARIANT_ONE_TILE`, twice the CTAs for the
same rows).  Which one is faster depends on the shape, so the choice is made
by measured time:

* `time_variants(q, k, v, causal=...)` times both on the caller's tensors
  (the tuner's `tune_by_time=True` mode);
* `python tune_table.py --out tuned_variants.json` sweeps representative
  shapes on the current GPU and writes the winners; `measured_variant(...)`
  answers from that file for shapes it did not see (nearest measured shape
  with the same dtype width, padded head dim and causality).

The file beside this module is the sm_100a table the library ships; without
it every shape uses the default family.
"""
from __future__ import annotations

import argparse
import json
import math
import os
from functools import lru_cache
from pathlib import Path

import torch

import _native

TABLE_PATH = Path(__file__).resolve().parent / "tuned_variants.json"
VARIANTS = (_native.FAB_FA_VARIANT_TWO_TILES, _native.FAB_FA_VARIANT_ONE_TILE)


def _width(dtype_code: int) -> int:
    return 4 if dtype_code == _native.FAB_DTYPE_F32 else 2


def candidate_variants(dtype_code: int, head_dim: int) -> list[int]:
    """The tile families that cover head_dim, without duplicates (both may name the same tile)."""
    seen, out = set(), []
    for variant in VARIANTS:
        cfg = _native.fa_config_variant(dtype_code, head_dim, variant)
        if cfg is None:
            continue
        key = (cfg.q_tiles_per_cta, cfg.block_n, cfg.stages, cfg.s_buffers)
        if key not in seen:
            seen.add(key)
            out.append(variant)
    return out


def time_variants(q, k, v, *, causal: bool, sm_scale: float | None = None, reps: int = 5, warmup: int = 2,
                  variants=None) -> dict[int, float]:
    """Median milliseconds per call of each tile family on these tensors (CUDA events on the current stream)."""
    from flash_atten import _launch_attention

    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    if variants is None:
        variants = candidate_variants(_native.dtype_code(q.dtype), q.shape[-1])
    o = torch.empty_like(q)
    out: dict[int, float] = {}
    for variant in variants:
        def run():
            _launch_attention(q, k, v, o, None, causal=causal, sm_scale=sm_scale, what="time_variants",
                              variant=variant)
        for _ in range(warmup):
            run()
        times = []
        for _ in range(reps):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            run()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end))
        out[variant] = sorted(times)[len(times) // 2]
    return out


def _shape_point(batch_heads: int, seqlen_q: int, seqlen_k: int) -> tuple[float, float]:
    """Where a shape sits for the nearest-neighbour lookup: log2 of 128-row query tiles and of keys."""
    tiles = batch_heads * max(1, math.ceil(seqlen_q / 128))
    return math.log2(max(tiles, 1)), math.log2(max(seqlen_k, 1))


@lru_cache(maxsize=1)
def _load_table(path: str) -> tuple[dict, ...]:
    try:
        return tuple(json.loads(Path(path).read_text())["entries"])
    except (OSError, ValueError, KeyError):
        return ()


def measured_variant(dtype_code: int, head_dim: int, causal: bool, batch_heads: int, seqlen_q: int,
                     seqlen_k: int, path: str | os.PathLike | None = None) -> int:
    """The family the shipped measurements favour for this shape; the default family when nothing applies."""
    return _measured_variant(int(dtype_code), int(head_dim), bool(causal), int(batch_heads), int(seqlen_q),
                             int(seqlen_k), str(path or TABLE_PATH))


@lru_cache(maxsize=4096)
def _measured_variant(dtype_code: int, head_dim: int, causal: bool, batch_heads: int, seqlen_q: int,
                      seqlen_k: int, path: str) -> int:
    cands = candidate_variants(dtype_code, head_dim)
    if len(cands) < 2:
        return cands[0] if cands else VARIANTS[0]
    d_pad = _native.fa_config(dtype_code, head_dim).head_dim_padded
    entries = [e for e in _load_table(path)
               if e["width"] == _width(dtype_code) and e["head_dim_padded"] == d_pad and e["causal"] == bool(causal)]
    if not entries:
        return VARIANTS[0]
    x, y = _shape_point(batch_heads, seqlen_q, seqlen_k)
    best = min(entries, key=lambda e: (_shape_point(e["batch_heads"], e["seqlen_q"], e["seqlen_k"])[0] - x) ** 2
               + (_shape_point(e["batch_heads"], e["seqlen_q"], e["seqlen_k"])[1] - y) ** 2)
    return int(best["best_variant"]) if int(best["best_variant"]) in cands else VARIANTS[0]


def sweep(dtypes=(torch.bfloat16, torch.float32), head_dims=(64, 128, 256), seqlens=(512, 1024, 2048, 4096, 8192),
          batch_heads=((1, 8), (1, 32), (4, 32)), reps: int = 5) -> list[dict]:
    """Times both families over a grid of shapes on the current GPU."""
    dev = torch.device("cuda", torch.cuda.current_device())
    entries = []
    for dtype in dtypes:
        code = _native.dtype_code(dtype)
        for D in head_dims:
            cands = candidate_variants(code, D)
            if len(cands) < 2:
                continue
            d_pad = _native.fa_config(code, D).head_dim_padded
            for causal in (False, True):
                for S in seqlens:
                    for B, H in batch_heads:
                        g = torch.Generator(device=dev).manual_seed(S + 7 * H + D)
                        q, k, v = (torch.randn(B, H, S, D, device=dev, dtype=dtype, generator=g) for _ in range(3))
                        times = time_variants(q, k, v, causal=causal, reps=reps, variants=cands)
                        best = min(times, key=times.get)
                        entries.append({
                            "width": _width(code), "head_dim_padded": d_pad, "causal": causal,
                            "batch_heads": B * H, "seqlen_q": S, "seqlen_k": S,
                            "ms": {str(k_): round(t, 4) for k_, t in times.items()}, "best_variant": int(best),
                        })
                        del q, k, v
    return entries


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default=str(TABLE_PATH))
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args(argv)
    entries = sweep(reps=args.reps)
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    Path(args.out).write_text(json.dumps({"device": props.name, "sms": props.multi_processor_count,
                                          "entries": entries}, indent=1) + "\n")
    wins = sum(e["best_variant"] == _native.FAB_FA_VARIANT_ONE_TILE for e in entries)
    print(f"wrote {len(entries)} shapes to {args.out}; one-tile family faster on {wins}")


if __name__ == "__main__":
    main()
