"""Generate the golden vectors in this directory from the reference itself.

Runs the reference's own Triton kernels (flash_atten.py, mma.py of
josephzhong/flash-attn-economical-gpu) in Triton's CPU interpreter
(TRITON_INTERPRET=1) on small seeded inputs and stores inputs and outputs in
golden.npz plus a case list in golden.json.  It needs the reference checkout
(its directory is the one required argument) and Triton, so it runs only
where those exist; the committed .npz/.json files are what the tests read.

Triton's interpreter computes bf16 incorrectly (it round-trips through numpy,
which has no bf16), so the cases are fp16 and fp32, the dtypes the reference's
own tests and its fp32 correctness case use.

Usage: python tests/golden/make_golden.py <reference checkout directory>
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent


def main() -> None:
    if len(sys.argv) != 2 or not (Path(sys.argv[1]) / "flash_atten.py").is_file():
        sys.exit("usage: make_golden.py <reference checkout directory holding flash_atten.py and mma.py>")
    sys.path.insert(0, str(Path(sys.argv[1]).resolve()))
    import numpy as np
    import torch

    import flash_atten as ref_fa  # the reference's module, under the interpreter
    import mma as ref_mma

    arrays: dict[str, np.ndarray] = {}
    cases: list[dict] = []

    def rand(gen, shape, dtype):
        return torch.randn(*shape, generator=gen, dtype=torch.float32).to(dtype)

    def store(name, **tensors):
        for key, t in tensors.items():
            if t is None:
                continue
            a = t.detach().cpu()
            arrays[f"{name}.{key}"] = a.numpy() if a.dtype in (torch.float16, torch.float32) else a.float().numpy()

    def strided_case(name, kernel, B, H, M, N, D, causal, has_lse, dtype, blocks, seed, sm_scale=None):
        gen = torch.Generator().manual_seed(seed)
        q, k, v = rand(gen, (B, H, M, D), dtype), rand(gen, (B, H, N, D), dtype), rand(gen, (B, H, N, D), dtype)
        o = torch.empty_like(q)
        lse = torch.empty((B, H, M), dtype=torch.float32) if has_lse else None
        scale = D ** -0.5 if sm_scale is None else sm_scale
        bm, bn, bd = blocks
        grid = ((M + bm - 1) // bm, B * H)
        kern = getattr(ref_fa, kernel)
        kern[grid](
            q, k, v, o, lse if lse is not None else 0,
            *q.stride(), *k.stride(), *v.stride(), *o.stride(),
            *(lse.stride() if lse is not None else (0, 0, 0)),
            H, M, N, D, scale,
            causal=causal, HAS_LSE=has_lse, BLOCK_M=bm, BLOCK_N=bn, BLOCK_N_PAD=bn, BLOCK_DMODEL=bd,
        )
        store(name, q=q, k=k, v=v, o=o, lse=lse)
        cases.append(dict(name=name, kind="attention", kernel=kernel, B=B, Hq=H, Hkv=H, M=M, N=N, D=D, causal=causal,
                          has_lse=has_lse, dtype=str(dtype).replace("torch.", ""), sm_scale=scale, seed=seed,
                          blocks=list(blocks)))

    def nomask_case(name, B, Hq, Hkv, S, D, bd, outer, dtype, seed):
        gen = torch.Generator().manual_seed(seed)
        q = rand(gen, (B, Hq, S, D), dtype)
        k = rand(gen, (B, Hkv, S, D), dtype)
        v = rand(gen, (B, Hkv, S, D), dtype)
        # The reference's SDPA path repeats K/V heads for grouped queries (ttft.py:203-219).
        kr = k.repeat_interleave(Hq // Hkv, dim=1).contiguous()
        vr = v.repeat_interleave(Hq // Hkv, dim=1).contiguous()
        o = torch.empty_like(q)
        scale = D ** -0.5
        bm = bn = 64
        ref_fa._flash_attn_fwd_kernel_block_d_nomask_contiguous[(S // bm, B * Hq)](
            q, kr, vr, o, Hq, S, S, D, scale, BLOCK_M=bm, BLOCK_N=bn, BLOCK_DMODEL=bd, BLOCK_DMODEL_OUTER=outer,
        )
        store(name, q=q, k=k, v=v, o=o)
        cases.append(dict(name=name, kind="attention", kernel="_flash_attn_fwd_kernel_block_d_nomask_contiguous",
                          B=B, Hq=Hq, Hkv=Hkv, M=S, N=S, D=D, causal=False, has_lse=False,
                          dtype=str(dtype).replace("torch.", ""), sm_scale=scale, seed=seed, blocks=[bm, bn, bd, outer]))

    def mma_case(name, M, K, N, dtype, seed, blocks=(64, 64, 32, 2)):
        gen = torch.Generator().manual_seed(seed)
        a = (torch.randn(M, K, generator=gen) / K ** 0.5).to(dtype)
        b = (torch.randn(K, N, generator=gen) / K ** 0.5).to(dtype)
        c = torch.empty((M, N), dtype=dtype)
        bm, bn, bk, gm = blocks
        grid = ((M // bm) * (N // bn),)
        ref_mma._matmul_contiguous_kernel[grid](
            a, b, c, M, N, K, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk, GROUP_M=gm, USE_CACHE_EVICTION_HINTS=False,
        )
        store(name, a=a, b=b, c=c)
        cases.append(dict(name=name, kind="matmul", M=M, K=K, N=N, dtype=str(dtype).replace("torch.", ""),
                          seed=seed, blocks=list(blocks)))

    f16, f32 = torch.float16, torch.float32
    # the fp32 benchmark case exactly: B1 H4 S256 D64 fp32, seed 0, scale 1/8, non-causal.
    strided_case("cfg1_fp32", "_flash_attn_fwd_kernel_basic", 1, 4, 256, 256, 64, False, True, f32, (64, 64, 64), 0, 0.125)
    strided_case("basic_ragged_causal", "_flash_attn_fwd_kernel_basic", 1, 2, 40, 37, 64, True, True, f16, (16, 16, 64), 1)
    strided_case("basic_d128", "_flash_attn_fwd_kernel_basic", 2, 1, 70, 130, 128, False, True, f16, (32, 32, 128), 2)
    strided_case("basic_d256_causal", "_flash_attn_fwd_kernel_basic", 1, 1, 96, 96, 256, True, True, f16, (32, 32, 256), 3)
    strided_case("basic_tiny", "_flash_attn_fwd_kernel_basic", 1, 1, 1, 1, 64, True, True, f16, (16, 16, 64), 4)
    strided_case("basic_rect_causal", "_flash_attn_fwd_kernel_basic", 1, 2, 150, 50, 64, True, True, f16, (32, 32, 64), 5)
    strided_case("opt_causal_d128", "_flash_attn_fwd_kernel_optimize_shared_mem", 1, 2, 100, 100, 128, True, True, f16,
                 (32, 32, 128), 6)
    strided_case("opt_d64", "_flash_attn_fwd_kernel_optimize_shared_mem", 2, 2, 64, 200, 64, False, False, f16,
                 (32, 32, 64), 7)
    strided_case("basic_fp32_causal", "_flash_attn_fwd_kernel_basic", 1, 2, 100, 100, 128, True, True, f32,
                 (32, 32, 128), 8)
    nomask_case("nomask_d128", 1, 2, 2, 128, 128, 64, 64, f16, 9)
    nomask_case("nomask_d256", 1, 1, 1, 128, 256, 32, 64, f16, 10)
    nomask_case("gqa_d128", 1, 4, 2, 128, 128, 128, 64, f16, 11)
    mma_case("mma_128x64x128", 128, 64, 128, f16, 12)
    mma_case("mma_256x96x192", 256, 96, 192, f16, 13)

    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps({"generator": "tests/golden/make_golden.py",
                                                  "source": "reference Triton kernels under TRITON_INTERPRET=1",
                                                  "cases": cases}, indent=1) + "\n")
    print(f"wrote {len(cases)} cases, {sum(a.nbytes for a in arrays.values())} bytes of arrays")


if __name__ == "__main__":
    main()
