"""CPU oracle for the matmul -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

* `tiled_matmul`: numpy restatement of the reference's Triton GEMM
  (mma.py:8-52): fp32 accumulation over K in BLOCK_K slices
  (mma.py:39-49), accumulator rounded to fp16 for the store (mma.py:51-52),
  then to the output dtype.
* `matmul_reference`: the reference's oracle, torch.matmul on CPU
  (test_mma.py:260-261, 296-297).
"""
from __future__ import annotations

import numpy as np

from oracle.rounding import round_to


def tiled_matmul(a: np.ndarray, b: np.ndarray, *, block_k: int = 32, round_f16: bool = True, out_dtype: str = "fp16"):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError("inner dimensions differ")
    acc = np.zeros((M, N), dtype=np.float32)
    for k0 in range(0, K, block_k):
        acc += a[:, k0:k0 + block_k] @ b[k0:k0 + block_k]
    if round_f16:
        acc = round_to(acc, "fp16")
    return round_to(acc, out_dtype)


def matmul_reference(a, b, *, dtype: str = "fp16"):
    """torch.matmul on CPU in the input dtype (the reference compares in fp16)."""
    import torch

    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    at = torch.as_tensor(np.asarray(a, dtype=np.float32)).to(tdt)
    bt = torch.as_tensor(np.asarray(b, dtype=np.float32)).to(tdt)
    return torch.matmul(at, bt).float().numpy()


def matmul_flops(M: int, N: int, K: int) -> float:
    """2*M*K*N (test_mma.py:78-83)."""
    return 2.0 * M * N * K
