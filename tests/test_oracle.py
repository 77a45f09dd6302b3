"""The CPU oracle against the reference's own outputs (golden vectors) and torch.

The golden vectors in tests/golden/ were produced by the reference's Triton
kernels running in Triton's CPU interpreter (tests/golden/make_golden.py), so
these tests pin the oracle to the reference itself before any GPU result is
compared with the oracle.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.fa_oracle import attention_flops, sdpa_reference, tiled_attention_forward
from oracle.mma_oracle import matmul_flops, matmul_reference, tiled_matmul
from oracle.rounding import round_to_bf16, round_to_fp16

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = json.loads((GOLDEN / "golden.json").read_text())["cases"]
ARRAYS = np.load(GOLDEN / "golden.npz")


def _arr(case, key):
    return ARRAYS[f"{case['name']}.{key}"].astype(np.float32)


ATT = [c for c in CASES if c["kind"] == "attention"]
MMA = [c for c in CASES if c["kind"] == "matmul"]


def test_golden_inventory():
    names = {c["name"] for c in CASES}
    assert "cfg1_fp32" in names  # the fp32 benchmark case exactly (B1 H4 S256 D64)
    assert any(c["causal"] for c in ATT) and any(c["Hkv"] < c["Hq"] for c in ATT)
    assert {c["kernel"] for c in ATT} == {
        "_flash_attn_fwd_kernel_basic",
        "_flash_attn_fwd_kernel_optimize_shared_mem",
        "_flash_attn_fwd_kernel_block_d_nomask_contiguous",
    }
    assert len(MMA) >= 2


@pytest.mark.parametrize("case", ATT, ids=lambda c: c["name"])
def test_oracle_matches_reference_attention(case):
    q, k, v = _arr(case, "q"), _arr(case, "k"), _arr(case, "v")
    p_dtype = "fp16" if case["dtype"] == "float16" else "fp32"
    bm, bn = case["blocks"][0], case["blocks"][1]
    o, lse = tiled_attention_forward(q, k, v, sm_scale=case["sm_scale"], causal=case["causal"], p_dtype=p_dtype,
                                     block_m=bm, block_n=bn)
    ref_o = _arr(case, "o")
    if case["dtype"] == "float16":
        o = round_to_fp16(o)
        np.testing.assert_allclose(o, ref_o, rtol=2e-3, atol=2e-3)
    else:
        np.testing.assert_allclose(o, ref_o, rtol=1e-4, atol=1e-5)
    if case["has_lse"]:
        np.testing.assert_allclose(lse, _arr(case, "lse"), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", ATT, ids=lambda c: c["name"])
def test_reference_outputs_match_sdpa(case):
    """The reference itself agrees with its own oracle (CPU fp32 SDPA) at its own tolerance."""
    q, k, v = _arr(case, "q"), _arr(case, "k"), _arr(case, "v")
    o, lse = sdpa_reference(q, k, v, causal=case["causal"], sm_scale=case["sm_scale"])
    np.testing.assert_allclose(_arr(case, "o"), o, rtol=1e-2, atol=2e-2)
    if case["has_lse"]:
        np.testing.assert_allclose(_arr(case, "lse"), lse, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("case", MMA, ids=lambda c: c["name"])
def test_oracle_matches_reference_matmul(case):
    a, b = _arr(case, "a"), _arr(case, "b")
    c = tiled_matmul(a, b, block_k=case["blocks"][2], round_f16=True, out_dtype="fp16")
    ref = _arr(case, "c")
    # Same fp32 sums in a different order: at most one fp16 ulp apart.
    np.testing.assert_allclose(c, ref, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(matmul_reference(a, b), ref, rtol=0.2, atol=0.2)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(1, 2, 2, 33, 70, 64), (2, 4, 1, 65, 65, 32), (1, 3, 3, 5, 300, 128)])
def test_oracle_matches_sdpa_fp32(shape, causal):
    B, Hq, Hkv, M, N, D = shape
    rng = np.random.default_rng(7)
    q = rng.standard_normal((B, Hq, M, D), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, N, D), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, N, D), dtype=np.float32)
    o, lse = tiled_attention_forward(q, k, v, causal=causal, block_m=16, block_n=32)
    ro, rl = sdpa_reference(q, k, v, causal=causal)
    np.testing.assert_allclose(o, ro, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse, rl, rtol=1e-5, atol=1e-5)


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(3)
    x = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * 10,
        # exact ties between two bf16 values (lower 16 bits = 0x8000)
        (np.arange(1, 2000, dtype=np.uint32) << 16 | 0x8000).view(np.float32),
        np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38, -3.4e38, 1e-40], dtype=np.float32),
    ])
    ours = round_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(ours, ref)
    assert np.isnan(round_to_bf16(np.array([np.nan], dtype=np.float32)))[0]


def test_fp16_rounding_matches_torch():
    rng = np.random.default_rng(4)
    x = rng.standard_normal(100000).astype(np.float32) * 100
    np.testing.assert_array_equal(round_to_fp16(x), torch.from_numpy(x).half().float().numpy())


def test_flop_formulas_follow_reference():
    # test_flash_atten.py:234-240 (square) and test_mma.py:78-83
    assert attention_flops(4, 32, 8192, 8192, 128, False) == 4 * 4 * 32 * 128 * 8192 * 8192
    assert attention_flops(1, 1, 10, 10, 8, True) == 4 * 8 * (10 * 11 / 2)
    assert matmul_flops(16384, 16384, 16384) == 2 * 16384 ** 3
