"""Attention forward on the GPU, through the C ABI, against the reference and the oracle.

Tolerance (the acceptance bar for 16-bit outputs): fp16/bf16 outputs within max-abs 2e-2 and
rtol 1e-2 of an fp32 reference on the same inputs; the LSE is compared in
fp32 (atol 2e-3).  fp32 inputs run on the tensor cores as tf32, like the
reference's Triton `tl.dot` default, under the same tolerance.
"""
from __future__ import annotations

import json
import zlib
from math import log as math_log
from pathlib import Path

import numpy as np
import pytest
import torch

import _native
import flash_atten
from flash_atten import attention_forward, flash_attention
from oracle.fa_oracle import tiled_attention_forward
from tuner import (
    FlashAttenTuneArguments,
    FlashAttentionBlockDNomaskTuner,
    FlashAttentionOptimizeSharedMemTuner,
    FlashAttentionTuner,
)

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
LSE_ATOL = 2e-3
GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = json.loads((GOLDEN / "golden.json").read_text())["cases"]
ARRAYS = np.load(GOLDEN / "golden.npz")
P_DTYPE = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _close(actual: torch.Tensor, expected, rtol=RTOL, atol=ATOL):
    expected = torch.as_tensor(np.asarray(expected, dtype=np.float32))
    torch.testing.assert_close(actual.detach().float().cpu(), expected, rtol=rtol, atol=atol)


def _inputs(shape, dtype, seed, dev):
    B, Hq, Hkv, M, N, D = shape
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, M, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    return q, k, v, q.to(dev), k.to(dev), v.to(dev)


def _oracle(q, k, v, causal, dtype, sm_scale=None):
    return tiled_attention_forward(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                                   p_dtype=P_DTYPE[dtype], sm_scale=sm_scale)


# ------------------------------------------------------------ golden vectors
ATT = [c for c in CASES if c["kind"] == "attention"]


@pytest.mark.parametrize("case", ATT, ids=lambda c: c["name"])
def test_reference_golden_through_dropin(case, cuda_device):
    """The reference's own outputs, reproduced through the same entry point the reference case used."""
    g = lambda key: torch.from_numpy(ARRAYS[f"{case['name']}.{key}"])  # noqa: E731
    q, k, v = (g(x).to(cuda_device) for x in ("q", "k", "v"))
    ref_o = ARRAYS[f"{case['name']}.o"]
    if case["Hkv"] != case["Hq"]:
        o = attention_forward(q, k, v, causal=case["causal"], sm_scale=case["sm_scale"])
        _close(o, ref_o)
        return
    tuner_cls = {
        "_flash_attn_fwd_kernel_basic": FlashAttentionTuner,
        "_flash_attn_fwd_kernel_optimize_shared_mem": FlashAttentionOptimizeSharedMemTuner,
        "_flash_attn_fwd_kernel_block_d_nomask_contiguous": FlashAttentionBlockDNomaskTuner,
    }[case["kernel"]]
    spec = tuner_cls(tuple(q.shape), tuple(k.shape), tuple(v.shape), q.element_size(), causal=case["causal"],
                     return_lse=case["has_lse"]).build_flash_attention_launch_spec(q, k, v, sm_scale=case["sm_scale"])
    out = flash_attention(spec)
    if case["has_lse"]:
        o, lse = out
        _close(lse, ARRAYS[f"{case['name']}.lse"], rtol=1e-4, atol=LSE_ATOL)
    else:
        o = out
    assert o.dtype == q.dtype and tuple(o.shape) == tuple(q.shape)
    _close(o, ref_o)


def test_config1_exact_baseline_case(cuda_device):
    """The fp32 benchmark case: B1 H4 S256 D64 fp32 N(0,1) from seed 0, scale 1/8, vs torch SDPA math on CPU."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, 256, 64, generator=g) for _ in range(3))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=0.125)
    spec = FlashAttentionTuner(tuple(q.shape), tuple(k.shape), tuple(v.shape), 4, causal=False,
                               return_lse=False).build_flash_attention_launch_spec(
        q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), sm_scale=0.125)
    _close(flash_attention(spec), ref.numpy())


# --------------------------------------------------------- oracle parity sweep
SHAPES = [
    (1, 2, 2, 128, 128, 64),
    (1, 2, 2, 257, 300, 64),
    (2, 2, 2, 384, 200, 128),
    (1, 3, 3, 1, 77, 128),
    (1, 2, 2, 129, 513, 128),
    (1, 2, 2, 200, 190, 256),
    (1, 2, 2, 65, 257, 256),
    (1, 2, 2, 100, 33, 80),
    (1, 1, 1, 33, 45, 16),
]


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}H{}/{}M{}N{}D{}".format(*s))
def test_oracle_parity_16bit(shape, dtype, causal, cuda_device):
    q, k, v, qd, kd, vd = _inputs(shape, dtype, seed=zlib.crc32(repr((shape, str(dtype), causal)).encode()),
                                  dev=cuda_device)
    o, lse = attention_forward(qd, kd, vd, causal=causal, return_lse=True)
    ro, rl = _oracle(q, k, v, causal, dtype)
    _close(o, ro)
    _close(lse, rl, rtol=1e-4, atol=LSE_ATOL)


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("shape", [(1, 4, 4, 256, 256, 64), (1, 2, 2, 150, 130, 128), (1, 2, 2, 70, 99, 32),
                                   (2, 2, 1, 129, 200, 100)], ids=lambda s: "B{}H{}/{}M{}N{}D{}".format(*s))
def test_oracle_parity_fp32_tf32(shape, causal, cuda_device):
    q, k, v, qd, kd, vd = _inputs(shape, torch.float32, seed=11, dev=cuda_device)
    o, lse = attention_forward(qd, kd, vd, causal=causal, return_lse=True)
    ro, rl = _oracle(q, k, v, causal, torch.float32)
    _close(o, ro)
    _close(lse, rl, rtol=1e-3, atol=1e-2)


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
def test_grouped_query_heads(causal, cuda_device):
    """The GQA benchmark shape (16 query heads over 4 KV heads, D=128), shortened sequence."""
    shape = (2, 16, 4, 640, 640, 128)
    q, k, v, qd, kd, vd = _inputs(shape, torch.bfloat16, seed=5, dev=cuda_device)
    o = attention_forward(qd, kd, vd, causal=causal)
    ro, _ = _oracle(q, k, v, causal, torch.bfloat16)
    _close(o, ro)


def test_strided_inputs_through_basic_launcher(cuda_device):
    """Non-contiguous q/k/v/o ([B,S,H,D] storage viewed as [B,H,S,D]) with explicit strides, as the
    reference's basic kernel accepts (flash_atten.py:21-39)."""
    B, H, S, D = 2, 3, 200, 64
    g = torch.Generator().manual_seed(3)
    qs, ks, vs = (torch.randn(B, S, H, D, generator=g).half().to(cuda_device) for _ in range(3))
    q, k, v = (t.transpose(1, 2) for t in (qs, ks, vs))
    o = torch.empty(B, S, H, D, dtype=torch.float16, device=cuda_device).transpose(1, 2)
    lse = torch.empty(B, H, S, dtype=torch.float32, device=cuda_device)
    args = (q, k, v, o, lse, *q.stride(), *k.stride(), *v.stride(), *o.stride(), *lse.stride(), H, S, S, D, D ** -0.5)
    flash_atten._flash_attn_fwd_kernel_basic[(2, B * H)](*args, causal=True, HAS_LSE=True, BLOCK_M=128, BLOCK_N=64,
                                                         BLOCK_N_PAD=64, BLOCK_DMODEL=64, num_warps=8, num_stages=1)
    ro, rl = _oracle(q.cpu(), k.cpu(), v.cpu(), True, torch.float16)
    _close(o, ro)
    _close(lse, rl, rtol=1e-4, atol=LSE_ATOL)


def test_unaligned_rows_and_offsets(cuda_device):
    """Head dim whose rows are not 16-byte multiples, and a storage offset that breaks 16-byte alignment."""
    q, k, v, qd, kd, vd = _inputs((1, 2, 2, 50, 70, 20), torch.float16, seed=8, dev=cuda_device)
    o = attention_forward(qd, kd, vd, causal=True)
    ro, _ = _oracle(q, k, v, True, torch.float16)
    _close(o, ro)
    base = torch.randn(1 + 2 * 64 * 64, dtype=torch.bfloat16, device=cuda_device)
    qo = base[1:].view(1, 2, 64, 64)  # data_ptr is 2 bytes past an aligned boundary
    o2 = attention_forward(qo, qo, qo)
    ro2, _ = _oracle(qo.cpu(), qo.cpu(), qo.cpu(), False, torch.bfloat16)
    _close(o2, ro2)


def test_contiguous_launcher_with_reference_tune_args(cuda_device):
    """The TTFT preset of the sliced kernel (ttft.py:145-166) on a non-tile-multiple sequence."""
    q, k, v, qd, kd, vd = _inputs((1, 4, 4, 300, 300, 128), torch.float16, seed=9, dev=cuda_device)
    tune = FlashAttenTuneArguments(BLOCK_N=64, BLOCK_M=128, BLOCK_N_PAD=64, BLOCK_DMODEL=128, BLOCK_DMODEL_OUTER=64,
                                   NUM_WARPS=8, NUM_STAGES=3)
    spec = FlashAttentionBlockDNomaskTuner(tuple(qd.shape), tuple(kd.shape), tuple(vd.shape), 2, causal=False,
                                           return_lse=False, tune_args=tune).build_flash_attention_launch_spec(qd, kd, vd)
    o = flash_attention(spec)
    ro, _ = _oracle(q, k, v, False, torch.float16)
    _close(o, ro)
    # update_data: same spec, new inputs, same output buffer
    q2, k2, v2, q2d, k2d, v2d = _inputs((1, 4, 4, 300, 300, 128), torch.float16, seed=10, dev=cuda_device)
    spec.update_data((q2d, k2d, v2d))
    o2 = flash_attention(spec)
    assert o2.data_ptr() == o.data_ptr()
    _close(o2, _oracle(q2, k2, v2, False, torch.float16)[0])


@pytest.mark.parametrize("scale", [-0.2, 0.0, 1.5])
def test_scale_variants(scale, cuda_device):
    q, k, v, qd, kd, vd = _inputs((1, 2, 2, 130, 140, 64), torch.bfloat16, seed=12, dev=cuda_device)
    o = attention_forward(qd, kd, vd, causal=True, sm_scale=scale)
    ro, _ = _oracle(q, k, v, True, torch.bfloat16, sm_scale=scale)
    _close(o, ro)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_dominant_key_at_every_tile_column(D, cuda_device):
    """One key per head scores so far above the rest that exp of it overflows fp32 unless the row maximum
    saw it; the heads place it at the first, middle and last columns of the first and second key tiles."""
    positions = [0, 7, 63, 64, 119, 120, 127, 128, 191, 248, 255]
    H, M, N = len(positions), 128, 256
    g = torch.Generator().manual_seed(21)
    q = torch.full((1, H, M, D), 4.0).to(torch.bfloat16)
    k = (0.1 * torch.randn(1, H, N, D, generator=g)).to(torch.bfloat16)
    v = torch.randn(1, H, N, D, generator=g).to(torch.bfloat16)
    for h, pos in enumerate(positions):
        k[0, h, pos] = 8.0
    o = attention_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    ro, _ = _oracle(q, k, v, False, torch.bfloat16)
    assert torch.isfinite(o.float()).all()
    _close(o, ro)


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_row_max_rising_every_key_tile(D, causal, cuda_device):
    """Scores grow by about 2^9 from one 64-key block to the next, so the running max moves on every KV
    tile and the kernel takes its rescale path each time."""
    M, N = 256, 1024
    g = torch.Generator().manual_seed(22)
    q = (1.0 + 0.05 * torch.randn(1, 2, M, D, generator=g)).to(torch.bfloat16)
    step = 9.0 * math_log(2.0) / (D ** 0.5)  # log2 gain of 9 per block at scale D^-0.5
    ramp = (torch.arange(N) // 64).float() * step
    k = (ramp[None, None, :, None] + 0.05 * torch.randn(1, 2, N, D, generator=g)).to(torch.bfloat16)
    v = torch.randn(1, 2, N, D, generator=g).to(torch.bfloat16)
    o, lse = attention_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=causal,
                               return_lse=True)
    ro, rl = _oracle(q, k, v, causal, torch.bfloat16)
    assert torch.isfinite(o.float()).all()
    _close(o, ro)
    _close(lse, rl, rtol=1e-3, atol=2e-3 * max(1.0, float(np.abs(rl).max()) / 100))


def test_empty_inputs(cuda_device):
    q = torch.randn(1, 2, 5, 64, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(1, 2, 0, 64, device=cuda_device, dtype=torch.bfloat16)
    o, lse = attention_forward(q, k, k, return_lse=True)
    assert torch.isnan(o.float()).all()  # 0/0, as the reference's acc / l_i with no keys
    assert torch.isneginf(lse).all()
    q0 = torch.randn(1, 2, 0, 64, device=cuda_device, dtype=torch.bfloat16)
    kk = torch.randn(1, 2, 7, 64, device=cuda_device, dtype=torch.bfloat16)
    assert attention_forward(q0, kk, kk).shape == (1, 2, 0, 64)


def test_deterministic(cuda_device):
    _, _, _, qd, kd, vd = _inputs((2, 4, 4, 700, 700, 128), torch.bfloat16, seed=13, dev=cuda_device)
    a = attention_forward(qd, kd, vd, causal=True)
    b = attention_forward(qd, kd, vd, causal=True)
    assert torch.equal(a, b)


def test_unsupported_head_dim_raises(cuda_device):
    x = torch.randn(1, 1, 8, 512, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        attention_forward(x, x, x)


# ------------------------------------------------------ full benchmark sizes
def _sampled_rows_check(q, k, v, o, causal, dtype, picks):
    """Oracle on selected (b, h, row-block) slices of a full-size problem."""
    for b, h, m0, m1 in picks:
        hk = h // (q.shape[1] // k.shape[1])
        n_end = min(k.shape[2], m1) if causal else k.shape[2]
        qs = q[b:b + 1, h:h + 1, m0:m1].float().cpu()
        ks = k[b:b + 1, hk:hk + 1, :n_end].float().cpu()
        vs = v[b:b + 1, hk:hk + 1, :n_end].float().cpu()
        ro, _ = tiled_attention_forward(qs.numpy(), ks.numpy(), vs.numpy(), causal=causal, p_dtype=P_DTYPE[dtype],
                                        block_m=128, block_n=512, q_row_offset=m0)
        _close(o[b, h, m0:m1], ro[0, 0])


def _spread_picks(B, H, S):
    """First, middle, last and one unaligned row block, on different (batch, head) pairs."""
    mid = S // 2
    return [(0, 0, 0, 128), (B // 2, H // 2, mid, mid + 128), (B - 1, H - 1, S - 128, S),
            (B - 1, H // 3, S // 3 + 5, S // 3 + 105)]


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("S", [1024, 2048, 4096, 8192])
def test_config2_full_size_sampled(S, causal, cuda_device):
    """BASELINE config 2 at every sequence length: B4 H32 D128 bf16 through attention_forward, whose
    measured tile-family choice switches kernels across these lengths; rows sampled across heads."""
    B, H, D = 4, 32, 128
    g = torch.Generator(device=cuda_device).manual_seed(21 + S)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=cuda_device, dtype=torch.bfloat16) for _ in range(3))
    o = attention_forward(q, k, v, causal=causal)
    assert not torch.isnan(o).any()
    picks = _spread_picks(B, H, S) + ([(1, 17, 4096, 4224), (2, 5, 1000, 1100)] if S == 8192 else [])
    _sampled_rows_check(q, k, v, o, causal, torch.bfloat16, picks)


@pytest.mark.parametrize("S", [2048, 4096, 8192])
def test_config3_d256_full_size_sampled(S, cuda_device):
    """BASELINE config 3, D=256: B2 H16 bf16, causal, scale 1/16, at every sequence length."""
    B, H, D = 2, 16, 256
    g = torch.Generator(device=cuda_device).manual_seed(22 + S)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=cuda_device, dtype=torch.bfloat16) for _ in range(3))
    o = attention_forward(q, k, v, causal=True, sm_scale=1 / 16)
    assert not torch.isnan(o).any()
    _sampled_rows_check(q, k, v, o, True, torch.bfloat16, _spread_picks(B, H, S))


@pytest.mark.parametrize("S", [16384, 32768, 65536])
@pytest.mark.parametrize("H, D", [(28, 128), (16, 256)], ids=["H28D128", "H16D256"])
def test_reference_large_cases_sampled(H, D, S, cuda_device):
    """The reference's long-sequence pipeline cases (test_flash_atten.py:82-88: B1, H28 D128 and H16 D256,
    non-causal, asserted at rtol 1e-2 / atol 2e-2, :489-495) at S 16K-64K: 32-bit offsets and long
    online-softmax accumulation.  First and last row blocks included."""
    g = torch.Generator(device=cuda_device).manual_seed(S + D)
    q, k, v = (torch.randn(1, H, S, D, generator=g, device=cuda_device, dtype=torch.bfloat16) for _ in range(3))
    o = attention_forward(q, k, v)
    assert not torch.isnan(o).any()
    picks = [(0, 0, 0, 128), (0, H // 2, S // 2 - 64, S // 2 + 64), (0, H - 1, S - 128, S)]
    _sampled_rows_check(q, k, v, o, False, torch.bfloat16, picks)


# ------------------------------------------- the two-CTAs-per-SM one-tile kernel
DUAL_CASES = [
    # (B, Hq, Hkv, S, D, dtype, causal)
    (4, 32, 32, 1024, 128, torch.bfloat16, False),
    (4, 32, 32, 1024, 128, torch.bfloat16, True),
    (4, 32, 32, 2048, 128, torch.bfloat16, False),
    (4, 32, 32, 2048, 128, torch.bfloat16, True),
    (4, 32, 32, 1024, 128, torch.float16, True),
    (4, 32, 32, 2048, 128, torch.float16, False),
    (4, 32, 32, 1024, 64, torch.float16, False),
    (4, 32, 32, 1024, 64, torch.float16, True),
    (4, 32, 32, 2048, 64, torch.bfloat16, True),
    (4, 32, 32, 1024, 64, torch.float32, False),
    (4, 32, 32, 1024, 64, torch.float32, True),
    (1, 28, 4, 2048, 128, torch.bfloat16, True),  # the TTFT prefill: Qwen2.5-7B heads at 2048 tokens
]


@pytest.mark.parametrize("case", DUAL_CASES,
                         ids=lambda c: "B{}H{}/{}S{}D{}-{}-{}".format(*c[:5], P_DTYPE[c[5]],
                                                                      "causal" if c[6] else "full"))
def test_two_ctas_per_sm_kernel_matches_oracle(case, cuda_device):
    """The one-tile, one-S-buffer kernel that two CTAs share an SM with (the measured choice for causal
    S <= 2048 and for the TTFT prefill).  It runs only with at least 1.5 CTAs per SM, so the grid here is
    asserted to be that large; rows are checked against the oracle at the normal tolerance, LSE too."""
    B, Hq, Hkv, S, D, dtype, causal = case
    q, k, v, qd, kd, vd = _inputs((B, Hq, Hkv, S, S, D), dtype, seed=zlib.crc32(repr(case).encode()), dev=cuda_device)
    plan = flash_atten.attention_plan(qd, kd, vd, causal=causal, variant=1)
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    assert plan["ctas_per_sm"] == 2 and plan["s_buffers"] == 1 and plan["q_tiles_per_cta"] == 1
    assert 2 * plan["ctas"] >= 3 * sms, plan
    o = torch.empty_like(qd)
    lse = torch.empty(B, Hq, S, device=cuda_device, dtype=torch.float32)
    flash_atten._launch_attention(qd, kd, vd, o, lse, causal=causal, sm_scale=D ** -0.5, what="test", variant=1)
    torch.cuda.synchronize()
    assert not torch.isnan(o).any()
    tf32 = dtype == torch.float32
    for b, h, m0, m1 in _spread_picks(B, Hq, S):
        hk = h // (Hq // Hkv)
        n_end = min(S, m1) if causal else S
        ro, rl = tiled_attention_forward(q[b:b + 1, h:h + 1, m0:m1].float().numpy(),
                                         k[b:b + 1, hk:hk + 1, :n_end].float().numpy(),
                                         v[b:b + 1, hk:hk + 1, :n_end].float().numpy(), causal=causal,
                                         p_dtype=P_DTYPE[dtype], block_m=128, block_n=512, q_row_offset=m0)
        _close(o[b, h, m0:m1], ro[0, 0])
        _close(lse[b, h, m0:m1], rl[0, 0], rtol=1e-3 if tf32 else 1e-4, atol=1e-2 if tf32 else LSE_ATOL)


def test_measured_choice_takes_two_ctas_per_sm_for_short_causal(cuda_device):
    """attention_forward's measured family choice for BASELINE config 2 causal S1024/S2048 is the
    two-CTAs-per-SM kernel, so the parity cases above cover what those calls run.  (The TTFT prefill's
    28 heads at 2048 take the two-tile kernel; the forced-variant case above covers the other.)"""
    for B, Hq, Hkv, S in ((4, 32, 32, 1024), (4, 32, 32, 2048)):
        q = torch.empty(B, Hq, S, 128, device=cuda_device, dtype=torch.bfloat16)
        kv = torch.empty(B, Hkv, S, 128, device=cuda_device, dtype=torch.bfloat16)
        plan = flash_atten.attention_plan(q, kv, kv, causal=True)
        assert plan["variant"] == 1 and plan["ctas_per_sm"] == 2, (B, Hq, Hkv, S, plan)


def test_config3_gqa_full_size_sampled(cuda_device):
    """The GQA benchmark shape: 16 query heads over 4 KV heads, D=128, S=8192, causal."""
    B, Hq, Hkv, S, D = 2, 16, 4, 8192, 128
    g = torch.Generator(device=cuda_device).manual_seed(23)
    q = torch.randn(B, Hq, S, D, generator=g, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g, device=cuda_device, dtype=torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g, device=cuda_device, dtype=torch.bfloat16)
    o = attention_forward(q, k, v, causal=True)
    _sampled_rows_check(q, k, v, o, True, torch.bfloat16, [(0, 3, 0, 128), (1, 12, 6000, 6128), (1, 15, 8064, 8192)])


# ----------------------------------------------- the second compiled tile family
@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("shape, dtype", [((1, 2, 2, 257, 300, 64), torch.bfloat16),
                                          ((2, 4, 2, 384, 200, 128), torch.float16),
                                          ((1, 2, 2, 129, 513, 128), torch.bfloat16),
                                          ((1, 2, 2, 150, 130, 64), torch.float32),
                                          ((1, 2, 2, 100, 33, 80), torch.bfloat16)],
                         ids=lambda x: "B{}H{}/{}M{}N{}D{}".format(*x) if isinstance(x, tuple) else str(x)[6:])
def test_one_tile_family_matches_oracle(shape, dtype, causal, cuda_device):
    """FAB_FA_VARIANT_ONE_TILE (one query tile, two S buffers) through the reference-named launcher."""
    q, k, v, qd, kd, vd = _inputs(shape, dtype, seed=zlib.crc32(repr(("one", shape, str(dtype), causal)).encode()),
                                  dev=cuda_device)
    B, Hq, M, D = q.shape
    o = torch.empty_like(qd)
    lse = torch.empty(B, Hq, M, device=cuda_device, dtype=torch.float32)
    if Hq == k.shape[1]:
        args = (qd, kd, vd, o, lse, *qd.stride(), *kd.stride(), *vd.stride(), *o.stride(), *lse.stride(), Hq, M,
                k.shape[2], D, D ** -0.5)
        flash_atten._flash_attn_fwd_kernel_basic[(1, B * Hq)](*args, causal=causal, HAS_LSE=True, sm100_variant=1)
    else:
        flash_atten._launch_attention(qd, kd, vd, o, lse, causal=causal, sm_scale=D ** -0.5, what="test", variant=1)
    ro, rl = _oracle(q, k, v, causal, dtype)
    _close(o, ro)
    _close(lse, rl, rtol=1e-3 if dtype == torch.float32 else 1e-4, atol=1e-2 if dtype == torch.float32 else LSE_ATOL)


def test_tuner_times_both_families(cuda_device):
    """tune_by_time=True measures the compiled families on the caller's tensors and launches the faster."""
    _, _, _, qd, kd, vd = _inputs((1, 4, 4, 512, 512, 128), torch.bfloat16, seed=61, dev=cuda_device)
    spec = FlashAttentionTuner(tuple(qd.shape), tuple(kd.shape), tuple(vd.shape), 2, causal=True, return_lse=False,
                               tune_by_time=True).build_flash_attention_launch_spec(qd, kd, vd)
    assert spec.kernel_kwargs["sm100_variant"] in (0, 1)
    assert spec.tune_args.BLOCK_M == (256 if spec.kernel_kwargs["sm100_variant"] == 0 else 128)
    o = flash_attention(spec)
    ro, _ = _oracle(qd.cpu(), kd.cpu(), vd.cpu(), True, torch.bfloat16)
    _close(o, ro)


# ------------------------------------------------------------ host-buffer entry point
@pytest.mark.parametrize("shape, chunks", [((2, 4, 4, 300, 300, 64), 16), ((1, 8, 2, 257, 513, 128), 3),
                                           ((3, 6, 3, 128, 1000, 128), 1), ((2, 4, 2, 200, 200, 256), 64)],
                         ids=["mha", "gqa", "one_piece", "d256"])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_host_entry_equals_device_call(shape, chunks, causal, cuda_device):
    """attention_forward_host on host tensors, pipelined in pieces, returns attention_forward's bits."""
    q, k, v, qd, kd, vd = _inputs(shape, torch.bfloat16, seed=sum(shape) + chunks, dev=cuda_device)
    want = attention_forward(qd, kd, vd, causal=causal).cpu()
    qp, kp, vp = q.pin_memory(), k.pin_memory(), v.pin_memory()
    got = flash_atten.attention_forward_host(qp, kp, vp, causal=causal, chunks=chunks, device=cuda_device)
    assert got.device.type == "cpu" and got.is_pinned()
    assert torch.equal(got, want)
    # caller-supplied output, pageable inputs, sm_scale passed through
    out = torch.full_like(q, 7.0)
    flash_atten.attention_forward_host(q, k, v, causal=causal, sm_scale=0.05, out=out, chunks=chunks,
                                       device=cuda_device)
    assert torch.equal(out, attention_forward(qd, kd, vd, causal=causal, sm_scale=0.05).cpu())


def test_host_entry_fp32_and_oracle(cuda_device):
    q, k, v, _, _, _ = _inputs((2, 2, 1, 192, 320, 64), torch.float32, seed=5, dev=cuda_device)
    got = flash_atten.attention_forward_host(q, k, v, causal=True, chunks=4, device=cuda_device)
    _close(got, _oracle(q, k, v, True, torch.float32)[0])
