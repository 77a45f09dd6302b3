"""RMSNorm folded into the GEMM after it (fab_gemm_params.row_scale + fab_rmsnorm_rstd).

The decoder's input and post-attention norms feed the QKV and gate/up projections (the steps on either side
of the attention call in the reference's forward, ttft.py:401-412).  Folded, a stats pass writes each row's
1/rms, the norm weight is multiplied into the GEMM's B once, and the GEMM scales row r by rstd[r] before its
epilogue.  The normalised activations are never written.  This changes where rounding happens, so the
folded results are not bit-identical to the unfused bf16 expressions.  They are judged against an fp32
reference of the same expression: the folded path's error must be no larger than the unfused bf16 path's
own error (which rounds h, every GEMM output and every RoPE/SwiGLU step in bf16, exactly as the PyTorch
model does) -- max error within 1.5x and mean error within 1.25x of it.  The plain row-scaled GEMM is
checked at the north-star tolerance (max-abs 2e-2, rtol 1e-2); the stats pass is exact.
"""
from __future__ import annotations

import pytest
import torch

import _native
import mma
import ttft
from mma import fold_rmsnorm_weight, matmul_bias_rope, matmul_swiglu

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
EPS = 1e-6


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def _rms_norm_torch(x, w):
    """The Qwen2 RMSNorm expression (HF): fp32 statistics, rounded to x's dtype, times the weight."""
    xf = x.float()
    return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)).to(x.dtype)


def _tables(S, D, device, dtype):
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    emb = torch.outer(torch.arange(S, device=device, dtype=torch.float32), inv)
    emb = torch.cat([emb, emb], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _no_worse(folded, unfused, ref32):
    """The folded path's error against the fp32 reference is no worse than the unfused bf16 path's."""
    ef = (folded.float() - ref32).abs()
    eu = (unfused.float() - ref32).abs()
    assert float(ef.max()) <= 1.5 * float(eu.max()) + 1e-3, (float(ef.max()), float(eu.max()))
    assert float(ef.mean()) <= 1.25 * float(eu.mean()) + 1e-5, (float(ef.mean()), float(eu.mean()))


def _inputs(S, K, N, device, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(S, K, generator=g, device=device).to(dtype)
    res = torch.randn(S, K, generator=g, device=device).to(dtype)
    ln = (1.0 + 0.2 * torch.randn(K, generator=g, device=device)).to(dtype)
    w = (0.02 * torch.randn(K, N, generator=g, device=device)).to(dtype)
    return x, res, ln, w


@pytest.mark.parametrize("rows, cols, with_res", [(2048, 3584, True), (77, 3584, False), (5, 512, True)])
def test_rstd_pass_matches_the_norm_statistics(rows, cols, with_res, cuda_device):
    x, res, ln, _ = _inputs(rows, cols, 8, cuda_device, seed=rows + cols)
    x1, x2 = x.clone(), x.clone()
    h = ttft._native_rmsnorm(x1, ln, EPS, residual=res if with_res else None)
    rstd = ttft._native_rmsnorm_rstd(x2, EPS, residual=res if with_res else None)
    assert torch.equal(x1, x2)  # the residual update is the same pass
    xf = x2.float()
    want = torch.rsqrt(xf.pow(2).mean(-1) + EPS)
    torch.testing.assert_close(rstd, want, rtol=2e-6, atol=0)
    # the unfused norm's output is the rounded product of the same statistics
    want_h = (ln.float() * (xf * rstd[:, None]).to(x.dtype).float()).to(x.dtype)
    assert torch.equal(h, want_h)


def test_row_scale_plain_store(cuda_device):
    S, K, N = 300, 1024, 768
    x, _, _, w = _inputs(S, K, N, cuda_device, seed=5)
    rs = torch.rand(S, device=cuda_device) + 0.5
    c = torch.empty(S, N, device=cuda_device, dtype=torch.bfloat16)
    mma._gemm(x, w, c, S, N, K, lda=K, ldb=N, ldc=N, round_f16=False, row_scale=rs)
    want = rs[:, None] * (x.float() @ w.float())
    torch.testing.assert_close(c.float(), want, rtol=RTOL, atol=ATOL)
    # without a scale the same call is the plain GEMM, bit for bit
    c2 = torch.empty_like(c)
    mma._gemm(x, w, c2, S, N, K, lda=K, ldb=N, ldc=N, round_f16=False)
    assert torch.equal(c2, mma.matmul(x, w))


@pytest.mark.parametrize("S", [2048, 300])
def test_folded_qkv_projection_matches_pytorch(S, cuda_device):
    """Residual add + input RMSNorm + QKV GEMM + bias + RoPE: folded form against the PyTorch expressions."""
    K, nq, nkv, D = 3584, 28, 4, 128
    N = (nq + 2 * nkv) * D
    x, res, ln, w = _inputs(S, K, N, cuda_device, seed=S)
    g = torch.Generator(device=cuda_device).manual_seed(9)
    bias = (0.1 * torch.randn(N, generator=g, device=cuda_device)).to(torch.bfloat16)
    cos, sin = _tables(S, D, cuda_device, torch.bfloat16)
    # fp32 reference of x' = x + res; h = RMSNorm(x'); qkv = h @ W + b; RoPE on q and k
    xr = x + res
    xf = xr.float()
    hf = ln.float() * xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)
    ref = (hf @ w.float()) + bias.float()
    q = ref[:, : nq * D].view(S, nq, D)
    k = ref[:, nq * D:(nq + nkv) * D].view(S, nkv, D)
    cf, sf = cos.float()[:, None, :], sin.float()[:, None, :]
    ref[:, : nq * D] = (q * cf + ttft._rotate_half(q) * sf).reshape(S, -1)
    ref[:, nq * D:(nq + nkv) * D] = (k * cf + ttft._rotate_half(k) * sf).reshape(S, -1)
    # unfused bf16 path (the PyTorch bf16 expressions): norm kernel, then the fused QKV GEMM
    xu = x.clone()
    h = ttft._native_rmsnorm(xu, ln, EPS, residual=res)
    unfused = matmul_bias_rope(h, w, bias, cos, sin, rope_cols=(nq + nkv) * D, head_dim=D)
    # folded
    xx = x.clone()
    rstd = ttft._native_rmsnorm_rstd(xx, EPS, residual=res)
    assert torch.equal(xx, xr)
    out = matmul_bias_rope(xx, fold_rmsnorm_weight(ln, w), bias, cos, sin, rope_cols=(nq + nkv) * D, head_dim=D,
                           row_scale=rstd)
    _no_worse(out, unfused, ref)


@pytest.mark.parametrize("S", [2048, 129])
def test_folded_gate_up_swiglu_matches_pytorch(S, cuda_device):
    """Post-attention RMSNorm + gate/up GEMM + SwiGLU: folded form against silu(h Wg) * (h Wu)."""
    K, m = 3584, 1024
    x, _, ln, wg = _inputs(S, K, m, cuda_device, seed=S + 1)
    wu = (0.02 * torch.randn(K, m, generator=torch.Generator(device=cuda_device).manual_seed(3),
                             device=cuda_device)).to(torch.bfloat16)
    xf = x.float()
    hf = ln.float() * xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)
    ref = torch.nn.functional.silu(hf @ wg.float()) * (hf @ wu.float())
    wgu = mma.interleave_gate_up(wg, wu)
    unfused = matmul_swiglu(_rms_norm_torch(x, ln), wgu)
    rstd = ttft._native_rmsnorm_rstd(x, EPS)
    out = matmul_swiglu(x, fold_rmsnorm_weight(ln, wgu), row_scale=rstd)
    _no_worse(out, unfused, ref)


def test_row_scale_never_splits_k(cuda_device):
    """Few rows and a deep K would take the split-K kernel, which has no row-scaled epilogue."""
    assert mma.kernel_plan(16, 3584, 18944, torch.bfloat16)[0] == "splitk"
    S, K, N = 16, 18944, 512
    x, _, _, w = _inputs(S, K, N, cuda_device, seed=6)
    rs = torch.rand(S, device=cuda_device) + 0.5
    c = torch.empty(S, N, device=cuda_device, dtype=torch.bfloat16)
    mma._gemm(x, w, c, S, N, K, lda=K, ldb=N, ldc=N, round_f16=False, row_scale=rs)
    torch.testing.assert_close(c.float(), rs[:, None] * (x.float() @ w.float()), rtol=RTOL, atol=ATOL)


def _fp32_copy(shard):
    """The same model with every weight in fp32 (no bf16 rounding of activations either on torch ops)."""
    import copy

    s32 = copy.copy(shard)
    s32.embed, s32.ln_final, s32.lm_head = shard.embed.float(), shard.ln_final.float(), shard.lm_head.float()
    s32.layers = []
    for layer in shard.layers:
        l32 = copy.copy(layer)
        for name in ("ln_in", "w_qkv", "b_qkv", "w_o", "ln_post", "w_gate_up", "w_down"):
            t = getattr(layer, name)
            setattr(l32, name, t.float() if t is not None else None)
        l32.folded = None
        s32.layers.append(l32)
    return s32


def test_decoder_with_folded_norms(cuda_device):
    """Full-width 7B decoder (4 layers, random norm weights): with folded norms the logits depart from an
    fp32 forward of the same model no more than the unfused bf16 forward's do, the unfused forward meets the
    reference's TTFT check against torch (ttft.py:442), and the next token matches the fp32 model's."""
    arch = ttft.KNOWN_ARCHS["Qwen/Qwen2.5-7B"]
    shard = ttft.build_model_shard(arch, 1, 0, seed=3, device=cuda_device, num_layers=4)
    g = torch.Generator(device=cuda_device).manual_seed(11)
    for layer in shard.layers:
        layer.ln_in = (1.0 + 0.2 * torch.randn(arch.hidden_size, generator=g, device=cuda_device)).to(torch.bfloat16)
        layer.ln_post = (1.0 + 0.2 * torch.randn(arch.hidden_size, generator=g, device=cuda_device)).to(torch.bfloat16)
    ids = ttft._make_random_input_ids(2048, arch.vocab_size, cuda_device, seed=4)
    with torch.inference_mode():
        folded = ttft.decoder_forward(shard, ids, ttft.Backends(norm_fold=True))
        plain = ttft.decoder_forward(shard, ids, ttft.Backends())
        ref = ttft.decoder_forward(shard, ids, ttft.Backends(attention="cudnn", gemm="cublas", elementwise="torch"))
        ref32 = ttft.decoder_forward(_fp32_copy(shard), ids, ttft.Backends(attention="math", gemm="cublas",
                                                                            elementwise="torch"))
    torch.testing.assert_close(plain, ref, rtol=0.1, atol=0.1)
    ef, eu = (folded - ref32).abs(), (plain - ref32).abs()
    assert float(ef.max()) <= 1.5 * float(eu.max()) and float(ef.mean()) <= 1.25 * float(eu.mean()), \
        (float(ef.max()), float(eu.max()), float(ef.mean()), float(eu.mean()))
    # the same next token as the fp32 model, unless its top two are tied within the unfused forward's own error
    tf, tr = int(folded.argmax()), int(ref32.argmax())
    assert tf == tr or float(ref32[0, tr] - ref32[0, tf]) <= float(eu.max()), (tf, tr)
    del shard
    torch.cuda.empty_cache()
