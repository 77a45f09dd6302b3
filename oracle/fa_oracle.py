"""CPU oracle for the attention forward -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Two checkers live here:

* `tiled_attention_forward`: a numpy restatement of the reference's Triton
  kernels' algorithm, tile by tile, in fp32:
    - Q tile loaded once, KV streamed in BLOCK_N steps (flash_atten.py:62-96);
    - qk = (q k^T) * sm_scale in fp32 (flash_atten.py:98);
    - out-of-range keys and, when causal, keys n > query m set to -inf
      (flash_atten.py:100-105; top-left aligned: visible iff m >= n);
    - online softmax: m_ij = max(m_i, rowmax), p = exp(qk - m_ij),
      alpha = exp(m_i - m_ij), acc = acc * alpha + p.to(v.dtype) @ v,
      l_i = l_i * alpha + rowsum(p) (flash_atten.py:107-116);
    - out = acc / l_i, lse = m_i + log(l_i) (flash_atten.py:118, 130-133).
  The `p.to(v.dtype)` rounding before the P*V product is reproduced with
  oracle.rounding.  Grouped-query heads follow the reference's SDPA path,
  which repeats each K/V head Hq/Hkv times (ttft.py:203-219).

* `sdpa_reference`: the reference's own correctness oracle, torch
  `F.scaled_dot_product_attention` on fp32 CPU copies
  (test_flash_atten.py:459-461, 498-499).
"""
from __future__ import annotations

import numpy as np

from oracle.rounding import round_to


def tiled_attention_forward(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    *,
    sm_scale: float | None = None,
    causal: bool = False,
    p_dtype: str = "fp32",
    block_m: int = 64,
    block_n: int = 64,
    q_row_offset: int = 0,
) -> tuple[np.ndarray, np.ndarray]:
    """Returns (o [B,Hq,M,D] fp32, lse [B,Hq,M] fp32) for q [B,Hq,M,D], k/v [B,Hkv,N,D].

    `q_row_offset` treats q as rows [offset, offset + M) of a longer query
    sequence (the causal mask then compares offset + m with n), so a slice of
    a large problem can be checked on its own.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, Hq, M, D = q.shape
    _, Hkv, N, _ = k.shape
    if Hq % Hkv:
        raise ValueError("query heads must be a multiple of key/value heads")
    group = Hq // Hkv
    if sm_scale is None:
        sm_scale = D ** -0.5
    o = np.empty((B, Hq, M, D), dtype=np.float32)
    lse = np.empty((B, Hq, M), dtype=np.float32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        for b in range(B):
            for h in range(Hq):
                hk = h // group
                for m0 in range(0, M, block_m):
                    rows = np.arange(m0, min(m0 + block_m, M))
                    qt = q[b, h, rows]
                    m_i = np.full(len(rows), -np.inf, dtype=np.float32)
                    l_i = np.zeros(len(rows), dtype=np.float32)
                    acc = np.zeros((len(rows), D), dtype=np.float32)
                    for n0 in range(0, N, block_n):
                        cols = np.arange(n0, min(n0 + block_n, N))
                        qk = (qt @ k[b, hk, cols].T).astype(np.float32) * np.float32(sm_scale)
                        if causal:
                            visible = (rows[:, None] + q_row_offset) >= cols[None, :]
                            qk = np.where(visible, qk, -np.inf).astype(np.float32)
                        m_ij = np.maximum(m_i, qk.max(axis=1))
                        p = np.exp(qk - m_ij[:, None]).astype(np.float32)
                        l_ij = p.sum(axis=1, dtype=np.float32)
                        alpha = np.exp(m_i - m_ij).astype(np.float32)
                        acc = acc * alpha[:, None] + round_to(p, p_dtype) @ v[b, hk, cols]
                        l_i = l_i * alpha + l_ij
                        m_i = m_ij
                    o[b, h, rows] = acc / l_i[:, None]
                    lse[b, h, rows] = m_i + np.log(l_i)
    return o, lse


def sdpa_reference(q, k, v, *, causal: bool = False, sm_scale: float | None = None):
    """torch SDPA (math) on fp32 CPU copies, GQA by repeating K/V heads; returns (o, lse) as numpy fp32."""
    import torch
    import torch.nn.functional as F

    qt = torch.as_tensor(np.asarray(q, dtype=np.float32))
    kt = torch.as_tensor(np.asarray(k, dtype=np.float32))
    vt = torch.as_tensor(np.asarray(v, dtype=np.float32))
    group = qt.shape[1] // kt.shape[1]
    if group > 1:
        kt = kt.repeat_interleave(group, dim=1)
        vt = vt.repeat_interleave(group, dim=1)
    o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, scale=sm_scale)
    scale = qt.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    s = (qt @ kt.transpose(-1, -2)) * scale
    if causal:
        M, N = s.shape[-2:]
        keep = torch.ones(M, N, dtype=torch.bool).tril()
        s = s.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    return o.numpy(), lse.numpy()


def attention_flops(B: int, H: int, M: int, N: int, D: int, causal: bool) -> float:
    """4*B*H*D*score_count; score_count = S(S+1)/2 causal, M*N otherwise (test_flash_atten.py:234-240)."""
    if causal:
        # keys visible to query m: min(m + 1, N)
        m = np.arange(M, dtype=np.float64)
        count = float(np.minimum(m + 1, N).sum())
    else:
        count = float(M) * float(N)
    return 4.0 * B * H * D * count
