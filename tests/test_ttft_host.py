"""TTFT model host logic on CPU: tensor-parallel plans, equivalence with HF Qwen2, the SDPA swap API,
and a world-size-2 gloo run of the sharded decoder (all-reduce after o_proj and down_proj)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.nn.functional as F

import ttft

SEVEN_B = ttft.KNOWN_ARCHS["Qwen/Qwen2.5-7B"]
TINY = ttft.ArchConfig(hidden_size=256, num_attention_heads=8, num_key_value_heads=2, num_hidden_layers=2,
                       head_dim=32, intermediate_size=512, vocab_size=1024)
TORCH = ttft.Backends(attention="math", gemm="cublas", elementwise="torch")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rank_plan_covers_every_head_once(world):
    group = SEVEN_B.num_attention_heads // SEVEN_B.num_key_value_heads
    seen_q, mlp = [], []
    for r in range(world):
        p = ttft.rank_plan(SEVEN_B, world, r)
        seen_q += list(p.q_heads)
        mlp += list(p.mlp_cols)
        # every segment's query heads share one key/value head, and it is the one the plan loads
        for first, count, kv in p.segments:
            heads = p.q_heads[first:first + count]
            assert {h // group for h in heads} == {p.kv_heads[kv]}
        assert sum(c for _, c, _ in p.segments) == len(p.q_heads)
        assert len(p.mlp_cols) % 64 == 0  # whole gate/up interleave blocks
    assert seen_q == list(range(SEVEN_B.num_attention_heads))
    assert mlp == list(range(SEVEN_B.intermediate_size))


def test_uneven_split_at_eight_ranks():
    sizes = [len(ttft.rank_plan(SEVEN_B, 8, r).q_heads) for r in range(8)]
    assert sizes == [4, 4, 4, 4, 3, 3, 3, 3]
    assert ttft.rank_plan(SEVEN_B, 8, 1).kv_heads == (0, 1)  # heads 4-7 span key/value heads 0 and 1
    assert len(ttft.rank_plan(SEVEN_B, 8, 0).mlp_cols) == 18944 // 8
    with pytest.raises(ValueError):
        ttft.rank_plan(SEVEN_B, 29, 0)


def test_decoder_matches_hf_qwen2():
    hf = ttft.load_model(TINY, device="cpu")
    shard = ttft.load_hf_weights_into_shard(hf, TINY)
    ids = ttft._make_random_input_ids(40, TINY.vocab_size, "cpu", seed=3)
    with torch.inference_mode():
        ref = ttft._forward_final_logits(hf, ids).float()
        ours = ttft.decoder_forward(shard, ids, TORCH)
    torch.testing.assert_close(ours, ref, rtol=2e-2, atol=2e-2)
    assert ours.argmax() == ref.argmax()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, out_path):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = ttft.build_model_shard(TINY, world, rank, seed=5, device="cpu")
        ids = ttft._make_random_input_ids(33, TINY.vocab_size, "cpu", seed=4)
        with torch.inference_mode():
            logits = ttft.decoder_forward(shard, ids, TORCH)
        if rank == 0:
            torch.save(logits, out_path)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_world_size_2_matches_single_rank(tmp_path):
    import torch.multiprocessing as mp

    out = str(tmp_path / "tp2.pt")
    mp.start_processes(_tp_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    tp2 = torch.load(out)
    single = ttft.build_model_shard(TINY, 1, 0, seed=5, device="cpu")
    ids = ttft._make_random_input_ids(33, TINY.vocab_size, "cpu", seed=4)
    with torch.inference_mode():
        tp1 = ttft.decoder_forward(single, ids, TORCH)
    torch.testing.assert_close(tp2, tp1, rtol=2e-2, atol=2e-2)
    assert tp2.argmax() == tp1.argmax()


def test_patched_sdpa_rejects_what_the_reference_rejects():
    x = torch.zeros(1, 2, 8, 32)
    with ttft.backend_context("triton_gqa", allow_causal_custom=False):
        with pytest.raises(RuntimeError, match="unsupported SDPA call: dropout_p=0.1"):
            F.scaled_dot_product_attention(x, x, x, dropout_p=0.1)
        with pytest.raises(RuntimeError, match="attn_mask is not None"):
            F.scaled_dot_product_attention(x, x, x, attn_mask=torch.ones(8, 8, dtype=torch.bool))
        with pytest.raises(RuntimeError, match="is_causal=True"):
            F.scaled_dot_product_attention(x, x, x, is_causal=True)
        # an accepted call goes to the GPU kernel, which refuses CPU tensors: there is no CPU path
        with pytest.raises(ValueError, match="CUDA tensor"):
            F.scaled_dot_product_attention(x, x, x)
    assert F.scaled_dot_product_attention is torch._C._nn.scaled_dot_product_attention or callable(
        F.scaled_dot_product_attention)


def test_backend_context_restores_sdpa_and_counts_calls():
    original = F.scaled_dot_product_attention
    stats = ttft.BackendUseStats("math")
    x = torch.randn(1, 4, 8, 16)
    k = torch.randn(1, 2, 8, 16)
    with ttft.backend_context("math", allow_causal_custom=False, stats=stats):
        y = F.scaled_dot_product_attention(x, k, k)  # GQA enabled by the wrapper
    assert stats.calls == 1 and y.shape == x.shape
    assert F.scaled_dot_product_attention is original
    with pytest.raises(ValueError, match="unknown backend"):
        with ttft.backend_context("nope", allow_causal_custom=False):
            pass


def test_repeat_kv_and_presets():
    k = torch.randn(1, 2, 5, 8)
    assert ttft._repeat_kv_for_gqa(k, 6).shape == (1, 6, 5, 8)
    with pytest.raises(ValueError):
        ttft._repeat_kv_for_gqa(k, 5)
    assert ttft._block_d_tune_args(128).BLOCK_DMODEL_OUTER == 64
    with pytest.raises(ValueError):
        ttft._block_d_tune_args(96)
    assert ttft.inspect_model_shape("Qwen/Qwen2.5-7B").num_key_value_heads == 4
