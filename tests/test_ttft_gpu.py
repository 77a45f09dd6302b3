"""TTFT path on the GPU: the SDPA swap inside an HF Qwen2 model, and the tensor-parallel decoder on the
native kernels against the same decoder on torch SDPA (cuDNN) + cuBLAS.

Tolerance: the reference's own TTFT check, final-token logits allclose(rtol=0.1, atol=0.1) against
torch's flash backend (ttft.py:442), plus the same next token."""
from __future__ import annotations

import os
import socket

import pytest
import torch

import _native
import ttft

pytestmark = pytest.mark.gpu

SEVEN_B = ttft.KNOWN_ARCHS["Qwen/Qwen2.5-7B"]


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    torch.cuda.synchronize()
    assert _native.device_error() == 0, "a kernel gave up on a bounded wait"


def test_hf_model_through_the_sdpa_swap(cuda_device):
    """Qwen2.5-7B architecture (2 of 28 layers), causal prefill: the patched SDPA matches torch flash."""
    model = ttft.load_model("Qwen/Qwen2.5-7B", num_layers=2, seed=1)
    ids = ttft._make_random_input_ids(1000, SEVEN_B.vocab_size, cuda_device, seed=2)
    summary = ttft.verify_against_flash(model, ids, backend="triton_gqa", allow_causal_custom=True,
                                        force_noncausal=False)
    assert "next_token_match=True" in summary
    # the reference's non-causal mode too
    ttft.verify_against_flash(model, ids, backend="triton_gqa", allow_causal_custom=True, force_noncausal=True)
    samples = ttft.time_ttft_ms(model, ids, backend="triton_gqa", repeats=1, warmups=1, allow_causal_custom=True,
                                force_noncausal=False)
    assert len(samples) == 1 and samples[0] > 0
    del model
    torch.cuda.empty_cache()


def test_decoder_native_matches_torch(cuda_device):
    """Full-width 7B decoder (4 layers): native attention + GEMM against torch cuDNN SDPA + cuBLAS."""
    shard = ttft.build_model_shard(SEVEN_B, 1, 0, seed=3, device=cuda_device, num_layers=4)
    ids = ttft._make_random_input_ids(2048, SEVEN_B.vocab_size, cuda_device, seed=4)
    with torch.inference_mode():
        ours = ttft.decoder_forward(shard, ids, ttft.Backends(attention="native", gemm="native"))
        ref = ttft.decoder_forward(shard, ids, ttft.Backends(attention="cudnn", gemm="cublas", elementwise="torch"))
        mixed = ttft.decoder_forward(shard, ids, ttft.Backends(attention="native", gemm="cublas"))
        torch_ops = ttft.decoder_forward(shard, ids, ttft.Backends(attention="native", gemm="native",
                                                                   elementwise="torch"))
    torch.testing.assert_close(torch_ops, ours, rtol=0.1, atol=0.1)
    torch.testing.assert_close(ours, ref, rtol=0.1, atol=0.1)
    torch.testing.assert_close(mixed, ref, rtol=0.1, atol=0.1)
    assert ours.argmax() == ref.argmax()
    del shard
    torch.cuda.empty_cache()


def test_decoder_uneven_tp8_plan_on_one_gpu(cuda_device):
    """The 8-way plan's rank 1 (query heads 4-7 over key/value heads 0 and 1, two attention calls) computes
    the same partial o_proj input as slicing the single-rank computation."""
    full = ttft.build_model_shard(SEVEN_B, 1, 0, seed=6, device=cuda_device, num_layers=1)
    part = ttft.build_model_shard(SEVEN_B, 8, 1, seed=6, device=cuda_device, num_layers=1)
    S, D = 512, SEVEN_B.head_dim
    g = torch.Generator(device=cuda_device).manual_seed(7)
    x = torch.randn(S, SEVEN_B.hidden_size, generator=g, device=cuda_device).to(torch.bfloat16)
    outs = []
    for shard in (full, part):
        layer, plan = shard.layers[0], shard.plan
        nq, nkv = len(plan.q_heads), len(plan.kv_heads)
        qkv = x @ layer.w_qkv + layer.b_qkv
        q = qkv[:, :nq * D].view(S, nq, D).unsqueeze(0).transpose(1, 2)
        k = qkv[:, nq * D:(nq + nkv) * D].view(S, nkv, D).unsqueeze(0).transpose(1, 2)
        v = qkv[:, (nq + nkv) * D:].view(S, nkv, D).unsqueeze(0).transpose(1, 2)
        out = torch.empty(1, nq, S, D, device=cuda_device, dtype=torch.bfloat16)
        ttft._attention_segments(q, k, v, out, plan, "native")
        outs.append(out)
    torch.testing.assert_close(outs[1], outs[0][:, 4:8], rtol=2e-2, atol=2e-2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_path):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        shard = ttft.build_model_shard(SEVEN_B, world, rank, seed=8, device=f"cuda:{rank}", num_layers=2)
        ids = ttft._make_random_input_ids(1024, SEVEN_B.vocab_size, f"cuda:{rank}", seed=9)
        with torch.inference_mode():
            logits = ttft.decoder_forward(shard, ids, ttft.Backends())
        if rank == 0:
            torch.save(logits.cpu(), out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_nccl_two_gpus(tmp_path, cuda_device):
    import torch.multiprocessing as mp

    out = str(tmp_path / "tp2.pt")
    mp.start_processes(_nccl_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    tp2 = torch.load(out)
    single = ttft.build_model_shard(SEVEN_B, 1, 0, seed=8, device=cuda_device, num_layers=2)
    ids = ttft._make_random_input_ids(1024, SEVEN_B.vocab_size, cuda_device, seed=9)
    with torch.inference_mode():
        tp1 = ttft.decoder_forward(single, ids, ttft.Backends()).cpu()
    torch.testing.assert_close(tp2, tp1, rtol=0.1, atol=0.1)


def test_cuda_graph_replay_matches_eager(cuda_device):
    """The captured prefill replays to the same logits as the eager forward, for two different prompts."""
    shard = ttft.build_model_shard(SEVEN_B, 1, 0, seed=12, device=cuda_device, num_layers=2)
    graphed = ttft.GraphedDecoder(shard, 1024, ttft.Backends(), device=cuda_device)
    try:
        for seed in (13, 14):
            ids = ttft._make_random_input_ids(1024, SEVEN_B.vocab_size, cuda_device, seed=seed)
            with torch.inference_mode():
                eager = ttft.decoder_forward(shard, ids, ttft.Backends())
                replay = graphed(ids).clone()
            assert torch.equal(replay, eager)
    finally:
        graphed.close()
    del shard
    torch.cuda.empty_cache()
