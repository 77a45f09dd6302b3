"""Fused GEMM + all-reduce over NVLink peer memory (tp_allreduce.FusedGemmAllReduce / fab_gemm_allreduce).

One GPU: a group of one (every tile owned locally) against torch.matmul, over several calls on the same
buffers.  Two GPUs: two NCCL ranks, each with its own a_r and b_r, against sum_r a_r @ b_r computed in fp32,
and the tensor-parallel decoder with the fused kernel against the same decoder on NCCL all-reduce.
Tolerance: each rank's partial tile is rounded to bf16 before the fp32 sum (as an NCCL bf16 all-reduce
receives bf16 partials), so the error grows like sqrt(world) bf16 steps of O(1) partials: rtol 1e-2 and
atol 0.015 * sqrt(world) against the exact fp32 sum.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

import _native
import ttft
from tp_allreduce import FusedGemmAllReduce

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _operands(rank, M, K, N, device, seed=0):
    g = torch.Generator(device=device).manual_seed(seed + 17 * rank)
    a = (torch.randn(M, K, generator=g, device=device) / K ** 0.25).to(torch.bfloat16)
    b = (torch.randn(K, N, generator=g, device=device) / K ** 0.25).to(torch.bfloat16)
    return a, b


def test_group_of_one_matches_matmul(cuda_device):
    fused = FusedGemmAllReduce(None, max_rows=1000, cols=3584, dtype=torch.bfloat16, device=cuda_device)
    for call, (M, K) in enumerate([(1000, 512), (300, 448), (1000, 2368)]):
        a, b = _operands(0, M, K, 3584, cuda_device, seed=call)
        out = fused(a, b).clone()
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        torch.testing.assert_close(out.float(), (a.float() @ b.float()), rtol=1e-2, atol=2e-2)
    assert fused.calls == 3
    assert int(fused.counters.abs().sum()) == 0  # every counter back at zero


def _worker(rank, world, port, out_path):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    fused = None
    try:
        fused = FusedGemmAllReduce(dist.group.WORLD, max_rows=2048, cols=3584, dtype=torch.bfloat16, device=dev)
        errs = []
        for call, (M, K) in enumerate([(2048, 1792), (777, 448), (2048, 9472)]):
            a, b = _operands(rank, M, K, 3584, dev, seed=10 * call)
            out = fused(a, b).clone()
            torch.cuda.synchronize()
            ref = sum(x.float() @ y.float() for x, y in (_operands(r, M, K, 3584, dev, seed=10 * call)
                                                          for r in range(world)))
            errs.append(float((out.float() - ref).abs().max()))
            torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=0.015 * world ** 0.5)
        assert _native.device_error() == 0
        # the tensor-parallel decoder: fused kernel against NCCL all-reduce
        arch = ttft.KNOWN_ARCHS["Qwen/Qwen2.5-7B"]
        shard = ttft.build_model_shard(arch, world, rank, seed=8, device=dev, num_layers=2)
        ids = ttft._make_random_input_ids(1024, arch.vocab_size, dev, seed=9)
        with torch.inference_mode():
            base = ttft.decoder_forward(shard, ids, ttft.Backends(), group=dist.group.WORLD)
            fz = ttft.decoder_forward(shard, ids, ttft.Backends(fused_allreduce=fused), group=dist.group.WORLD)
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        if rank == 0:
            torch.save({"errs": errs, "base": base.cpu(), "fused": fz.cpu()}, out_path)
        dist.barrier()
    finally:
        if fused is not None:
            torch.cuda.synchronize()
            fused.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ranks_over_nvlink(tmp_path, cuda_device):
    """As many ranks as the box has GPUs (2 to 8); at 8 the decoder's heads split 4,4,4,4,3,3,3,3, so the
    ranks' o_proj GEMMs have different K over the same output tiles."""
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    out = str(tmp_path / "ar.pt")  # rank 0 saves its results here
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    res = torch.load(out)
    # each rank checked out against sum_r a_r @ b_r; |out| reaches ~3 sqrt(world) here
    assert max(res["errs"]) < 0.05 * world ** 0.5
    torch.testing.assert_close(res["fused"], res["base"], rtol=0.1, atol=0.1)
    assert res["fused"].argmax() == res["base"].argmax()
