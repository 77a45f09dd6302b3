"""Host-side behaviour of the drop-in modules (no GPU needed).

Mirrors what the reference's Python layer guarantees: argument validation
and error types of tuner.py, the dispatch contract of flash_atten.py and the
shape acceptance of mma.py.
"""
from __future__ import annotations

import pickle

import pytest
import torch

import exceptions
import flash_atten
import mma
import tuner
from tuner import (
    FlashAttenTuneArguments,
    FlashAttentionBlockDNomaskTuner,
    FlashAttentionLaunchSpec,
    FlashAttentionOptimizeSharedMemTuner,
    FlashAttentionTuner,
)


# ------------------------------------------------------------- tune arguments
@pytest.mark.parametrize(
    "kwargs, message",
    [
        (dict(BLOCK_N=0), "BLOCK_N must be positive when provided"),
        (dict(BLOCK_M=0), "BLOCK_M must be positive when provided"),
        (dict(BLOCK_M=48), "BLOCK_M must be a power of 2 when provided"),
        (dict(BLOCK_N_PAD=24), "BLOCK_N_PAD must be a power of 2 when provided"),
        (dict(BLOCK_DMODEL=-2), "BLOCK_DMODEL must be positive when provided"),
        (dict(BLOCK_DMODEL=96), "BLOCK_DMODEL must be a power of 2 when provided"),
        (dict(BLOCK_DMODEL_OUTER=12), "BLOCK_DMODEL_OUTER must be a power of 2 when provided"),
        (dict(NUM_WARPS=0), "NUM_WARPS must be positive when provided"),
        (dict(NUM_STAGES=-1), "NUM_STAGES must be positive when provided"),
    ],
)
def test_tune_argument_validation(kwargs, message):
    with pytest.raises(ValueError, match=message):
        FlashAttenTuneArguments(**kwargs)


def test_tune_arguments_accept_reference_presets():
    # the presets the reference's tests and ttft.py use (test_flash_atten.py:641-724, ttft.py:145-166)
    FlashAttenTuneArguments(BLOCK_N=64, BLOCK_M=128, BLOCK_N_PAD=64, BLOCK_DMODEL=128, BLOCK_DMODEL_OUTER=64,
                            NUM_WARPS=8, NUM_STAGES=3)
    FlashAttenTuneArguments(BLOCK_N=48, NUM_WARPS=3, NUM_STAGES=5)  # BLOCK_N / warps / stages need not be powers of 2


# ------------------------------------------------------------------- tuners
def test_tuner_shape_validation(fake_limits):
    q, k = (1, 2, 128, 64), (1, 2, 128, 64)
    with pytest.raises(ValueError, match="must all be 4D"):
        FlashAttentionTuner((2, 128, 64), k, k, 2, causal=False, return_lse=False)
    with pytest.raises(ValueError, match="Batch and head dimensions must match"):
        FlashAttentionTuner(q, (1, 1, 128, 64), (1, 1, 128, 64), 2, causal=False, return_lse=False)
    with pytest.raises(ValueError, match="Last dimension must match"):
        FlashAttentionTuner(q, (1, 2, 128, 32), (1, 2, 128, 32), 2, causal=False, return_lse=False)
    with pytest.raises(ValueError, match="sequence lengths must match"):
        FlashAttentionTuner(q, k, (1, 2, 64, 64), 2, causal=False, return_lse=False)
    with pytest.raises(ValueError, match="BLOCK_DMODEL must be >= D"):
        FlashAttentionTuner(q, k, k, 2, causal=False, return_lse=False, tune_args=FlashAttenTuneArguments(BLOCK_DMODEL=32))
    with pytest.raises(ValueError, match="BLOCK_N cannot exceed BLOCK_N_PAD"):
        FlashAttentionTuner(q, k, k, 2, causal=False, return_lse=False,
                            tune_args=FlashAttenTuneArguments(BLOCK_N=128, BLOCK_N_PAD=64))
    with pytest.raises(ValueError, match="NUM_WARPS must be <= 32"):
        FlashAttentionTuner(q, k, k, 2, causal=False, return_lse=False, tune_args=FlashAttenTuneArguments(NUM_WARPS=64))
    # the sliced variant allows BLOCK_DMODEL < D (tuner.py:604-605)
    FlashAttentionBlockDNomaskTuner(q, k, k, 2, causal=False, return_lse=False,
                                    tune_args=FlashAttenTuneArguments(BLOCK_DMODEL=32))


def test_tuner_candidates_are_the_compiled_tile_families(fake_limits):
    t = FlashAttentionTuner((4, 32, 8192, 128), (4, 32, 8192, 128), (4, 32, 8192, 128), 2, causal=True, return_lse=False)
    two, one = t._candidate_configs()
    assert two["variant"] == 0 and one["variant"] == 1
    assert two["BLOCK_M"] == 256 and two["BLOCK_N"] == 128 and two["BLOCK_DMODEL"] == 128
    assert two["num_warps"] == 12 and two["num_stages"] == 5
    assert one["BLOCK_M"] == 128 and one["BLOCK_N"] == 128 and one["num_warps"] == 8
    # D=256: both families name the same tile, so it is the only candidate
    t256 = FlashAttentionOptimizeSharedMemTuner((2, 16, 64, 256), (2, 16, 64, 256), (2, 16, 64, 256), 2,
                                                causal=True, return_lse=False)
    (cfg,) = t256._candidate_configs()
    assert cfg["BLOCK_M"] == 128 and cfg["BLOCK_N"] == 128 and cfg["BLOCK_DMODEL"] == 256
    t512 = FlashAttentionTuner((1, 1, 64, 512), (1, 1, 64, 512), (1, 1, 64, 512), 2, causal=False, return_lse=False)
    assert t512._candidate_configs() == []
    # the reference's shared-memory estimate formula (tuner.py:237-245)
    assert t.estimate_flash_fwd_shared_bytes(block_m=128, block_n_pad=64, block_dmodel=128, element_size=2) == 2 * 128 * 256


def test_runtime_shape_mismatch(fake_limits):
    t = FlashAttentionTuner((1, 1, 16, 64), (1, 1, 16, 64), (1, 1, 16, 64), 2, causal=False, return_lse=False)
    x = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="do not match the tuner shapes"):
        t.build_launch_spec(x, x, x, sm_scale=0.1, o=x, lse=None)
    with pytest.raises(ValueError, match="expects \\(q, k, v\\)"):
        t.build_launch_spec(x, x, sm_scale=0.1, o=x, lse=None)


def test_update_data_swaps_inputs_only():
    spec = FlashAttentionLaunchSpec(grid=(1, 1), kernel_args=("q", "k", "v", "o", "lse", 1, 2), kernel_kwargs={},
                                    launch_context={}, function_name="x", tune_args=FlashAttenTuneArguments(),
                                    input_shapes={})
    spec.update_data(("q2", "k2", "v2"))
    assert spec.kernel_args == ("q2", "k2", "v2", "o", "lse", 1, 2)


def test_power_of_two_helpers():
    assert [tuner._next_power_of_two(x) for x in (1, 2, 3, 5, 64, 65)] == [1, 2, 4, 8, 64, 128]
    with pytest.raises(ValueError):
        tuner._next_power_of_two(0)


# -------------------------------------------------------------- dispatch
def test_unknown_kernel_name_raises_name_error():
    spec = FlashAttentionLaunchSpec(grid=(1, 1), kernel_args=(None,) * 5, kernel_kwargs={}, launch_context={},
                                    function_name="_no_such_kernel", tune_args=FlashAttenTuneArguments(),
                                    input_shapes={})
    with pytest.raises(NameError, match="No such kernel named _no_such_kernel"):
        flash_atten.flash_attention(spec)


def test_kernel_mapping_names_match_reference():
    assert set(flash_atten.flash_attention_kernel_mapping) == {
        "_flash_attn_fwd_kernel_basic",
        "_flash_attn_fwd_kernel_optimize_shared_mem",
        "_flash_attn_fwd_kernel_block_d_nomask_contiguous",
    }
    assert flash_atten._flash_attn_fwd_kernel_basic is flash_atten.flash_attention_kernel_mapping["_flash_attn_fwd_kernel_basic"]


def test_launchers_refuse_cpu_tensors():
    x = torch.zeros(1, 1, 16, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA tensor"):
        flash_atten.attention_forward(x, x, x)
    args = (x, x, x, x, 0, *x.stride(), *x.stride(), *x.stride(), *x.stride(), 0, 0, 0, 1, 16, 16, 64, 0.125)
    with pytest.raises(ValueError, match="CUDA tensor"):
        flash_atten._flash_attn_fwd_kernel_basic[(1, 1)](*args, causal=False, HAS_LSE=False)
    with pytest.raises(TypeError, match="29 positional arguments"):
        flash_atten._flash_attn_fwd_kernel_basic[(1, 1)](*args[:-1])
    with pytest.raises(TypeError, match="9 positional arguments"):
        flash_atten._flash_attn_fwd_kernel_block_d_nomask_contiguous[(1, 1)](x, x, x, x, 1, 16, 16, 64)
    a = torch.zeros(128, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA tensor"):
        mma._matmul_contiguous_kernel[(1,)](a, a.T.contiguous(), a, 128, 128, 64)


def test_launcher_grid_must_cover_batch_times_heads():
    x = torch.zeros(1, 3, 16, 64, dtype=torch.float16)
    args = (x, x, x, x, 0, *x.stride(), *x.stride(), *x.stride(), *x.stride(), 0, 0, 0, 2, 16, 16, 64, 0.125)
    with pytest.raises(ValueError, match="grid\\[1\\] must be batch\\*H"):
        flash_atten._flash_attn_fwd_kernel_basic[(1, 3)](*args)


# ------------------------------------------------------------------ matmul
def _reference_acceptance(m, n, k):
    """mma.py:63-81 restated: which shapes the reference accepts."""
    if k % 32:
        return False
    return (m >= 2048 and n >= 2048 and m % 128 == 0 and n % 128 == 0) or (m % 128 == 0 and n % 64 == 0) or (
        m % 128 == 0 and n % 128 == 0) or (m % 64 == 0 and n % 256 == 0)


@pytest.mark.parametrize("m", [64, 128, 192, 1000, 1024, 4096])
@pytest.mark.parametrize("n", [64, 96, 256, 512, 1000, 16384])
@pytest.mark.parametrize("k", [32, 48, 256])
def test_select_config_accepts_what_the_reference_accepts(m, n, k):
    if _reference_acceptance(m, n, k):
        cfg = mma._select_2d_contiguous_config(m, n, k)
        assert len(cfg) == 6 and cfg[:3] == (128, 256, 64)
    else:
        with pytest.raises(ValueError, match="fast 2D contiguous matmul requires"):
            mma._select_2d_contiguous_config(m, n, k)


def test_cache_hints_probe_without_cuda():
    if not torch.cuda.is_available():
        assert mma._supports_contiguous_cache_eviction_hints() is False


# -------------------------------------------------------------- exceptions
def test_out_of_resources_message_and_pickle():
    exc = exceptions.OutOfResourcesWithDetail(
        300000, 232448, "shared memory", kernel_name="k", launch_context={"a": 1}, extra_detail="nothing fit."
    )
    text = str(exc)
    assert text.startswith("out of resource: shared memory, Required: 300000, Hardware limit: 232448.")
    assert "more shared memory per SM" in text and "Kernel: k." in text and "Launch context: a=1." in text
    assert text.endswith("nothing fit.")
    assert isinstance(exc, exceptions.OutOfResources)
    base = pickle.loads(pickle.dumps(exceptions.OutOfResources(1, 2, "registers")))
    assert (base.required, base.limit, base.name) == (1, 2, "registers")
    wrapped = exceptions.OutOfResourcesWithDetail.from_out_of_resources(base, kernel_name="x")
    assert wrapped.original_exception is base and "register file" in str(wrapped)


def test_resource_usage_summary_format():
    ctx = {
        "compiled_shared_memory_bytes_per_block": 197728,
        "available_shared_memory_bytes_per_sm": 232448,
        "attempted_register_file_size_bytes_per_block": 258048,
        "available_register_file_size_bytes_per_sm": 262144,
        "attempted_registers_per_block": 64512,
        "available_registers_per_sm": 65536,
    }
    s = exceptions._resource_usage_summary("k", ctx, tune_args=FlashAttenTuneArguments(BLOCK_M=256),
                                           input_shapes={"q": (1, 2, 3, 4), "lse": None})
    assert s.startswith("k tuner resources: \nshared=197728/232448 bytes per block/SM, ")
    assert "registers=64512/65536 per block/SM" in s
    assert "tune_args=BLOCK_M=256" in s and "input_shapes=q=(1, 2, 3, 4)" in s


def test_measured_variant_lookup(tmp_path):
    """Nearest measured shape with the same dtype width, padded head dim and causality decides; shapes with
    nothing measured, or head dims with a single family, get the default family."""
    import json

    import _native
    import tune_table

    table = tmp_path / "t.json"
    entries = [
        {"width": 2, "head_dim_padded": 128, "causal": False, "batch_heads": 8, "seqlen_q": 512, "seqlen_k": 512,
         "ms": {"0": 0.02, "1": 0.015}, "best_variant": 1},
        {"width": 2, "head_dim_padded": 128, "causal": False, "batch_heads": 128, "seqlen_q": 8192,
         "seqlen_k": 8192, "ms": {"0": 3.6, "1": 4.3}, "best_variant": 0},
    ]
    table.write_text(json.dumps({"entries": entries}))
    bf16 = _native.FAB_DTYPE_BF16
    assert tune_table.measured_variant(bf16, 128, False, 8, 600, 600, path=table) == 1
    assert tune_table.measured_variant(bf16, 128, False, 128, 4096, 4096, path=table) == 0
    assert tune_table.measured_variant(bf16, 96, False, 8, 600, 600, path=table) == 1  # pads to 128
    assert tune_table.measured_variant(bf16, 128, True, 8, 600, 600, path=table) == 0  # nothing causal measured
    assert tune_table.measured_variant(bf16, 256, False, 8, 600, 600, path=table) == 0  # one family only
    assert tune_table.measured_variant(bf16, 128, False, 8, 600, 600, path=tmp_path / "missing.json") == 0


def test_gate_up_interleave_round_trip():
    g = torch.Generator().manual_seed(4)
    wg, wu = torch.randn(5, 192, generator=g), torch.randn(5, 192, generator=g)
    w = mma.interleave_gate_up(wg, wu)
    assert w.shape == (5, 384)
    assert torch.equal(w[:, :64], wg[:, :64]) and torch.equal(w[:, 64:128], wu[:, :64])
    assert torch.equal(w[:, 256:320], wg[:, 128:])
    gate, up = mma.split_gate_up(w)
    assert torch.equal(gate, wg) and torch.equal(up, wu)
    with pytest.raises(ValueError):
        mma.interleave_gate_up(torch.zeros(5, 100), torch.zeros(5, 100))


def test_matmul_swiglu_refuses_cpu_and_odd_widths():
    with pytest.raises(ValueError):
        mma.matmul_swiglu(torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(8, 192, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        mma.matmul_swiglu(torch.zeros(4, 8), torch.zeros(8, 256))


def test_host_entry_validation():
    x = torch.zeros(1, 2, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="q must be a CPU tensor"):
        flash_atten.attention_forward_host(torch.zeros(1, 2, 16, 64, dtype=torch.bfloat16, device="meta"), x, x)
    with pytest.raises(ValueError, match="shape \\[batch, heads, seq, head_dim\\]"):
        flash_atten.attention_forward_host(x[0], x, x)
    with pytest.raises(ValueError, match="kv_heads dividing"):
        flash_atten.attention_forward_host(x, torch.zeros(1, 3, 16, 64, dtype=torch.bfloat16),
                                           torch.zeros(1, 3, 16, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="out must be a CPU tensor"):
        flash_atten.attention_forward_host(x, x, x, out=torch.zeros(1, 2, 16, 32, dtype=torch.bfloat16))
    # nothing to compute: returns without touching a device
    e = torch.zeros(0, 2, 16, 64, dtype=torch.bfloat16)
    assert flash_atten.attention_forward_host(e, e, e).shape == e.shape


@pytest.mark.parametrize("batch, kv_heads, chunks", [(4, 32, 16), (1, 4, 16), (3, 5, 7), (2, 1, 64), (5, 8, 1)])
def test_host_entry_pieces_cover_every_unit_once(batch, kv_heads, chunks):
    pieces = flash_atten._host_pieces(batch, kv_heads, chunks)
    seen = [(b, h) for b, h0, h1 in pieces for h in range(h0, h1)]
    assert sorted(seen) == [(b, h) for b in range(batch) for h in range(kv_heads)]
    assert len(pieces) <= batch * -(-chunks // batch) and all(h1 > h0 for _, h0, h1 in pieces)
