"""Benchmark of the hot path: attention forward (and matmul) on B200.

Contract: `python bench.py --gpus N --steps K --warmup W [--impl ours|reference]`
prints ONE JSON line on rank 0.  For N > 1 it runs under torchrun, one rank
per GPU; each rank owns an independent shard of (batch, head) work units
(weak scaling, no data-path collective), timing is the max over ranks.

Default workload (the north-star case): attention forward,
B=4 per GPU, H=32, S=8192, D=128, bf16, non-causal, seeded N(0,1) inputs.
  value  : whole-job TFLOP/s with inputs resident in HBM (CUDA events around
           K steps; the 805 MB of inputs per step exceed the 126 MB L2, so no
           flush is needed between steps).
  e2e    : the same metric through the public API (`flash_atten.attention_forward`)
           with host buffers: every step copies q, k, v from pinned host memory
           and reads o back, inside the timed region.
  roofline: tensor-bound; achieved = algorithmic FLOPs per launch / mean launch
           time (CUDA events on the launch stream), peak = measured dense bf16
           from MEASURED_PEAKS.json.
  cpu_baseline: the reference's CPU path (torch SDPA on fp32 CPU copies,
           test_flash_atten.py:459-461, 498-499) on a bounded sample of the
           same workload, timed on this host's cores.

`--impl reference` times that same CPU path as the benchmark arm (the
reference has no GPU path that runs without Triton; its published numbers
are for its Triton kernels on T4/A10).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "flash-attn-economical-gpu_b200"
for _p in (str(PKG), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

NCCL_LOG = None
if int(os.environ.get("WORLD_SIZE", "1")) > 1 and os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
    # NCCL reads these when torch first calls into it (the GPU boxes preset NCCL_DEBUG=VERSION, which prints
    # only the version).  Its communicator set-up lines (ranks, devices, transports) go to a per-process file
    # that setup_dist copies to stderr once the communicator exists, so a multi-rank run records which ranks
    # joined while stdout keeps rank 0's one JSON line.
    import tempfile

    NCCL_LOG = os.path.join(tempfile.gettempdir(), f"bench_nccl_{os.getpid()}.log")
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    os.environ["NCCL_DEBUG_FILE"] = NCCL_LOG

import torch  # noqa: E402

METRIC = "FA fwd TFLOPS (% of B200 bf16 peak) vs torch SDPA; Qwen2.5-7B-arch TTFT ms"
FALLBACK_BF16_TFLOPS = 1590.0
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    # name: (B, Hq, Hkv, S, D, causal)
    "fa_s8192_noncausal": (4, 32, 32, 8192, 128, False),
    "fa_s8192_causal": (4, 32, 32, 8192, 128, True),
    "fa_s4096_noncausal": (4, 32, 32, 4096, 128, False),
    "fa_s2048_noncausal": (4, 32, 32, 2048, 128, False),
    "fa_s1024_noncausal": (4, 32, 32, 1024, 128, False),
    "fa_s4096_causal": (4, 32, 32, 4096, 128, True),
    "fa_s2048_causal": (4, 32, 32, 2048, 128, True),
    "fa_s1024_causal": (4, 32, 32, 1024, 128, True),
    "fa_d256_s4096_causal": (2, 16, 16, 4096, 256, True),
    "fa_d256_s2048_causal": (2, 16, 16, 2048, 256, True),
    "fa_d256_s8192_causal": (2, 16, 16, 8192, 256, True),
    "fa_gqa_s8192_causal": (2, 16, 4, 8192, 128, True),
    # the reference's long-sequence pipeline cases (test_flash_atten.py:82-88), non-causal
    "fa_b1h28_s16384_noncausal": (1, 28, 28, 16384, 128, False),
    "fa_b1h28_s32768_noncausal": (1, 28, 28, 32768, 128, False),
    "fa_b1h28_s65536_noncausal": (1, 28, 28, 65536, 128, False),
    "fa_b1h16_d256_s16384_noncausal": (1, 16, 16, 16384, 256, False),
    "fa_b1h16_d256_s32768_noncausal": (1, 16, 16, 32768, 256, False),
    "fa_b1h16_d256_s65536_noncausal": (1, 16, 16, 65536, 256, False),
}
# Square matmuls of BASELINE config 4; any other shape as gemm_<M>x<K>x<N> (e.g. gemm_2048x3584x3584).
GEMM_WORKLOADS = {"gemm_8192": 8192, "gemm_16384": 16384, "gemm_4096": 4096, "gemm_2048": 2048, "gemm_1024": 1024}


def gemm_shape(workload: str):
    """(M, K, N) of a matmul workload name, or None when it names none."""
    if workload in GEMM_WORKLOADS:
        n = GEMM_WORKLOADS[workload]
        return n, n, n
    if workload.startswith("gemm_"):
        parts = workload[5:].split("x")
        if len(parts) == 3 and all(x.isdigit() and int(x) > 0 for x in parts):
            return tuple(int(x) for x in parts)
    return None


def input_sets(input_bytes: int) -> int:
    """How many distinct input sets a timed run rotates through: enough that the inputs of one step were
    last read at least 2 x L2 bytes of other inputs ago (the reference draws fresh inputs every
    iteration, test_flash_atten.py:516-531); one set when a step's inputs alone are that large."""
    return max(1, math.ceil(2 * L2_BYTES / max(input_bytes, 1)))


def l2_policy(input_bytes: int) -> str:
    sets = input_sets(input_bytes)
    mb = input_bytes / 1e6
    if sets == 1:
        return f"inputs {mb:.0f} MB per step >= 2 x 126 MB L2; no flush"
    return (f"inputs {mb:.0f} MB per step < 2 x 126 MB L2: {sets} seeded input sets in rotation "
            f"({sets * mb:.0f} MB), so no step reads inputs left in L2 by the previous one")
# Split-KV decode steps (not a BASELINE config; K/V cache resident on the device):
# name: (B, Hq, Hkv, query rows, keys, D)
DECODE_WORKLOADS = {
    "decode_n131072": (1, 28, 4, 1, 131072, 128),
    "decode_n32768_b8": (8, 28, 4, 1, 32768, 128),
}


def attention_config(workload, world):
    """The `config` object of an attention workload, the same on both arms."""
    B, Hq, Hkv, S, D, causal = WORKLOADS[workload]
    in_bytes = (B * Hq + 2 * B * Hkv) * S * D * 2
    return {
        "workload": f"attention forward B{B} Hq{Hq} Hkv{Hkv} S{S} D{D} bf16 {'causal' if causal else 'non-causal'}"
                    " per GPU (BASELINE config 2/3)",
        "global_batch": B * world,
        "seq_len": S,
        "heads_q": Hq,
        "heads_kv": Hkv,
        "head_dim": D,
        "causal": causal,
        "parallelism": f"dp{world} (each rank owns {B} sequences x {Hq} heads; no collective)",
        "l2_policy": l2_policy(in_bytes),
    }


def attention_flops(B, H, S, D, causal):
    score = S * (S + 1) / 2 if causal else S * S
    return 4.0 * B * H * D * score


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        try:
            d = json.loads(path.read_text())
            return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
        except Exception:
            pass
    return FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def committed_traffic(workload: str):
    """DRAM bytes per launch from the committed ncu summary for this workload, if one exists."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.is_file():
        return None
    try:
        value = json.loads(path.read_text()).get(workload)
        return int(value) if isinstance(value, (int, float)) else None
    except Exception:
        return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle",
        0x2: "applications_clocks_setting",
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x10: "sync_boost",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[int] = []
        self.masks: set[int] = set()
        self.errors: set[str] = set()
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._handle = None
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(visible.split(",")[device_index]) if visible else device_index
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self._handle = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(int(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)))
                mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle))
                self.masks.add(mask)
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception as exc:
                self.errors.add(f"{type(exc).__name__}: {exc}"[:120])
            time.sleep(self._period)

    def __enter__(self):
        if self._handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._handle is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        out = {
            "sm_mhz": statistics.median(self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
            "reason_masks": sorted(hex(m) for m in self.masks),
        }
        if self.errors:
            out["nvml_errors"] = sorted(self.errors)
        return out


# ---------------------------------------------------------------- helpers
def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)  # one communicator per rank, made here
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300), **kwargs)
        dist.barrier()
        nccl = ".".join(str(x) for x in torch.cuda.nccl.version()) if backend == "nccl" else "-"
        print(f"[bench] rank {rank} of {world}: {backend} (NCCL {nccl}), device cuda:{local}", file=sys.stderr,
              flush=True)
        if NCCL_LOG is not None and os.path.isfile(NCCL_LOG):
            with open(NCCL_LOG) as f:
                sys.stderr.write(f.read())
            sys.stderr.flush()
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def host_lead(ms=3.0):
    """Queue a device-side sleep ahead of the timed launches.

    The host then enqueues the timed steps while the GPU is still busy, so each event pair brackets device time
    only, not the host's launch latency (tens of microseconds per call through Python and ctypes, as long as a
    whole 1024^3 matmul).  The sleep itself ends before the first timed event.  Without torch's sleep kernel the
    lead is skipped (the events then also include host launch latency)."""
    sleep = getattr(torch.cuda, "_sleep", None)
    if sleep is not None:
        sleep(int(ms * 1e-3 * 1.965e9))


def warm_up(fn, count: int, min_s: float = 0.02) -> None:
    """`count` untimed calls, then more until `min_s` of wall time has passed (synchronised), so that a short
    kernel's timed calls do not follow a fraction of a millisecond of work; every timed leg, ours and each
    comparator, warms this way.  Warming much longer (0.1-0.3 s back to back) runs the timed calls under the
    power cap instead (1.5-1.9 GHz on B200)."""
    for _ in range(count):
        fn()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < min_s:
        for _ in range(4):
            fn()
        torch.cuda.synchronize()


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def shard_units(total_units: int, world: int, rank: int) -> range:
    """Contiguous block of work units owned by `rank` (balanced to within one unit)."""
    base, extra = divmod(total_units, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def cpu_attention_sample(S, D, causal, target_s=10.0, max_heads=64):
    """The reference's CPU path (fp32 torch SDPA on CPU) on a bounded sample of the workload."""
    import torch.nn.functional as F

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)

    def run(h):
        q, k, v = (torch.randn(1, h, S, D, generator=g) for _ in range(3))
        t0 = time.perf_counter()
        F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        return time.perf_counter() - t0

    run(1)  # warm-up
    t1 = run(1)
    heads = max(1, min(max_heads, int(target_s / max(t1, 1e-6))))
    t = run(heads) if heads > 1 else t1
    flops = attention_flops(1, heads, S, D, causal)
    return {
        "value": flops / t / 1e12,
        "unit": "TFLOP/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{heads} of the workload's (batch, head) units at S={S} D={D} causal={causal}, fp32 torch SDPA "
                  f"on CPU copies (the reference's oracle path), one timed pass of {t:.2f} s",
        "seconds": t,
    }


def measured_hbm_gbs():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def peaks_entry(achieved_tflops, workload):
    burst, sustained, source = measured_peaks()
    traffic = committed_traffic(workload)
    return {
        "bound": "tensor",
        "achieved": round(achieved_tflops, 1),
        "peak": burst,
        "unit": "TFLOP/s",
        "frac": round(achieved_tflops / burst, 4),
        "peak_source": f"{source} dense bf16 (burst; a kernel timed alone); sustained {sustained}",
        "traffic": traffic,
    }


# ------------------------------------------------------------ attention arm
def run_attention(args, world, rank, local):
    import _native
    from flash_atten import attention_forward, attention_forward_host

    B, Hq, Hkv, S, D, causal = WORKLOADS[args.workload]
    dev = torch.device("cuda", local)
    dtype = torch.bfloat16
    # Each rank owns batch rows [rank*B, (rank+1)*B) of a global batch of B*world sequences.
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    in_bytes = (B * Hq + 2 * B * Hkv) * S * D * 2
    sets = []
    for _ in range(input_sets(in_bytes)):
        q = torch.randn(B, Hq, S, D, generator=g, device=dev, dtype=dtype)
        k = torch.randn(B, Hkv, S, D, generator=g, device=dev, dtype=dtype)
        v = torch.randn(B, Hkv, S, D, generator=g, device=dev, dtype=dtype)
        sets.append((q, k, v))
    q, k, v = sets[0]
    o = torch.empty_like(q)
    flops = attention_flops(B, Hq, S, D, causal)
    stream = torch.cuda.current_stream(dev)

    warm_step = [0]

    def warm_call():
        attention_forward(*sets[warm_step[0] % len(sets)], causal=causal, out=o)
        warm_step[0] += 1

    warm_up(warm_call, args.warmup)
    if _native.device_error():
        raise RuntimeError("device error during warm-up")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        t_begin = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        host_lead()
        t_begin.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            attention_forward(*sets[(args.warmup + i) % len(sets)], causal=causal, out=o)
            ends[i].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    elapsed_ms = max_over_ranks(t_begin.elapsed_time(t_end), world)
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    if _native.device_error():
        raise RuntimeError("device error during the timed region")
    total_flops = sum_over_ranks(flops * args.steps, world)
    value = total_flops / (elapsed_ms / 1e3) / 1e12
    achieved = flops / (launch_ms / 1e3) / 1e12

    # ---- e2e through the public API with host buffers
    qh = q.cpu().pin_memory()
    kh = k.cpu().pin_memory()
    vh = v.cpu().pin_memory()
    oh = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_step():
        # q, k, v in from pinned host memory and O back, pipelined in pieces on three streams
        attention_forward_host(qh, kh, vh, causal=causal, out=oh, device=dev)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = sum_over_ranks(flops * e2e_steps, world) / (e2e_ms / 1e3) / 1e12
    h2d = (q.numel() + k.numel() + v.numel()) * q.element_size()
    d2h = o.numel() * o.element_size()

    # ---- same-box comparators (rank 0 only, not part of the metric)
    comparators = {}
    if rank == 0 and not args.no_compare:
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        for name, be in (("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("torch_sdpa_flash", SDPBackend.FLASH_ATTENTION)):
            try:
                rep = Hq // Hkv
                csets = [(qq, kk if rep == 1 else kk.repeat_interleave(rep, dim=1),
                          vv if rep == 1 else vv.repeat_interleave(rep, dim=1)) for qq, kk, vv in sets]
                with sdpa_kernel([be]):
                    warm_up(lambda: F.scaled_dot_product_attention(*csets[0], is_causal=causal), 3)
                    c0 = torch.cuda.Event(enable_timing=True)
                    c1 = torch.cuda.Event(enable_timing=True)
                    host_lead()
                    c0.record(stream)
                    for i in range(10):
                        F.scaled_dot_product_attention(*csets[(3 + i) % len(csets)], is_causal=causal)
                    c1.record(stream)
                    torch.cuda.synchronize(dev)
                comparators[name + "_tflops"] = round(flops * 10 / (c0.elapsed_time(c1) / 1e3) / 1e12, 1)
            except Exception as exc:  # a backend may not support the shape
                comparators[name + "_tflops"] = f"unavailable: {type(exc).__name__}"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_attention_sample(S, D, causal, target_s=args.cpu_seconds)

    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/k/v per rank (no dataset in the reference for this path)",
        "config": attention_config(args.workload, world),
        "e2e": {
            "value": round(e2e_value, 1),
            "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "flash_atten.attention_forward_host on pinned host buffers (H2D q,k,v and D2H o inside the timed "
                   "region, pipelined with the kernels in 16 pieces)",
        },
        "roofline": peaks_entry(achieved, args.workload),
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "comparators": comparators,
    }
    if cpu is not None:
        cpu = dict(cpu)
        cpu.pop("seconds", None)
        result["cpu_baseline"] = cpu
    return result


# ---------------------------------------------------------------- decode
def run_decode(args, world, rank, local):
    """Split-KV decode step: one query row per head against a long resident K/V cache (HBM-bound)."""
    import _native
    from flash_atten import attention_forward_splitkv, splitkv_workspace_bytes

    B, Hq, Hkv, M, N, D = DECODE_WORKLOADS[args.workload]
    dev = torch.device("cuda", local)
    dtype = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    q = torch.randn(B, Hq, M, D, generator=g, device=dev, dtype=dtype)
    k = torch.randn(B, Hkv, N, D, generator=g, device=dev, dtype=dtype)
    v = torch.randn(B, Hkv, N, D, generator=g, device=dev, dtype=dtype)
    o = torch.empty_like(q)
    need, splits = splitkv_workspace_bytes(tuple(q.shape), tuple(k.shape), dtype)
    ws = torch.zeros(max(need, 256), device=dev, dtype=torch.uint8)  # counters start at zero
    kv_bytes = 2 * k.numel() * k.element_size()
    algo_bytes = kv_bytes + 2 * q.numel() * q.element_size()  # K, V read once; q read, o written
    stream = torch.cuda.current_stream(dev)

    def step(qq):
        return attention_forward_splitkv(qq, k, v, out=o, workspace=ws)

    warm_up(lambda: step(q), args.warmup)

    def graph_of(fn, n):
        """n calls of fn captured as one CUDA graph, the way a decode loop runs them: a step is ~50 us of
        device time, shorter than a Python call's host overhead, so calls issued one by one from Python
        would time the host."""
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(n):
                fn()
        torch.cuda.synchronize(dev)
        return graph

    steps_graph = graph_of(lambda: step(q), args.steps)
    steps_graph.replay()  # one untimed replay
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        host_lead()
        t0.record(stream)
        steps_graph.replay()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    elapsed_ms = max_over_ranks(t0.elapsed_time(t1), world)
    launch_ms = elapsed_ms / args.steps
    del steps_graph
    if _native.device_error():
        raise RuntimeError("device error during the timed region")
    value = sum_over_ranks(algo_bytes * args.steps, world) / (elapsed_ms / 1e3) / 1e9

    # e2e: each step's new query rows come from pinned host memory and its output goes back
    qh = q.cpu().pin_memory()
    oh = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    for _ in range(2):
        oh.copy_(step(qh.to(dev, non_blocking=True)), non_blocking=True)
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        oh.copy_(step(qh.to(dev, non_blocking=True)), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = sum_over_ranks(algo_bytes * args.steps, world) / (e2e_ms / 1e3) / 1e9

    comparators = {}
    if rank == 0 and not args.no_compare:
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        for name, be in (("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("torch_sdpa_flash", SDPBackend.FLASH_ATTENTION)):
            try:
                with sdpa_kernel([be]):
                    warm_up(lambda: F.scaled_dot_product_attention(q, k, v, enable_gqa=True), 3)
                    cgraph = graph_of(lambda: F.scaled_dot_product_attention(q, k, v, enable_gqa=True), 20)
                    cgraph.replay()
                    torch.cuda.synchronize(dev)
                    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    host_lead()
                    c0.record(stream)
                    cgraph.replay()
                    c1.record(stream)
                    torch.cuda.synchronize(dev)
                    del cgraph
                comparators[name + "_gbs"] = round(algo_bytes * 20 / (c0.elapsed_time(c1) / 1e3) / 1e9, 1)
            except Exception as exc:
                comparators[name + "_gbs"] = f"unavailable: {type(exc).__name__}"
    peak, source = measured_hbm_gbs()
    achieved = algo_bytes / (launch_ms / 1e3) / 1e9
    return {
        "metric": "split-KV decode attention, K/V cache bytes read per second",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q and K/V cache per rank",
        "config": {
            "workload": f"decode step B{B} Hq{Hq} Hkv{Hkv} {M} query row(s) against {N} cached keys D{D} bf16 "
                        f"per GPU, {splits} key splits",
            "global_batch": B * world,
            "seq_len": N,
            "parallelism": f"dp{world} (no collective)",
            "l2_policy": f"K/V cache {kv_bytes / 1e6:.0f} MB per step > 126 MB L2; no flush",
            "timing": "device time of the steps captured as one CUDA graph (comparators likewise)",
        },
        "e2e": {
            "value": round(e2e_value, 1),
            "unit": "GB/s",
            "h2d_bytes_per_step": q.numel() * q.element_size(),
            "d2h_bytes_per_step": o.numel() * o.element_size(),
            "api": "flash_atten.attention_forward_splitkv called from Python each step, with the query rows copied "
                   "from pinned host memory and the output copied back (the K/V cache stays resident)",
        },
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": f"{source} HBM copy bandwidth",
                     "traffic": committed_traffic(args.workload)},
        "gpu_launches": args.steps,  # one split kernel per step; its last CTAs merge the splits
        "clocks": clocks.summary(),
        "comparators": comparators,
    }


# ------------------------------------------------------------------- ttft
def run_ttft(args, world, rank, local):
    """Qwen2.5-7B-architecture prefill TTFT, tensor-parallel over the job's GPUs.

    Same seeded random weights for every tensor-parallel degree; NCCL all-reduce after o_proj and
    down_proj.  Three builds of the same decoder are timed: this repository's attention + GEMM, this
    repository's attention + cuBLAS, and torch SDPA (cuDNN) + cuBLAS (the same-box comparator)."""
    import ttft

    dev = torch.device("cuda", local)
    arch = ttft.KNOWN_ARCHS["Qwen/Qwen2.5-7B"]
    shard = ttft.build_model_shard(arch, world, rank, seed=0, device=dev)
    group = None
    out = {"model": "Qwen2.5-7B architecture, random N(0,0.02) bf16 weights", "tp": world, "batch": 1,
           "causal": True, "unit": "ms", "timing": "wall clock per prefill, synchronised, max over ranks"}
    builds = {
        "ours": ttft.Backends(attention="native", gemm="native"),
        "ours_norm_folded": ttft.Backends(attention="native", gemm="native", norm_fold=True),
        "ours_attention_cublas_gemm": ttft.Backends(attention="native", gemm="cublas"),
        "torch_cudnn_sdpa_cublas": ttft.Backends(attention="cudnn", gemm="cublas", elementwise="torch"),
    }
    fused = None
    if world > 1:
        # o_proj / down_proj GEMMs fused with their all-reduce over NVLink peer memory
        import _native
        from tp_allreduce import FusedGemmAllReduce

        fused = FusedGemmAllReduce(None, max_rows=max(args.ttft_lengths), cols=arch.hidden_size,
                                   dtype=torch.bfloat16, device=dev)
        builds["ours_fused_allreduce"] = ttft.Backends(attention="native", gemm="native", fused_allreduce=fused)
    for S in args.ttft_lengths:
        ids = ttft._make_random_input_ids(S, arch.vocab_size, dev, seed=S)
        row = {}
        for name, be in builds.items():
            try:
                samples = ttft.time_decoder_ttft_ms(shard, ids, be, repeats=args.ttft_repeats, warmups=1, group=group)
                row[name] = round(statistics.median(samples), 2)
            except Exception as exc:
                row[name] = f"unavailable: {type(exc).__name__}: {str(exc)[:80]}"
            if be.fused_allreduce is not None:
                # every rank learns whether any rank's fused call gave up on a bounded wait
                import torch.distributed as dist

                err = torch.tensor([float(_native.device_error())], device=dev)
                dist.all_reduce(err, op=dist.ReduceOp.MAX)
                if err.item():
                    row[name] = "unavailable: a fused all-reduce wait timed out"
                    del builds[name]
                    break
        # the all-native build again, as one CUDA graph per prompt length (host launch time removed)
        best = "ours_fused_allreduce" if "ours_fused_allreduce" in builds else "ours"
        graphed = None
        try:
            graphed = ttft.GraphedDecoder(shard, S, builds[best], group=group, device=dev)
            samples = ttft.time_decoder_ttft_ms(shard, ids, builds[best], repeats=args.ttft_repeats, warmups=1,
                                                group=group, graphed=graphed)
            row[best + "_cuda_graph"] = round(statistics.median(samples), 2)
        except Exception as exc:
            row[best + "_cuda_graph"] = f"unavailable: {type(exc).__name__}: {str(exc)[:80]}"
        finally:
            if graphed is not None:
                graphed.close()
                del graphed
        out[f"prompt_{S}"] = row
    if fused is not None:
        torch.cuda.synchronize(dev)
        barrier(world)
        fused.close()
    del shard
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ gemm arm
def run_gemm(args, world, rank, local):
    import _native
    import mma
    from mma import matmul

    M, K, N = gemm_shape(args.workload)
    dev = torch.device("cuda", local)
    dtype = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    # Rank r owns output column block r of an M x (N * world) product; A is replicated.
    a = (torch.randn(M, K, generator=g, device=dev) / K ** 0.5).to(dtype)
    b = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).to(dtype)
    flops = 2.0 * M * N * K
    stream = torch.cuda.current_stream(dev)
    operand_bytes = (M * K + K * N + M * N) * 2
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if operand_bytes < L2_BYTES * 2 else None
    c = torch.empty(M, N, device=dev, dtype=dtype)

    def timed_steps(fn, steps):
        """Device ms of `steps` calls, each after an L2 flush (small sizes), events around the call alone."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        host_lead()
        for i in range(steps):
            if flush is not None:
                flush.zero_()
            starts[i].record(stream)
            fn()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        return sum(s.elapsed_time(e) for s, e in zip(starts, ends))

    def ours():
        matmul(a, b)

    def flushed(fn):
        """A warm-up call the way timed_steps makes it, flush first: on B200 a 2048 x 3584 x 4608 matmul timed
        in the first loop to follow the flush measured 24 % slower than in later ones."""
        def call():
            if flush is not None:
                flush.zero_()
            fn()
        return call

    warm_up(flushed(ours), args.warmup)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        total_ms = timed_steps(ours, args.steps)
    barrier(world)
    total_ms = max_over_ranks(total_ms, world)
    if _native.device_error():
        raise RuntimeError("device error during the timed region")
    value = sum_over_ranks(flops * args.steps, world) / (total_ms / 1e3) / 1e12
    achieved = flops / (total_ms / args.steps / 1e3) / 1e12
    comparators = {}
    if rank == 0 and not args.no_compare:
        def cublas():
            torch.matmul(a, b, out=c)

        warm_up(flushed(cublas), 3)
        # As many calls as the timed region (at least 10), so a long run compares both under the power cap.
        n_cmp = max(10, args.steps)
        with ClockSampler(local) as cmp_clocks:
            ms = timed_steps(cublas, n_cmp)
        comparators["torch_matmul_cublas_tflops"] = round(flops * n_cmp / (ms / 1e3) / 1e12, 1)
        comparators["torch_matmul_cublas_clocks"] = cmp_clocks.summary()
    return {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)/sqrt(K)",
        "config": {"workload": f"matmul {M}x{K}x{N} (M x K x N) bf16 per GPU"
                               + (" (BASELINE config 4)" if M == K == N else ""),
                   "parallelism": f"dp{world} (output-column shards, A replicated; no collective)",
                   "l2_policy": "L2 flushed between steps" if flush is not None else "operands > L2"},
        "roofline": peaks_entry(achieved, args.workload),
        "gpu_launches": args.steps,
        "kernel_plan": list(mma.kernel_plan(M, N, K, dtype, device=dev)),
        "clocks": clocks.summary(),
        "comparators": comparators,
    }


# ------------------------------------------------------------- reference arm
def run_reference(args, world, rank):
    """The reference's CPU path (fp32 torch SDPA on CPU copies) as the benchmark arm; rank 0 only."""
    if rank != 0:
        return None
    B, Hq, Hkv, S, D, causal = WORKLOADS.get(args.workload, WORKLOADS["fa_s8192_noncausal"])
    import torch.nn.functional as F

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    probe = cpu_attention_sample(S, D, causal, target_s=1.0, max_heads=1)
    per_head_s = probe["seconds"]
    # Each step: a bounded sample of the workload sized so the whole run stays within a few minutes.
    budget_s = 150.0 / max(1, args.steps + args.warmup)
    heads = max(1, min(Hq, int(budget_s / max(per_head_s, 1e-6))))
    q, k, v = (torch.randn(1, heads, S, D, generator=g) for _ in range(3))
    for _ in range(args.warmup):
        F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        times.append(time.perf_counter() - t0)
    flops = attention_flops(1, heads, S, D, causal)
    value = flops * len(times) / sum(times) / 1e12
    sample = (f"{heads} (batch, head) unit(s) of the workload per step at S={S} D={D} causal={causal}, fp32 torch "
              "SDPA on CPU (the reference's oracle path, test_flash_atten.py:459-461, 498-499)")
    return {
        "metric": METRIC,
        "impl": "reference",
        "value": round(value, 4),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * sum(times) / len(times), 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded N(0,1)",
        "config": attention_config(args.workload if args.workload in WORKLOADS else "fa_s8192_noncausal", world),
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="fa_s8192_noncausal",
                    help="one of " + ", ".join(sorted(WORKLOADS) + sorted(GEMM_WORKLOADS) + sorted(DECODE_WORKLOADS))
                         + ", or gemm_<M>x<K>x<N>")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-compare", action="store_true", help="skip the torch comparators")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target length of the CPU baseline sample")
    ap.add_argument("--no-ttft", action="store_true", help="skip the Qwen2.5-7B-architecture TTFT measurement")
    ap.add_argument("--ttft-lengths", type=int, nargs="+", default=[2048, 8192])
    ap.add_argument("--ttft-repeats", type=int, default=3)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.workload not in WORKLOADS and args.workload not in DECODE_WORKLOADS and gemm_shape(args.workload) is None:
        ap.error(f"unknown workload {args.workload}")
    if args.impl == "reference":
        # CPU-only arm: no process group; ranks other than 0 exit without work.
        world = int(os.environ.get("WORLD_SIZE", "1"))
        result = run_reference(args, world, int(os.environ.get("RANK", "0")))
        if result is not None:
            print(json.dumps(result), flush=True)
        return
    world, rank, local = setup_dist(args)
    result = None
    try:
        if gemm_shape(args.workload) is not None:
            result = run_gemm(args, world, rank, local)
        elif args.workload in DECODE_WORKLOADS:
            result = run_decode(args, world, rank, local)
        else:
            result = run_attention(args, world, rank, local)
            torch.cuda.empty_cache()
            if not args.no_ttft:
                ttft_result = run_ttft(args, world, rank, local)
                if result is not None:
                    result["ttft"] = ttft_result
    finally:
        if world > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()
    # After the process group is gone, so the JSON line is the last thing rank 0 writes.
    if rank == 0 and result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
