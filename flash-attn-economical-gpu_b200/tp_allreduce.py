"""Tensor-parallel GEMM + all-reduce in one kernel over NVLink peer memory.

`FusedGemmAllReduce(group, max_rows, cols, dtype, device)` owns, on every
rank of a process group, the buffers the fused kernel (`fab_gemm_allreduce`)
reads and writes -- an inbox for the partial tiles this rank owns, the
reduced output and a counter array -- and maps the other ranks' buffers
into this process with CUDA IPC.  Calling it with this rank's a [M, K] and
b [K, cols] returns sum over ranks of a_r @ b_r, the o_proj / down_proj
product followed by an all-reduce in a tensor-parallel decoder, computed as
the tiles come off the tensor cores instead of after the GEMM.

Every rank must make the same sequence of calls with the same M and K (the
decoder's layers do).  The returned tensor is a view of the output buffer,
valid until the next call.  Built on plain peer loads and stores, no NVLink
multicast.
"""
from __future__ import annotations

import ctypes

import torch

import _native

HANDLE_BYTES = 64


class FusedGemmAllReduce:
    def __init__(self, group, max_rows: int, cols: int, dtype: torch.dtype, device: torch.device):
        import torch.distributed as dist

        if group is None and dist.is_available() and dist.is_initialized():
            group = dist.group.WORLD
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if not 1 <= self.world <= _native.MAX_TP_RANKS:
            raise ValueError(f"FusedGemmAllReduce supports 1..{_native.MAX_TP_RANKS} ranks, got {self.world}")
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("FusedGemmAllReduce computes in bf16 or fp16")
        self.max_rows, self.cols, self.dtype, self.device = int(max_rows), int(cols), dtype, device
        per_owner, inbox_bytes, counter_bytes = self._layout(self.max_rows)
        self.inbox = torch.empty(inbox_bytes, device=device, dtype=torch.uint8)
        self.out = torch.empty(self.max_rows, self.cols, device=device, dtype=dtype)
        self.counters = torch.zeros(counter_bytes // 8, device=device, dtype=torch.int64)
        self.calls = 0
        self._mapped: list[int] = []  # bases this process mapped and must unmap
        local = [self.inbox.data_ptr(), self.out.data_ptr(), self.counters.data_ptr()]
        if self.world == 1:
            self.ptrs = [[p] for p in local]
        else:
            exports = []
            with torch.cuda.device(device):
                for p in local:
                    handle = (ctypes.c_char * HANDLE_BYTES)()
                    offset = ctypes.c_size_t(0)
                    _native.check(_native.lib.fab_ipc_export(p, handle, ctypes.byref(offset)), "fab_ipc_export")
                    exports.append((bytes(handle), offset.value))
            everyone: list = [None] * self.world
            dist.all_gather_object(everyone, exports, group=group)
            self.ptrs = [[0] * self.world for _ in range(3)]
            with torch.cuda.device(device):
                for r in range(self.world):
                    for i in range(3):
                        if r == self.rank:
                            self.ptrs[i][r] = local[i]
                            continue
                        handle, offset = everyone[r][i]
                        base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
                        _native.check(_native.lib.fab_ipc_import(handle, offset, ctypes.byref(base),
                                                                  ctypes.byref(ptr)), "fab_ipc_import")
                        self._mapped.append(base.value)
                        self.ptrs[i][r] = ptr.value
            # nobody writes into a peer before every peer has mapped everything
            dist.barrier(group=group)

    def _layout(self, rows: int) -> tuple[int, int, int]:
        per_owner, inbox, counters = ctypes.c_int(0), ctypes.c_size_t(0), ctypes.c_size_t(0)
        _native.check(_native.lib.fab_gemm_allreduce_layout(rows, self.cols, self.world, ctypes.byref(per_owner),
                                                            ctypes.byref(inbox), ctypes.byref(counters)),
                      "fab_gemm_allreduce_layout")
        return per_owner.value, inbox.value, counters.value

    def __call__(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        if a.dtype != self.dtype or b.dtype != self.dtype or a.device != self.device or b.device != self.device:
            raise ValueError("FusedGemmAllReduce: a and b must be on the buffers' device in their dtype")
        M, K = a.shape
        Kb, N = b.shape
        if Kb != K or N != self.cols or M > self.max_rows:
            raise ValueError(f"FusedGemmAllReduce: shapes a={tuple(a.shape)} b={tuple(b.shape)} do not fit "
                             f"rows<={self.max_rows}, cols={self.cols}")
        if a.stride(1) != 1 or b.stride(1) != 1 or a.data_ptr() % 16 or b.data_ptr() % 16 or \
                (a.stride(0) * a.element_size()) % 16 or (b.stride(0) * b.element_size()) % 16:
            a, b = a.contiguous(), b.contiguous()
        self.calls += 1
        p = _native.FabGemmAllreduceParams()
        p.a, p.b = a.data_ptr(), b.data_ptr()
        p.lda, p.ldb, p.ldo = a.stride(0), b.stride(0), self.cols
        p.M, p.N, p.K = M, N, K
        p.in_dtype = _native.dtype_code(self.dtype)
        p.world, p.rank = self.world, self.rank
        for r in range(self.world):
            p.inbox[r], p.out[r], p.counters[r] = self.ptrs[0][r], self.ptrs[1][r], self.ptrs[2][r]
        with torch.cuda.device(self.device):
            stream = ctypes.c_void_p(_native.current_stream_handle(self.device))
            _native.check(_native.lib.fab_gemm_allreduce(ctypes.byref(p), stream), "fab_gemm_allreduce")
        return self.out[:M]

    def close(self) -> None:
        """Unmap the peers' buffers (after every rank's last call has completed)."""
        with torch.cuda.device(self.device):
            for base in self._mapped:
                _native.lib.fab_ipc_close(base)
        self._mapped = []
