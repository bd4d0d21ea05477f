"""One-shot all-reduce over NVLink peer memory (``cb_peer_allreduce``).

For the small ``[T, hidden]`` 16-bit partial outputs of row-parallel projections
in tensor-parallel decode. Each rank allocates one symmetric area, exports it as
a CUDA IPC handle, and maps every peer's area; the handles travel through the
torch.distributed process group (``all_gather_object``). Every rank must make
the same sequence of calls with the same element counts.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib as L
from .ops import dtype_code


class PeerAllReduce:
    def __init__(self, max_elems: int, group=None, device: torch.device | None = None):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_elems = (int(max_elems) + 7) // 8 * 8  # slots start on 16-byte boundaries
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        lib = L.load()
        nbytes = lib.cb_symm_bytes(self.world, self.max_elems)
        if nbytes == 0:
            raise ValueError(f"unsupported world size {self.world}")
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.check("cb_symm_alloc", lib.cb_symm_alloc(nbytes, ctypes.byref(own)))
            handle = (ctypes.c_ubyte * 64)()
            L.check("cb_ipc_get_handle", lib.cb_ipc_get_handle(own, handle))
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            areas, self._opened = [], []
            for r, h in enumerate(handles):
                if r == self.rank:
                    areas.append(own.value)
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                L.check("cb_ipc_open_handle", lib.cb_ipc_open_handle(hb, ctypes.byref(p)))
                areas.append(p.value)
                self._opened.append(p)
        self._own = own
        self._areas = (ctypes.c_void_p * self.world)(*areas)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.dtype not in (torch.bfloat16, torch.float16) or not x.is_contiguous():
            raise ValueError("peer all-reduce takes a contiguous bf16/f16 tensor")
        if x.numel() > self.max_elems:
            raise ValueError(f"{x.numel()} elements exceed the symmetric area ({self.max_elems})")
        if out is None:
            out = torch.empty_like(x)
        if out.dtype != x.dtype or not out.is_contiguous() or out.numel() != x.numel():
            raise ValueError("out must be a contiguous tensor like x")
        code = L.load().cb_peer_allreduce(x.data_ptr(), out.data_ptr(), x.numel(), dtype_code(x.dtype), self._areas,
                                          self.rank, self.world, self.max_elems, self.status.data_ptr(),
                                          torch.cuda.current_stream(x.device).cuda_stream)
        L.check("cb_peer_allreduce", code)
        return out

    def close(self):
        """Unmaps the peers' areas and frees this rank's (all ranks call it together)."""
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = L.load()
        for p in self._opened:
            lib.cb_ipc_close_handle(p)
        dist.barrier(group=self.group)
        lib.cb_symm_free(self._own)
        self._own = None
