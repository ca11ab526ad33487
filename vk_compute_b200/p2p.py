"""NVLink peer all-gather and all-reduce for the sharded decoder chain.

`PeerGather` allocates, on every rank of a torch.distributed group (one GPU
per rank, one node), one device region holding named fp32 "full" buffers and
an arrival-counter array, exports it through CUDA IPC, and maps every other
rank's region into this rank's device (plain peer memory).  `gather(name,
part)` then runs the library's all-gather kernel: this rank's slice is stored
directly into every rank's copy of the buffer, and the kernel returns on the
GPU once all slices have arrived (bounded wait; see vkc_allgather_p2p).  No
collective library is on the data path, so a gather is one small kernel launch
that can be captured in a CUDA graph.  `allreduce(name, part, residual, out)`
stores `part` into this rank's slot of every rank's buffer [world][n] and
writes out = residual + the slots summed in rank order.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from ._lib import check, lib

_ALIGN = 256


class _DeviceRange:
    """A device range presented to torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, nfloats: int):
        self.__cuda_array_interface__ = {"shape": (nfloats,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3}


class PeerGather:
    def __init__(self, sizes: dict[str, int], device, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device)
        names = sorted(sizes)
        # region layout: counters, then each buffer, 256-byte aligned
        offs, at = {}, (4 * self.world + _ALIGN - 1) // _ALIGN * _ALIGN
        for n in names:
            offs[n] = at
            at += (4 * sizes[n] + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = at
        with torch.cuda.device(self.device):
            ptr = C.c_void_p()
            handle = (C.c_char * 64)()
            check(lib().vkc_ipc_alloc(self.nbytes, C.byref(ptr), handle))
            self.base = ptr.value
            everyone: list = [None] * self.world
            dist.all_gather_object(everyone, bytes(handle), group=group)
            self.peer_bases = []
            for r in range(self.world):
                if r == self.rank:
                    self.peer_bases.append(self.base)
                    continue
                p = C.c_void_p()
                check(lib().vkc_ipc_open(everyone[r], C.byref(p)))
                self.peer_bases.append(p.value)
            region = torch.as_tensor(_DeviceRange(self.base, self.nbytes // 4), device=self.device)
            self.counters = region[: self.world].view(torch.int32)
            self.buffers = {n: region[offs[n] // 4: offs[n] // 4 + sizes[n]] for n in names}
            self.dsts = {n: torch.tensor([b + offs[n] for b in self.peer_bases], dtype=torch.int64,
                                         device=self.device) for n in names}
            self.ctr_ptrs = torch.tensor(self.peer_bases, dtype=torch.int64, device=self.device)
            self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._gather_step = None
            self._region = region
            torch.cuda.synchronize(self.device)
        dist.barrier(group=group)  # every rank has mapped every region (counters start at zero)

    def gather(self, name: str, part: torch.Tensor) -> torch.Tensor:
        full = self.buffers[name]
        n = part.numel()
        if full.numel() != n * self.world:
            raise ValueError(f"{name}: slice of {n} for a buffer of {full.numel()} over {self.world} ranks")
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().vkc_allgather_p2p(part.data_ptr(), self.dsts[name].data_ptr(), self.ctr_ptrs.data_ptr(), n,
                                      self.rank, self.world, self.status.data_ptr(), st))
        return full

    def rmsnorm_gemv_gather(self, name: str, w, x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-6,
                            rms_dim: int | None = None) -> torch.Tensor:
        """Row-sharded RmsNorm-GEMV with the all-gather in its epilogue
        (vkc_rmsnorm_gemv_gather, then vkc_gather_wait): this rank's w (its
        rows of the matrix, w.N outputs) writes its outputs at rank * w.N of
        every rank's buffers[name]; returns buffers[name] once every rank's
        part has arrived (on the GPU).  Uses the counters of this PeerGather:
        do not mix with gather()/allreduce() on the same instance."""
        full = self.buffers[name]
        if full.numel() != w.N * self.world:
            raise ValueError(f"{name}: {full.numel()} floats for {w.N} outputs x {self.world} ranks")
        if self._gather_step is None:
            self._gather_step = torch.zeros(1, dtype=torch.int32, device=self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        ptr = lambda t: t.data_ptr() if t is not None else None
        check(lib().vkc_rmsnorm_gemv_gather(w.bits, w.packed.data_ptr(), ptr(w.scale), ptr(w.zero), x.data_ptr(),
                                            gamma.data_ptr(), self.dsts[name].data_ptr(), self.rank, self.world,
                                            self.rank * w.N, w.N, w.K, eps, rms_dim or w.K, st))
        check(lib().vkc_gather_wait(self.ctr_ptrs.data_ptr(), self.rank, self.world, self._gather_step.data_ptr(),
                                    self.status.data_ptr(), st))
        return full

    def allreduce(self, name: str, part: torch.Tensor, residual: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out = residual + sum over ranks of `part`; buffers[name] holds the
        world partial slots ([world][n])."""
        slots = self.buffers[name]
        n = part.numel()
        if slots.numel() != n * self.world or residual.numel() != n or out.numel() != n:
            raise ValueError(f"{name}: vector of {n} for {slots.numel()} slot floats over {self.world} ranks")
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().vkc_allreduce_residual_p2p(part.data_ptr(), self.dsts[name].data_ptr(), self.ctr_ptrs.data_ptr(),
                                               n, self.rank, self.world, residual.data_ptr(), out.data_ptr(),
                                               self.status.data_ptr(), st))
        return out

    def peer_input(self, name: str, save: torch.Tensor | None = None):
        """The fused-consumer descriptor of buffers[name] ([world][n] 8-byte
        words, i.e. 2*world*n floats of the region, filled by ops.gemv_peer
        with dsts[name])."""
        from .ops import PeerInput

        return PeerInput(self.buffers[name].data_ptr(), save.data_ptr() if save is not None else None, self.rank,
                         self.world)

    def timed_out(self) -> bool:
        """True if a wait of any gather so far ran out (reads the device)."""
        return bool(int(self.status.item()) & 8)

    def close(self) -> None:
        """Unmaps the peers' regions and frees this rank's (after a device sync
        and a barrier, so no rank is still writing here)."""
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for r, b in enumerate(self.peer_bases):
                if r != self.rank:
                    check(lib().vkc_ipc_close(b))
            self.buffers = {}
            self._region = None
            self.counters = None
            check(lib().vkc_ipc_free(self.base))
        self.base = None
