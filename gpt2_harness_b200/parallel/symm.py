"""Symmetric device buffers mapped into every rank over NVLink (CUDA IPC).

Each rank allocates a buffer of the same size with its own ``cudaMalloc`` and
publishes a CUDA IPC handle through the process group; every rank opens all
peers' handles. A native kernel then holds one device pointer per rank and
reads or writes any peer's buffer with ordinary loads/stores, which NVSwitch
routes over NVLink 5. This is the data plane of the fused collectives; the
process group (NCCL or gloo) is only the control plane used to exchange the
handles once.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.ops import native as N

__all__ = ["SymmetricBuffer", "MulticastBuffer", "multicast_supported", "wrap_device_pointer"]

_TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<V2", torch.int32: "<i4", torch.int64: "<i8",
            torch.uint8: "|u1"}


class _CudaArray:
    """Minimal ``__cuda_array_interface__`` exporter around a raw pointer."""

    def __init__(self, ptr: int, numel: int, typestr: str) -> None:
        self.__cuda_array_interface__ = {
            "shape": (numel,),
            "typestr": typestr,
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }


def wrap_device_pointer(ptr: int, numel: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A torch tensor aliasing ``numel`` elements at ``ptr`` (no copy, no
    ownership: the caller keeps the allocation alive)."""
    if dtype == torch.bfloat16:
        raw = torch.as_tensor(_CudaArray(ptr, numel, "<i2"), device=device)
        return raw.view(torch.bfloat16)
    return torch.as_tensor(_CudaArray(ptr, numel, _TYPESTR[dtype]), device=device)


class SymmetricBuffer:
    """One equally sized buffer per rank, all mapped into this process.

    Attributes:
        local: this rank's buffer as a flat uint8 tensor.
        peer_ptrs: python list of every rank's buffer address in THIS process.
        peer_ptrs_dev: the same as an int64 device tensor (kernel argument).
    """

    def __init__(self, nbytes: int, group=None, device: Optional[torch.device] = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = int((nbytes + 255) // 256 * 256)
        L = N.lib()
        self.ptr = L.symm_alloc(self.nbytes)
        handle = L.ipc_handle(self.ptr)
        if not handle:
            raise RuntimeError("cudaIpcGetMemHandle failed")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.peer_ptrs = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peer_ptrs.append(self.ptr)
            else:
                p = L.ipc_open(h)
                self._opened.append(p)
                self.peer_ptrs.append(p)
        self.peer_ptrs_dev = torch.tensor(self.peer_ptrs, dtype=torch.int64, device=self.device)
        self.local = wrap_device_pointer(self.ptr, self.nbytes, torch.uint8, self.device)

    def view(self, dtype: torch.dtype, numel: Optional[int] = None, offset_bytes: int = 0) -> torch.Tensor:
        esz = torch.tensor([], dtype=dtype).element_size()
        n = (self.nbytes - offset_bytes) // esz if numel is None else numel
        return wrap_device_pointer(self.ptr + offset_bytes, n, dtype, self.device)

    def close(self) -> None:
        L = N.lib()
        for p in self._opened:
            L.ipc_close(p)
        self._opened = []
        if self.ptr:
            torch.cuda.synchronize(self.device)
            L.symm_free(self.ptr)
            self.ptr = 0


def multicast_supported(device: Optional[torch.device] = None) -> bool:
    """Whether this GPU can bind memory to an NVLink multicast object (an
    NVSwitch system with a driver that exposes multicast)."""
    if not torch.cuda.is_available():
        return False
    try:
        from torch._C._distributed_c10d import _SymmetricMemory
        from torch._C._autograd import DeviceType
    except ImportError:
        return False
    idx = (device or torch.device("cuda", torch.cuda.current_device())).index or 0
    return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, idx))


class MulticastBuffer:
    """A symmetric buffer that is also bound to an NVLink multicast object.

    Same interface as :class:`SymmetricBuffer` (``local``, ``peer_ptrs``,
    ``peer_ptrs_dev``, ``view``, ``close``) plus ``mc_ptr``: an address whose
    ``multimem`` loads return the element summed over every rank's copy (the
    reduction runs in the NVSwitch) and whose ``multimem`` stores land in every
    rank's copy. Allocation, handle exchange and the multicast binding are
    torch's symmetric memory (``torch.distributed._symmetric_memory``,
    cuMem-backed); the kernels that use the addresses are this package's.
    """

    def __init__(self, nbytes: int, group=None, device: Optional[torch.device] = None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group or dist.group.WORLD
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = int((nbytes + 255) // 256 * 256)
        if not multicast_supported(self.device):
            raise RuntimeError("NVLink multicast is not available on this GPU")
        self._tensor = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=self.device)
        self._tensor.zero_()
        self._handle = symm_mem.rendezvous(self._tensor, self.group)
        mc = int(self._handle.multicast_ptr)
        if not mc:
            raise RuntimeError("symmetric memory has no multicast address on this system")
        # The handle's addresses are those of each rank's whole allocation
        # block; the tensor may sit at an offset inside it (pooled allocation),
        # the same offset on every rank.
        self.ptr = self._tensor.data_ptr()
        bases = [int(p) for p in self._handle.buffer_ptrs]
        off = self.ptr - bases[self.rank]
        if off < 0 or off + self.nbytes > int(self._handle.buffer_size) or off % 16:
            raise RuntimeError(f"symmetric tensor outside its block (offset {off}, "
                               f"block {self._handle.buffer_size} B)")
        self.mc_ptr = mc + off
        self.peer_ptrs = [b + off for b in bases]
        self.peer_ptrs_dev = torch.tensor(self.peer_ptrs, dtype=torch.int64, device=self.device)
        self.local = self._tensor

    def view(self, dtype: torch.dtype, numel: Optional[int] = None, offset_bytes: int = 0) -> torch.Tensor:
        esz = torch.tensor([], dtype=dtype).element_size()
        n = (self.nbytes - offset_bytes) // esz if numel is None else numel
        return self._tensor[offset_bytes:offset_bytes + n * esz].view(dtype)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self._handle = None
        self._tensor = None
        self.local = None


class P2PAllReducer:
    """Standalone fused peer-memory all-reduce over a symmetric fp32 buffer.

    ``tensor`` is this rank's buffer (write the data there); ``all_reduce(n,
    scale)`` reduces its first ``n`` elements across the group in one kernel
    (reduce-scatter by peer loads, scale, all-gather by peer stores, per-CTA
    flags with bounded waits) on the current stream.
    """

    def __init__(self, nbytes: int, group=None, device: Optional[torch.device] = None, nblocks: int = 128) -> None:
        self.data = SymmetricBuffer(nbytes, group, device)
        self.flags = SymmetricBuffer(N.lib().comm_flag_words() * 4, group, device)
        self.rank, self.world, self.device = self.data.rank, self.data.world, self.data.device
        self.tensor = self.data.view(torch.float32)
        self.nblocks = nblocks
        self.epoch = 0
        self.counter = torch.zeros(1, dtype=torch.int64, device=self.device)

    def all_reduce(self, numel: Optional[int] = None, scale: float = 1.0) -> torch.Tensor:
        n = self.tensor.numel() if numel is None else int(numel)
        self.epoch += 1
        N.lib().allreduce_p2p(self.data.peer_ptrs_dev.data_ptr(), self.flags.peer_ptrs_dev.data_ptr(), self.rank,
                              self.world, 0, n, 0, float(scale), self.epoch & 0xFFFFFFFF, self.counter.data_ptr(),
                              N.error_word().data_ptr(), self.nblocks, 2_000_000_000, -1,
                              torch.cuda.current_stream(self.device).cuda_stream)
        return self.tensor[:n]

    def close(self) -> None:
        self.data.close()
        self.flags.close()
