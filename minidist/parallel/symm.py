"""Symmetric peer memory over CUDA IPC: every rank of a group maps every peer's buffer.

A :class:`SymmBuffer` is one device allocation per rank (``cudaMalloc``) plus a
small flag allocation, whose IPC handles are exchanged through the process
group and opened on every peer.  Kernels receive the array of per-rank base
pointers and read or write any rank's memory directly over NVLink/NVSwitch.

Requirements checked at construction (otherwise :func:`communicator` returns
``None`` and callers use NCCL): CUDA + NCCL process group, every member on this
node, peer access between every pair of devices, group size <= 8.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from .. import comm
from ..ops import _native as nat

_SIGS = {
    "md_symm_alloc": "i:lpp",
    "md_symm_open": "i:pp",
    "md_symm_close": "i:p",
    "md_symm_free": "i:p",
    "md_symm_max_world": "i:",
    "md_symm_flag_bytes": "l:",
    "md_allreduce_ctas": "i:li",
}
for _n, _s in _SIGS.items():
    nat.declare(_n, _s)

_HANDLE = 64
_live: list["SymmBuffer"] = []
_comms: dict[tuple, "Communicator | None"] = {}


class _CudaArray:
    """Minimal ``__cuda_array_interface__`` owner used to view raw device memory as a tensor."""

    def __init__(self, ptr: int, numel: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


_TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<V2", torch.uint8: "|u1", torch.int32: "<i4"}


class SymmBuffer:
    """``nbytes`` of peer-mapped memory on each rank of ``group``."""

    def __init__(self, group, nbytes: int):
        self.group = group
        self.world = comm.get_world_size(group)
        self.rank = comm.get_rank(group)
        self.nbytes = int(nbytes)
        lib = nat.lib()
        self.device = torch.device("cuda", torch.cuda.current_device())
        own = ctypes.c_void_p()
        own_flags = ctypes.c_void_p()
        handles = (ctypes.c_ubyte * (2 * _HANDLE))()
        nat.check(lib.md_symm_alloc(self.nbytes, ctypes.byref(own), ctypes.addressof(handles)), "md_symm_alloc")
        flag_bytes = lib.md_symm_flag_bytes()
        nat.check(lib.md_symm_alloc(flag_bytes, ctypes.byref(own_flags), ctypes.addressof(handles) + _HANDLE),
                  "md_symm_alloc(flags)")
        mine = torch.tensor(bytearray(handles), dtype=torch.uint8, device=self.device)
        everyone = torch.empty(self.world * 2 * _HANDLE, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(everyone, mine, group=group)
        table = everyone.view(self.world, 2 * _HANDLE).cpu()
        self.ptrs: list[int] = []
        self.flag_ptrs: list[int] = []
        self._opened: list[int] = []
        for r in range(self.world):
            if r == self.rank:
                self.ptrs.append(own.value)
                self.flag_ptrs.append(own_flags.value)
                continue
            row = bytes(table[r].tolist())
            for k, dst in ((0, self.ptrs), (1, self.flag_ptrs)):
                buf = (ctypes.c_ubyte * _HANDLE).from_buffer_copy(row[k * _HANDLE:(k + 1) * _HANDLE])
                p = ctypes.c_void_p()
                nat.check(lib.md_symm_open(ctypes.addressof(buf), ctypes.byref(p)), "md_symm_open")
                dst.append(p.value)
                self._opened.append(p.value)
        self._own = (own.value, own_flags.value)
        self.closed = False
        _live.append(self)
        dist.barrier(group=group)

    def view(self, dtype: torch.dtype, byte_offset: int, numel: int) -> torch.Tensor:
        """Tensor over this rank's own buffer (no copy)."""
        if byte_offset + numel * dtype.itemsize > self.nbytes:
            raise ValueError("view exceeds the symmetric buffer")
        ptr = self.ptrs[self.rank] + byte_offset
        if dtype == torch.bfloat16:
            raw = torch.as_tensor(_CudaArray(ptr, numel, "<i2"), device=self.device)
            return raw.view(torch.bfloat16)
        return torch.as_tensor(_CudaArray(ptr, numel, _TYPESTR[dtype]), device=self.device)

    def close(self) -> None:
        if self.closed:
            return
        self.closed = True
        lib = nat.lib()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib.md_symm_close(p)
        if comm.is_distributed():
            dist.barrier(group=self.group)
        for p in self._own:
            lib.md_symm_free(p)


class Communicator:
    """Peer-memory state for one process group: its named symmetric buffers.  (Barrier epochs
    are counted on the device, per flag page and channel, by the kernels themselves.)"""

    def __init__(self, group, ranks: list[int]):
        self.group = group
        self.ranks = list(ranks)
        self.world = comm.get_world_size(group)
        self.rank = comm.get_rank(group)
        self.scratch: dict[str, SymmBuffer] = {}

    def zeroed_buffer(self, name: str, nbytes: int) -> SymmBuffer:
        """Like :meth:`buffer`, but a new allocation is zero-filled on every rank before any
        rank can use it (flag pages whose epochs must start below 1)."""
        b = self.scratch.get(name)
        if b is not None and b.nbytes >= nbytes:
            return b
        b = self.buffer(name, nbytes)
        b.view(torch.uint8, 0, b.nbytes).zero_()
        torch.cuda.synchronize(b.device)
        dist.barrier(group=self.group)
        return b

    def buffer(self, name: str, nbytes: int) -> SymmBuffer:
        """A named symmetric buffer of at least ``nbytes`` (collective on first use / growth)."""
        b = self.scratch.get(name)
        if b is None or b.nbytes < nbytes:
            if b is not None:
                b.close()
            b = SymmBuffer(self.group, nbytes)
            self.scratch[name] = b
        return b


def _same_node(group) -> bool:
    world = comm.get_world_size(group)
    lws = os.environ.get("LOCAL_WORLD_SIZE")
    if lws is not None and int(lws) == int(os.environ.get("WORLD_SIZE", "1")):
        return True
    host = torch.tensor(list(os.uname().nodename.encode()[:64].ljust(64, b"\0")), dtype=torch.uint8,
                        device=torch.device("cuda", torch.cuda.current_device()))
    allh = torch.empty(world * 64, dtype=torch.uint8, device=host.device)
    dist.all_gather_into_tensor(allh, host, group=group)
    rows = allh.view(world, 64).cpu()
    return all(torch.equal(rows[0], rows[i]) for i in range(world))


def supported(group) -> bool:
    if not (torch.cuda.is_available() and comm.is_distributed() and nat.available()):
        return False
    if dist.get_backend(group) != "nccl":
        return False
    world = comm.get_world_size(group)
    if world < 2 or world > nat.lib().md_symm_max_world():
        return False
    if os.environ.get("MINIDIST_PEER_MEMORY", "1") in ("0", "false", "no"):
        return False
    return _same_node(group)


def communicator(group, ranks) -> Communicator | None:
    """Shared :class:`Communicator` for ``group`` (``None`` where peer memory is unavailable)."""
    key = tuple(ranks)
    if key not in _comms:
        _comms[key] = Communicator(group, ranks) if supported(group) else None
    return _comms[key]


def release_all() -> None:
    """Unmap and free every symmetric buffer (collective; called by shutdown_distributed)."""
    while _live:
        _live.pop().close()
    _comms.clear()
