"""Symmetric device buffers shared across the ranks of one node through CUDA IPC.

Each rank allocates one zeroed block (``b2m_symm_alloc``), exports its IPC handle,
gathers every rank's handle over the process group and opens the peers' blocks
(``b2m_ipc_open``, lazy peer access).  Named sub-buffers sit at identical offsets
on every rank, so ``peer(name, r)`` is rank r's copy of ``name``.  Set-up only:
nothing here runs inside the timed forward.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

ALIGN = 256


class _CudaArray:
    """Minimal ``__cuda_array_interface__`` wrapper so torch can view a raw device pointer."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


_TYPESTR = {torch.uint8: "|u1", torch.int32: "<i4", torch.float32: "<f4", torch.bfloat16: "<u2",
            torch.float8_e4m3fn: "|u1"}


class SymmetricWorkspace:
    def __init__(self, layout: dict[str, int], group=None, device=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.offsets: dict[str, int] = {}
        off = 0
        for name, nbytes in layout.items():
            self.offsets[name] = off
            off += (int(nbytes) + ALIGN - 1) // ALIGN * ALIGN
        self.nbytes = off
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            _lib.call("b2m_symm_alloc", self.nbytes, ctypes.byref(ptr))
            self.base = ptr.value
            handle = ctypes.create_string_buffer(64)
            _lib.call("b2m_ipc_handle", self.base, handle)
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            self.bases: list[int] = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self.base)
                else:
                    peer = ctypes.c_void_p()
                    _lib.call("b2m_ipc_open", ctypes.create_string_buffer(h, 64), ctypes.byref(peer))
                    self.bases.append(peer.value)
        self._closed = False

    def peer(self, name: str, r: int) -> int:
        return self.bases[r] + self.offsets[name]

    def local(self, name: str) -> int:
        return self.peer(name, self.rank)

    def tensor(self, name: str, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        t = torch.as_tensor(_CudaArray(self.local(name), tuple(shape), _TYPESTR[dtype]), device=self.device)
        return t.view(dtype) if t.dtype != dtype else t

    def close(self) -> None:
        """Collective: every rank must call it; nobody frees before all peers have unmapped."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        self.dist.barrier(group=self.group)
        for r, b in enumerate(self.bases):
            if r != self.rank:
                _lib.call("b2m_ipc_close", b)
        self.dist.barrier(group=self.group)
        _lib.call("b2m_symm_free", self.base)
        self._closed = True


def ptr_array(ptrs: list[int]) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr
