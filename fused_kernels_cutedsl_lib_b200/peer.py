"""Peer memory shared by the ranks of one node (host side of ``csrc/peer.cu``).

:class:`PeerArena` allocates one zero-filled device buffer per rank through the
library, exchanges CUDA IPC handles over the process group and maps every
peer's buffer, so that kernels can store straight into other GPUs' memory at
the same offsets (plain stores over NVLink; no multicast objects, no NVLS).
Regions are carved at identical offsets on every rank: ``region(name, shape)``
returns the local torch view, ``peer_ptrs(name, offset_elems)`` the other
ranks' addresses of the same element. :meth:`barrier` is the stage barrier of
``fk_peer_barrier`` on the current stream.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _native

_ALIGN = 256


class _CudaArray:
    """Zero-copy torch view of raw device memory (``__cuda_array_interface__``)."""

    _TYPESTR = {torch.int16: "<i2", torch.int32: "<i4", torch.float32: "<f4"}

    def __init__(self, ptr: int, shape, dtype: torch.dtype):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": self._TYPESTR[dtype], "version": 3, "strides": None}


def _view(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    if dtype == torch.bfloat16:  # no bf16 typestr: view the memory as int16, then reinterpret
        return torch.as_tensor(_CudaArray(ptr, shape, torch.int16), device=device).view(torch.bfloat16)
    return torch.as_tensor(_CudaArray(ptr, shape, dtype), device=device)


class PeerArena:
    """One IPC-shared device buffer per rank with named regions at equal offsets."""

    def __init__(self, nbytes: int, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = _native.load()
        self.nbytes = (int(nbytes) + _ALIGN - 1) // _ALIGN * _ALIGN + 2 * _ALIGN
        base = ctypes.c_void_p()
        _native.check(lib.fk_peer_alloc(self.nbytes, ctypes.byref(base)))
        self.base = int(base.value)
        hb = lib.fk_ipc_handle_bytes()
        handle = (ctypes.c_char * hb)()
        _native.check(lib.fk_ipc_get_handle(ctypes.c_void_p(self.base), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases = []
        for r in range(self.world):
            if r == self.rank:
                self.bases.append(self.base)
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * hb).from_buffer_copy(handles[r])
            _native.check(lib.fk_ipc_open(buf, ctypes.byref(p)))
            self.bases.append(int(p.value))
        # barrier state at offset 0: [counter][pad][flags: world int32]
        self._counter = self.base
        self._flags_off = 64
        self._next = 2 * _ALIGN
        self._regions: dict = {}
        self._peer_flags = (ctypes.c_void_p * self.world)(
            *[b + self._flags_off for b in self.bases])

    def region(self, name: str, shape, dtype=torch.bfloat16) -> torch.Tensor:
        """Local view of a named region (allocated at the same offset on every rank)."""
        if name not in self._regions:
            elem = torch.empty((), dtype=dtype).element_size()
            size = math.prod(shape) * elem
            off = self._next
            if off + size > self.nbytes:
                raise ValueError(f"peer arena too small: {name} needs {size} bytes at {off} of {self.nbytes}")
            self._next = (off + size + _ALIGN - 1) // _ALIGN * _ALIGN
            self._regions[name] = (off, tuple(shape), dtype, elem)
        off, shp, dt, _ = self._regions[name]
        if tuple(shape) != shp or dtype != dt:
            raise ValueError(f"region {name} exists with shape {shp} / {dt}")
        return _view(self.base + off, shp, dt, self.device)

    def peer_ptrs(self, name: str, offset_elems: int = 0) -> list[int]:
        """Addresses of element ``offset_elems`` of region ``name`` on every other rank."""
        off, _, _, elem = self._regions[name]
        return [self.bases[r] + off + offset_elems * elem for r in range(self.world) if r != self.rank]

    def barrier(self, stream=None):
        """Stage barrier: order this stream's earlier writes (peer stores included) before every rank's next stage."""
        st = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        _native.check(_native.load().fk_peer_barrier(
            ctypes.c_void_p(self._counter), ctypes.c_void_p(self.base + self._flags_off), self._peer_flags,
            self.rank, self.world, ctypes.c_void_p(st)))

    def signal(self, stream=None):
        """The signal half of :meth:`barrier`: advance the counter and store it into
        every peer's flag slot, without waiting. The next launch on the stream must
        do the wait (``*_wait`` entry points with :meth:`wait_args`)."""
        st = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        _native.check(_native.load().fk_peer_signal(
            ctypes.c_void_p(self._counter), self._peer_flags, self.rank, self.world, ctypes.c_void_p(st)))

    def wait_args(self) -> tuple:
        """(counter, flags, rank, world) for the ``*_wait`` entry points."""
        return (ctypes.c_void_p(self._counter), ctypes.c_void_p(self.base + self._flags_off), self.rank, self.world)

    def close(self):
        lib = _native.load()
        for r, b in enumerate(self.bases):
            if r != self.rank and b:
                lib.fk_ipc_close(ctypes.c_void_p(b))
        self.bases = []
        if self.base:
            torch.cuda.synchronize(self.device)
            lib.fk_peer_free(ctypes.c_void_p(self.base))
            self.base = 0
