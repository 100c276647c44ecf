"""Expert-parallel plumbing for the MoE blocks: the symmetric heap and the per-rank context.

The experts of every MoE layer are sharded over the ranks of the data-parallel group (the
reference runs all experts on one device, crates/sejong-gpu/src/hierarchy_ops.rs:280-454).  Rows
cross NVLink as plain peer loads and stores issued by the library's kernels (sj_ep_*) into a
symmetric heap: one device allocation of the same size on every rank, exported with CUDA IPC and
mapped into every peer, laid out by the same plan everywhere so that a buffer has one offset on
all ranks.  The plan is built on the host before the allocation; `EpContext.finalize` allocates,
exchanges the IPC handles over the process group and maps the peers.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call

HANDLE_BYTES = 64
ALIGN = 256


class _DeviceArray:
    """A borrowed device buffer presented through __cuda_array_interface__ (for torch.as_tensor)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
                                         "strides": None, "version": 3}


class EpContext:
    """Rank, world, heap plan and heap of one rank's expert-parallel MoE layers.

    `reserve(name, nbytes)` adds a buffer to the plan (every rank must reserve the same buffers in
    the same order); after `finalize()` `offset(name)` is its byte offset in every rank's heap,
    `ptr(name)` its address in this rank's heap and `peers` the address of the table of heap bases
    the sj_ep_* calls take.  `timeout_ms` bounds every cross-rank wait."""

    def __init__(self, rank, world, device, group=None, timeout_ms=10000):
        if world > 8:
            raise ValueError("expert parallelism spans at most 8 ranks (one NVLink domain)")
        self.rank, self.world, self.dev, self.group = int(rank), int(world), device, group
        self.timeout_ms = int(timeout_ms)
        self.plan = {}
        self.size = 0
        self.local = None
        self.opened = []
        self._table = None
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)  # barrier epoch counter (uint32 on the device)
        self.reserve("flags", 4 * self.world)

    def reserve(self, name, nbytes):
        if self.local is not None:
            raise RuntimeError("heap already allocated")
        if name in self.plan:
            raise KeyError(f"heap buffer {name} reserved twice")
        off = (self.size + ALIGN - 1) // ALIGN * ALIGN
        self.plan[name] = off
        self.size = off + int(nbytes)
        return off

    def finalize(self):
        """Allocate this rank's heap (zero-filled), exchange IPC handles and map every peer's."""
        _lib.load()
        torch.cuda.set_device(self.dev)
        p = ctypes.c_void_p()
        call("sj_ipc_alloc", self.size, ctypes.byref(p))
        self.local = p.value
        bases = [0] * self.world
        bases[self.rank] = self.local
        if self.world > 1:
            h = (ctypes.c_char * HANDLE_BYTES)()
            call("sj_ipc_handle", self.local, h)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h), group=self.group)
            for r in range(self.world):
                if r == self.rank:
                    continue
                q = ctypes.c_void_p()
                buf = ctypes.create_string_buffer(handles[r], HANDLE_BYTES)
                call("sj_ipc_open", buf, ctypes.byref(q))
                bases[r] = q.value
                self.opened.append(q.value)
        self.bases = bases
        self._table = (ctypes.c_void_p * self.world)(*bases)

    @property
    def peers(self):
        return ctypes.addressof(self._table)

    def offset(self, name):
        return self.plan[name]

    def ptr(self, name):
        return self.local + self.plan[name]

    def view(self, name, shape, dtype):
        """A torch tensor over a heap buffer of this rank (no copy)."""
        typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.bfloat16: "<i2", torch.int16: "<i2"}[dtype]
        t = torch.as_tensor(_DeviceArray(self.ptr(name), shape, typestr), device=self.dev)
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    def close(self):
        """Unmap the peers' heaps and free this rank's (after every rank has stopped using it)."""
        for q in self.opened:
            call("sj_ipc_close", q)
        self.opened = []
        if self.local is not None:
            call("sj_ipc_free", self.local)
            self.local = None
