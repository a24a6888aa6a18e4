"""Symmetric peer buffers: one device allocation per rank, mapped into every other rank.

The C++ side (csrc/symm.cpp) allocates with cudaMalloc and exports/imports CUDA IPC
handles; here the handles are exchanged through the process group and every rank ends up
with the base address of every rank's buffer. Kernels read/write a peer's buffer through
those addresses directly over NVLink 5 / NVSwitch (plain P2P loads, stores and atomics).
"""
import torch
import torch.distributed as dist

from .. import native


class SymmBuffer:
    """`nbytes` of device memory on every rank of `group`, with all ranks' addresses known."""

    def __init__(self, nbytes, device, group=None):
        C = native()
        self.device = torch.device(device)
        self.dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.nbytes = int(max(nbytes, 256))
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.ptr = C.symm_alloc(self.nbytes, self.dev)
        self.ptrs = [self.ptr]
        self._imported = []
        if self.world > 1:
            handle = C.symm_export(self.ptr, self.dev)
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
            self.ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self.ptr)
                else:
                    p = C.symm_import(h, self.dev)
                    self._imported.append(p)
                    self.ptrs.append(p)

    def view(self, offset, shape, dtype):
        """A tensor view of this rank's buffer at byte `offset`."""
        return native().symm_view(self.ptr + int(offset), list(shape), dtype, self.dev)

    def peer_addr(self, rank, offset):
        return self.ptrs[rank] + int(offset)

    def close(self):
        if self.ptr is None:
            return
        C = native()
        for p in self._imported:
            C.symm_close(p, self.dev)
        C.symm_free(self.ptr, self.dev)
        self.ptr = None
        self._imported = []

    def __del__(self):
        try:
            if self.ptr is not None and torch.cuda.is_initialized():
                self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
