"""Exchange buffers of the multi-GPU decode: one per rank, mapped into every rank's process with CUDA IPC.

``PeerBuffers(group, hidden)`` is collective over ``group`` (one process per GPU): each rank allocates its buffer
(``flint_peer_alloc``), the 64-byte IPC handles are all-gathered, and every rank maps the others' buffers
(``flint_peer_open``).  ``ptrs[r]`` is rank r's buffer as mapped in this process; the expert-parallel MoE block and
the vocabulary-shard argmax exchange take that list.  ``close()`` (collective) unmaps and frees; call it after the
last exchange launch has completed on every rank and before the process group is destroyed.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class PeerBuffers:
    def __init__(self, group, hidden: int):
        import torch.distributed as dist
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 2 <= self.world <= 8:
            raise _lib.FlintError(f"peer exchange needs 2..8 ranks, got {self.world}")
        L = _lib.lib()
        nbytes = L.flint_peer_buffer_bytes(int(hidden))
        if nbytes <= 0:
            raise _lib.FlintError(f"peer exchange: unsupported hidden size {hidden}")
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _lib.check(L.flint_peer_alloc(nbytes, ctypes.byref(own), handle), "flint_peer_alloc")
        self.own, self.nbytes = own.value, nbytes
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened: list[int] = []
        self.ptrs: list[int] = []
        try:
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self.own)
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                _lib.check(L.flint_peer_open(hb, ctypes.byref(p)), "flint_peer_open")
                self._opened.append(p.value)
                self.ptrs.append(p.value)
        except Exception:
            self._release()
            raise
        dist.barrier(group)

    def status(self) -> int:
        """Sticky status word of this rank's buffer: bit 4 = a peer wait timed out (outputs since then are invalid)."""
        st = ctypes.c_uint32()
        _lib.check(_lib.lib().flint_peer_status(self.own, ctypes.byref(st)), "flint_peer_status")
        return int(st.value)

    def _release(self):
        L = _lib.lib()
        for p in self._opened:
            L.flint_peer_close(p)
        self._opened = []
        if self.own:
            L.flint_peer_free(self.own)
            self.own = None
        self.ptrs = []

    def close(self):
        import torch.distributed as dist
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)          # no rank still stores into or waits on these buffers
        self._release()
