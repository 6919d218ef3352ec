"""Pinned host arenas for LMCache objects on CUDA.

Counterpart of LMCache-Ascend's AscendPinMemoryAllocator /
AscendMixedMemoryAllocator (lmcache_ascend/v1/memory_management.py:33-106):
one pinned uint8 buffer is allocated up front and registered with
``c_ops.host_register`` so the transfer kernels can address any object carved
out of it (zero-copy over PCIe). Objects are dense views into the arena.

The sub-allocator is first-fit over an address-ordered free list with
coalescing on free, with 256-byte aligned blocks (so every object start is
16-byte aligned for the vectorised kernels).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from .. import c_ops

ALIGN = 256


@dataclass
class MemoryObj:
    """A dense tensor view into an arena; ``tensor`` is None once freed."""

    tensor: Optional[torch.Tensor]
    offset: int
    nbytes: int


class PinMemoryAllocator:
    """First-fit allocator over one pinned, host-registered buffer."""

    def __init__(self, size: int):
        self.size = int(size)
        self.buffer = torch.empty(self.size, dtype=torch.uint8, device="cpu", pin_memory=True)
        c_ops.host_register(self.buffer)
        self._free: List[Tuple[int, int]] = [(0, self.size)]  # (offset, length), sorted
        self._lock = threading.Lock()

    def allocate(self, shape, dtype: torch.dtype) -> Optional[MemoryObj]:
        shape = torch.Size(shape)
        elem = torch.empty((), dtype=dtype).element_size()
        nbytes = shape.numel() * elem
        need = max(ALIGN, (nbytes + ALIGN - 1) // ALIGN * ALIGN)
        with self._lock:
            for i, (off, length) in enumerate(self._free):
                if length >= need:
                    if length == need:
                        self._free.pop(i)
                    else:
                        self._free[i] = (off + need, length - need)
                    view = self.buffer[off : off + nbytes].view(dtype).view(shape)
                    return MemoryObj(view, off, need)
        return None

    def free(self, obj: MemoryObj) -> None:
        if obj is None or obj.tensor is None:
            return
        with self._lock:
            self._free.append((obj.offset, obj.nbytes))
            self._free.sort()
            merged: List[Tuple[int, int]] = []
            for off, length in self._free:
                if merged and merged[-1][0] + merged[-1][1] == off:
                    merged[-1] = (merged[-1][0], merged[-1][1] + length)
                else:
                    merged.append((off, length))
            self._free = merged
        obj.tensor = None

    def memcheck(self) -> bool:
        """Free blocks are in range, ordered, non-overlapping and coalesced."""
        with self._lock:
            prev_end = -1
            for off, length in self._free:
                if off < 0 or length <= 0 or off + length > self.size or off <= prev_end:
                    return False
                if off == prev_end:
                    return False
                prev_end = off + length
        return True

    def close(self) -> None:
        try:
            c_ops.host_unregister(self.buffer)
        except Exception:
            pass
