"""Pinned host arenas for LMCache objects on CUDA.

Counterpart of LMCache-Ascend's AscendPinMemoryAllocator /
AscendMixedMemoryAllocator (lmcache_ascend/v1/memory_management.py:33-106):
one pinned uint8 buffer is allocated up front and registered with
``c_ops.host_register`` so the transfer kernels can address any object carved
out of it (zero-copy over PCIe). Objects are dense views into the arena.

The sub-allocator is first-fit over an address-ordered free list with
coalescing on free, with 256-byte aligned blocks (so every object start is
16-byte aligned for the vectorised and bulk-copy kernels).
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


class TensorMemoryAllocator:
    """First-fit allocator over one uint8 buffer (any device).

    Same contract as upstream LMCache's TensorMemoryAllocator as the
    reference's tests use it (tests/v1/test_memory_management.py:22-67):
    ``allocate`` returns None when nothing fits, ``free`` tolerates a second
    free of the same object, ``memcheck`` validates the free list.
    """

    def __init__(self, buffer: torch.Tensor):
        assert buffer.dtype == torch.uint8 and buffer.dim() == 1
        self.buffer = buffer
        self.size = buffer.numel()
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
        """Free blocks are in range, sorted, disjoint and coalesced."""
        with self._lock:
            prev_end = -1
            for off, length in self._free:
                if off < 0 or length <= 0 or off + length > self.size or off <= prev_end:
                    return False
                prev_end = off + length
        return True

    def close(self) -> None:
        pass


class PinMemoryAllocator(TensorMemoryAllocator):
    """A TensorMemoryAllocator over a pinned host buffer registered with
    ``c_ops.host_register`` (lmcache_ascend/v1/memory_management.py:33-68)."""

    def __init__(self, size: int):
        buffer = torch.empty(int(size), dtype=torch.uint8, device="cpu", pin_memory=True)
        c_ops.host_register(buffer)
        super().__init__(buffer)

    def close(self) -> None:
        try:
            c_ops.host_unregister(self.buffer)
        except RuntimeError:
            pass
