"""LMCache objects and the allocators that own them, on CUDA.

Counterpart of LMCache-Ascend's AscendPinMemoryAllocator /
AscendMixedMemoryAllocator (lmcache_ascend/v1/memory_management.py:33-106),
which wrap upstream LMCache's allocators around a pinned buffer registered
with ``c_ops.host_register``. Upstream LMCache is not a dependency here, so
this module provides the part of its memory-management API the transfer path
and the reference's allocator tests (tests/v1/test_memory_management.py) use:

* ``MemoryFormat`` -- the layout tag a connector checks before a transfer
  (KV_2LTD [2, L, T, H], KV_T2D [T, 2, H], KV_MLA_FMT [1, L, T, H], and the
  byte formats BINARY / BINARY_BUFFER).
* ``TensorMemoryObj`` -- a typed view into an arena, with metadata (shape,
  dtype, address, physical size, format) and a reference count; the object
  returns its block to its allocator when the count drops to zero.
  ``BytesBufferMemoryObj`` holds a plain byte buffer.
* ``TensorMemoryAllocator`` -- first fit over an address-ordered explicit free
  list, coalescing on free; blocks are 256-byte aligned so every object start
  suits the vectorised and bulk-copy kernels.
* ``PagedTensorMemoryAllocator`` -- fixed pages of one object shape (the
  ``use_paging`` branch, memory_management.py:49-64, :84-95).
* ``HostMemoryAllocator`` (pageable host), ``PinMemoryAllocator`` (pinned and
  registered for zero-copy kernel access), ``GPUMemoryAllocator`` (HBM) and
  ``MixedMemoryAllocator`` (pinned arena plus byte buffers), all with the
  ``use_paging`` option.
"""

from __future__ import annotations

import enum
import threading
from dataclasses import dataclass
from typing import List, Optional, Tuple, Union

import torch

from .. import c_ops

ALIGN = 256


class MemoryFormat(enum.IntEnum):
    UNDEFINED = 0
    KV_2LTD = 1  # [2, num_layers, num_tokens, hidden]
    KV_T2D = 2  # [num_tokens, 2, hidden]
    BINARY = 3  # raw bytes in a tensor arena
    BINARY_BUFFER = 4  # raw bytes in a Python buffer
    KV_MLA_FMT = 5  # [1, num_layers, num_tokens, hidden]

    def token_dim(self) -> int:
        return {MemoryFormat.KV_2LTD: 2, MemoryFormat.KV_T2D: 0,
                MemoryFormat.KV_MLA_FMT: 2}.get(self, 0)


@dataclass
class MemoryObjMetadata:
    shape: torch.Size
    dtype: Optional[torch.dtype]
    address: int  # byte offset of the block in its arena
    phy_size: int  # bytes of the block (aligned)
    ref_count: int
    fmt: MemoryFormat = MemoryFormat.UNDEFINED


class MemoryObj:
    """Base of the LMCache objects: metadata plus a reference count."""

    def __init__(self, metadata: MemoryObjMetadata, parent=None):
        self.meta = metadata
        self.parent_allocator = parent
        self._lock = threading.Lock()

    @property
    def metadata(self) -> MemoryObjMetadata:
        return self.meta

    def get_shape(self) -> torch.Size:
        return self.meta.shape

    def get_dtype(self) -> Optional[torch.dtype]:
        return self.meta.dtype

    def get_memory_format(self) -> MemoryFormat:
        return self.meta.fmt

    def get_physical_size(self) -> int:
        return self.meta.phy_size

    def get_ref_count(self) -> int:
        with self._lock:
            return self.meta.ref_count

    def ref_count_up(self) -> None:
        with self._lock:
            self.meta.ref_count += 1

    def ref_count_down(self) -> None:
        """Drops one reference; the last one returns the block to the allocator."""
        with self._lock:
            self.meta.ref_count -= 1
            last = self.meta.ref_count == 0
        if last and self.parent_allocator is not None:
            self.parent_allocator.free(self)


class TensorMemoryObj(MemoryObj):
    """A typed view of ``metadata.shape`` / ``metadata.dtype`` into an arena."""

    def __init__(self, raw_data: torch.Tensor, metadata: MemoryObjMetadata, parent=None):
        super().__init__(metadata, parent)
        self.raw_data = raw_data  # uint8 slice of the arena, or None once freed
        self._tensor = None
        if raw_data is not None:
            nbytes = metadata.shape.numel() * torch.empty((), dtype=metadata.dtype).element_size()
            self._tensor = raw_data[:nbytes].view(metadata.dtype).view(metadata.shape)

    @classmethod
    def wrap(cls, tensor: torch.Tensor,
             fmt: MemoryFormat = MemoryFormat.KV_2LTD) -> "TensorMemoryObj":
        """An object over a tensor that no allocator owns (for example a
        buffer a caller allocated itself); freeing it only invalidates it."""
        assert tensor.is_contiguous()
        raw = tensor.view(-1).view(torch.uint8)
        meta = MemoryObjMetadata(tensor.shape, tensor.dtype, 0, raw.numel(), 1, fmt)
        return cls(raw, meta, None)

    @property
    def tensor(self) -> Optional[torch.Tensor]:
        return self._tensor

    def is_valid(self) -> bool:
        return self._tensor is not None

    def invalidate(self) -> None:
        self.raw_data = None
        self._tensor = None

    def get_size(self) -> int:
        return 0 if self._tensor is None else self._tensor.numel() * self._tensor.element_size()

    @property
    def byte_array(self) -> bytes:
        t = self._tensor
        if t is None:
            return b""
        return t.contiguous().view(torch.uint8).cpu().numpy().tobytes()


class BytesBufferMemoryObj(MemoryObj):
    """An object holding plain bytes (MemoryFormat.BINARY_BUFFER)."""

    def __init__(self, byte_array: Union[bytes, bytearray], parent=None):
        meta = MemoryObjMetadata(torch.Size([len(byte_array)]), None, 0, len(byte_array), 1,
                                 MemoryFormat.BINARY_BUFFER)
        super().__init__(meta, parent)
        self.byte_array = byte_array

    @property
    def tensor(self) -> None:
        return None

    def is_valid(self) -> bool:
        return self.byte_array is not None

    def invalidate(self) -> None:
        self.byte_array = None

    def get_size(self) -> int:
        return 0 if self.byte_array is None else len(self.byte_array)


@dataclass
class FreeBlock:
    start: int
    size: int


def _elem_size(dtype: torch.dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


class TensorMemoryAllocator:
    """First fit over one uint8 buffer (any device).

    ``allocate`` returns None when nothing fits; ``free`` of an already freed
    object is ignored; ``explicit_list`` is the address-ordered list of free
    blocks (never one of size 0); ``memcheck`` validates it.
    """

    def __init__(self, tensor: torch.Tensor, align: int = ALIGN):
        assert tensor.dtype == torch.uint8 and tensor.dim() == 1
        self.buffer = tensor
        self.size = tensor.numel()
        self.align = align
        self.explicit_list: List[FreeBlock] = [FreeBlock(0, self.size)]
        self._lock = threading.Lock()

    def _block_size(self, nbytes: int) -> int:
        return max(self.align, -(-nbytes // self.align) * self.align)

    def _take(self, need: int) -> Optional[int]:
        for i, blk in enumerate(self.explicit_list):
            if blk.size >= need:
                start = blk.start
                if blk.size == need:
                    self.explicit_list.pop(i)
                else:
                    blk.start += need
                    blk.size -= need
                return start
        return None

    def allocate(self, shape, dtype: Optional[torch.dtype],
                 fmt: MemoryFormat = MemoryFormat.KV_2LTD) -> Optional[TensorMemoryObj]:
        shape = torch.Size(shape)
        if dtype is None:
            dtype = torch.uint8
        need = self._block_size(shape.numel() * _elem_size(dtype))
        with self._lock:
            start = self._take(need)
        if start is None:
            return None
        meta = MemoryObjMetadata(shape, dtype, start, need, 1, fmt)
        return TensorMemoryObj(self.buffer[start:start + need], meta, self)

    def batched_allocate(self, shape, dtype: Optional[torch.dtype], batch_size: int,
                         fmt: MemoryFormat = MemoryFormat.KV_2LTD
                         ) -> Optional[List[TensorMemoryObj]]:
        """``batch_size`` objects of one shape, or None (and nothing held)."""
        objs = []
        for _ in range(batch_size):
            o = self.allocate(shape, dtype, fmt)
            if o is None:
                self.batched_free(objs)
                return None
            objs.append(o)
        return objs

    def free(self, obj: Optional[MemoryObj]) -> None:
        if obj is None or not isinstance(obj, TensorMemoryObj) or not obj.is_valid():
            return
        start, size = obj.meta.address, obj.meta.phy_size
        with self._lock:
            blocks = self.explicit_list
            i = 0
            while i < len(blocks) and blocks[i].start < start:
                i += 1
            blocks.insert(i, FreeBlock(start, size))
            if i + 1 < len(blocks) and blocks[i].start + blocks[i].size == blocks[i + 1].start:
                blocks[i].size += blocks[i + 1].size
                blocks.pop(i + 1)
            if i > 0 and blocks[i - 1].start + blocks[i - 1].size == blocks[i].start:
                blocks[i - 1].size += blocks[i].size
                blocks.pop(i)
        obj.invalidate()

    def batched_free(self, objs) -> None:
        for o in objs:
            self.free(o)

    def memcheck(self) -> bool:
        """Free blocks are non-empty, in range, address-ordered, disjoint and
        coalesced."""
        with self._lock:
            prev_end = -1
            for blk in self.explicit_list:
                if blk.size <= 0 or blk.start < 0 or blk.start + blk.size > self.size:
                    return False
                if blk.start <= prev_end:  # overlapping, or adjacent but not merged
                    return False
                prev_end = blk.start + blk.size
        return True

    @property
    def _free(self) -> List[Tuple[int, int]]:
        return [(b.start, b.size) for b in self.explicit_list]

    def close(self) -> None:
        pass


class PagedTensorMemoryAllocator:
    """Fixed pages, each able to hold one object of ``shape`` / ``dtype``.

    Objects of that shape or smaller take one page; ``batched_allocate`` of
    more pages than are free returns None and holds nothing.
    """

    def __init__(self, tensor: torch.Tensor, shape, dtype: torch.dtype,
                 fmt: MemoryFormat = MemoryFormat.KV_2LTD):
        assert tensor.dtype == torch.uint8 and tensor.dim() == 1
        self.buffer = tensor
        self.shape = torch.Size(shape)
        self.dtype = dtype
        self.fmt = fmt
        self.page_bytes = -(-self.shape.numel() * _elem_size(dtype) // ALIGN) * ALIGN
        self.num_pages = tensor.numel() // self.page_bytes
        self.free_pages: List[int] = list(range(self.num_pages))
        self._lock = threading.Lock()

    def _make(self, page: int, shape, dtype, fmt) -> TensorMemoryObj:
        start = page * self.page_bytes
        meta = MemoryObjMetadata(torch.Size(shape), dtype, start, self.page_bytes, 1, fmt)
        return TensorMemoryObj(self.buffer[start:start + self.page_bytes], meta, self)

    def _fits(self, shape, dtype) -> bool:
        return torch.Size(shape).numel() * _elem_size(dtype) <= self.page_bytes

    def allocate(self, shape, dtype: Optional[torch.dtype] = None,
                 fmt: Optional[MemoryFormat] = None) -> Optional[TensorMemoryObj]:
        dtype = dtype or self.dtype
        if not self._fits(shape, dtype):
            return None
        with self._lock:
            if not self.free_pages:
                return None
            page = self.free_pages.pop(0)
        return self._make(page, shape, dtype, fmt or self.fmt)

    def batched_allocate(self, shape, dtype: Optional[torch.dtype], batch_size: int,
                         fmt: Optional[MemoryFormat] = None
                         ) -> Optional[List[TensorMemoryObj]]:
        dtype = dtype or self.dtype
        if not self._fits(shape, dtype):
            return None
        with self._lock:
            if len(self.free_pages) < batch_size:
                return None
            pages, self.free_pages = self.free_pages[:batch_size], self.free_pages[batch_size:]
        return [self._make(p, shape, dtype, fmt or self.fmt) for p in pages]

    def free(self, obj: Optional[MemoryObj]) -> None:
        if obj is None or not isinstance(obj, TensorMemoryObj) or not obj.is_valid():
            return
        page = obj.meta.address // self.page_bytes
        with self._lock:
            self.free_pages.append(page)
        obj.invalidate()

    def batched_free(self, objs) -> None:
        for o in objs:
            self.free(o)

    def memcheck(self) -> bool:
        with self._lock:
            pages = self.free_pages
            return len(set(pages)) == len(pages) and all(0 <= p < self.num_pages for p in pages)

    def close(self) -> None:
        pass


def _sub_allocator(buffer: torch.Tensor, use_paging: bool, kwargs):
    if use_paging:
        for key in ("shape", "dtype", "fmt"):
            assert key in kwargs, f"{key} must be specified for the paged memory allocator"
        return PagedTensorMemoryAllocator(buffer, kwargs["shape"], kwargs["dtype"], kwargs["fmt"])
    return TensorMemoryAllocator(buffer)


class _ArenaAllocator:
    """An arena buffer with a sub-allocator (``self.allocator``)."""

    allocator: Union[TensorMemoryAllocator, PagedTensorMemoryAllocator]

    def allocate(self, shape, dtype: Optional[torch.dtype] = None,
                 fmt: MemoryFormat = MemoryFormat.KV_2LTD):
        with self.host_mem_lock:
            return self.allocator.allocate(shape, dtype, fmt)

    def batched_allocate(self, shape, dtype: Optional[torch.dtype], batch_size: int,
                         fmt: MemoryFormat = MemoryFormat.KV_2LTD):
        with self.host_mem_lock:
            return self.allocator.batched_allocate(shape, dtype, batch_size, fmt)

    def free(self, obj) -> None:
        with self.host_mem_lock:
            self.allocator.free(obj)

    def batched_free(self, objs) -> None:
        with self.host_mem_lock:
            self.allocator.batched_free(objs)

    def memcheck(self) -> bool:
        return self.allocator.memcheck()

    def close(self) -> None:
        pass


class HostMemoryAllocator(_ArenaAllocator):
    """Pageable host arena (not reachable by the kernels)."""

    def __init__(self, size: int, use_paging: bool = False, **kwargs):
        self.buffer = torch.empty(int(size), dtype=torch.uint8, device="cpu")
        self.allocator = _sub_allocator(self.buffer, use_paging, kwargs)
        self.host_mem_lock = threading.Lock()


class PinMemoryAllocator(_ArenaAllocator):
    """Pinned host arena registered with ``c_ops.host_register``, so the
    kernels reach every object in it over PCIe
    (lmcache_ascend/v1/memory_management.py:33-68)."""

    def __init__(self, size: int, use_paging: bool = False, **kwargs):
        self.buffer = torch.empty(int(size), dtype=torch.uint8, device="cpu", pin_memory=True)
        c_ops.host_register(self.buffer)
        self.allocator = _sub_allocator(self.buffer, use_paging, kwargs)
        self.host_mem_lock = threading.Lock()
        self._registered = True

    def close(self) -> None:
        if self._registered:
            self._registered = False
            try:
                c_ops.host_unregister(self.buffer)
            except RuntimeError:
                pass


class GPUMemoryAllocator(_ArenaAllocator):
    """HBM arena on ``device`` (default: the current CUDA device)."""

    def __init__(self, size: int, device=None, use_paging: bool = False, **kwargs):
        device = device if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.buffer = torch.empty(int(size), dtype=torch.uint8, device=device)
        self.allocator = _sub_allocator(self.buffer, use_paging, kwargs)
        self.host_mem_lock = threading.Lock()


class BufferAllocator:
    """Plain byte buffers (MemoryFormat.BINARY_BUFFER) on the host."""

    def __init__(self, device: str = "cpu"):
        self.device = device

    def allocate(self, shape, dtype=None, fmt: MemoryFormat = MemoryFormat.BINARY_BUFFER
                 ) -> BytesBufferMemoryObj:
        n = int(torch.Size(shape)[0]) if len(shape) else 0
        return BytesBufferMemoryObj(bytearray(n), self)

    def free(self, obj) -> None:
        """Byte buffers are ordinary Python objects: a freed one stays readable
        until its last reference goes (upstream's BufferAllocator behaves the
        same; the reference's mixed-allocator test reads one after free)."""

    def memcheck(self) -> bool:
        return True


class MixedMemoryAllocator:
    """A registered pinned arena for tensor objects (``pin_allocator``) plus
    byte buffers for MemoryFormat.BINARY_BUFFER (``buffer_allocator``)
    (lmcache_ascend/v1/memory_management.py:71-106)."""

    def __init__(self, size: int, use_paging: bool = False, **kwargs):
        self.buffer = torch.empty(int(size), dtype=torch.uint8, device="cpu", pin_memory=True)
        c_ops.host_register(self.buffer)
        self._registered = True
        self.pin_allocator = _sub_allocator(self.buffer, use_paging, kwargs)
        self.buffer_allocator = BufferAllocator("cpu")
        self.host_mem_lock = threading.Lock()

    def allocate(self, shape, dtype: Optional[torch.dtype] = None,
                 fmt: MemoryFormat = MemoryFormat.KV_2LTD):
        if fmt == MemoryFormat.BINARY_BUFFER:
            return self.buffer_allocator.allocate(shape, dtype, fmt)
        with self.host_mem_lock:
            return self.pin_allocator.allocate(shape, dtype, fmt)

    def batched_allocate(self, shape, dtype: Optional[torch.dtype], batch_size: int,
                         fmt: MemoryFormat = MemoryFormat.KV_2LTD):
        if fmt == MemoryFormat.BINARY_BUFFER:
            return [self.buffer_allocator.allocate(shape, dtype, fmt) for _ in range(batch_size)]
        with self.host_mem_lock:
            return self.pin_allocator.batched_allocate(shape, dtype, batch_size, fmt)

    def free(self, obj) -> None:
        if isinstance(obj, BytesBufferMemoryObj):
            self.buffer_allocator.free(obj)
            return
        with self.host_mem_lock:
            self.pin_allocator.free(obj)

    def batched_free(self, objs) -> None:
        for o in objs:
            self.free(o)

    def memcheck(self) -> bool:
        return self.pin_allocator.memcheck()

    def close(self) -> None:
        if self._registered:
            self._registered = False
            try:
                c_ops.host_unregister(self.buffer)
            except RuntimeError:
                pass
