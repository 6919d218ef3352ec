"""Tests of the LMCache objects and allocators (lmcache_b200.v1.memory_management),
with the checks of LMCache-Ascend tests/v1/test_memory_management.py: the
general allocator sequence (:22-67), the paged one (:70-110), every allocator
class with and without paging (:113-158), in-place writes (:161-183), no
zero-size free blocks (:186-208), batched allocation (:211-238) and byte
buffers in the mixed allocator (:241-276). Host arenas run on the CPU; the
pinned, mixed and HBM arenas need CUDA and are marked gpu.
"""

import pytest
import torch

from lmcache_b200.v1.memory_management import (
    ALIGN,
    BytesBufferMemoryObj,
    GPUMemoryAllocator,
    HostMemoryAllocator,
    MemoryFormat,
    MixedMemoryAllocator,
    PagedTensorMemoryAllocator,
    PinMemoryAllocator,
    TensorMemoryAllocator,
)

PAGE_SHAPE = torch.Size([2, 32, 16, 1024])  # 2 MiB of bf16: 64 pages in 128 MiB


def gpu_param(cls):
    return pytest.param(cls, marks=pytest.mark.gpu, id=cls.__name__)


ALLOCATORS = [pytest.param(HostMemoryAllocator, id="HostMemoryAllocator"),
              gpu_param(PinMemoryAllocator), gpu_param(GPUMemoryAllocator),
              gpu_param(MixedMemoryAllocator)]


def free_list(allocator):
    inner = allocator.pin_allocator if isinstance(allocator, MixedMemoryAllocator) \
        else allocator.allocator
    return inner.explicit_list


def run_general_sequence(allocator, max_size):
    d1 = allocator.allocate([512, 512], torch.float)
    assert d1 is not None and d1.tensor.dtype == torch.float and d1.tensor.shape == (512, 512)
    d2 = allocator.allocate([1024, 1024], dtype=torch.bfloat16)
    assert d2 is not None and d2.tensor.dtype == torch.bfloat16
    assert d2.tensor.shape == (1024, 1024)
    d3 = allocator.allocate([2048, 2048], dtype=torch.int8)
    assert d3 is not None and d3.tensor.dtype == torch.int8 and d3.tensor.shape == (2048, 2048)
    allocator.free(d2)
    assert d2.tensor is None and allocator.memcheck()
    allocator.free(d1)
    assert d1.tensor is None and allocator.memcheck()
    allocator.free(d2)  # a second free is ignored
    d4 = allocator.allocate([3, 5, 7], dtype=torch.half)
    assert d4 is not None and d4.tensor.dtype == torch.half and d4.tensor.shape == (3, 5, 7)
    assert allocator.allocate([max_size], dtype=torch.float) is None  # does not fit
    assert allocator.memcheck()
    for d in (d1, d2, d3, d4):
        allocator.free(d)
    assert allocator.memcheck()
    allocator.close()


def run_paged_sequence(allocator, shape, dtype, fmt, max_pages):
    d1 = allocator.allocate(shape, dtype, fmt)
    assert d1 is not None and d1.tensor.dtype == dtype and d1.tensor.shape == shape
    d2 = allocator.batched_allocate(shape, dtype, 2, fmt)
    assert len(d2) == 2
    for d in d2:
        assert d is not None and d.tensor.dtype == dtype and d.tensor.shape == shape
    smaller = torch.Size([2, 32, 8, 1024])
    d3 = allocator.allocate(smaller, dtype, fmt)
    assert d3 is not None and d3.tensor.shape == smaller
    allocator.free(d3)
    assert allocator.memcheck()
    allocator.batched_free(d2)
    assert allocator.memcheck()
    allocator.free(d1)
    assert allocator.memcheck()
    assert allocator.batched_allocate(shape, dtype, max_pages + 1, fmt) is None
    assert allocator.memcheck()
    allocator.close()


@pytest.mark.parametrize("use_paging", [True, False])
def test_tensor_allocator(use_paging):
    total = 128 << 20
    buf = torch.zeros(total, dtype=torch.uint8)
    if use_paging:
        a = PagedTensorMemoryAllocator(buf, PAGE_SHAPE, torch.bfloat16, MemoryFormat.KV_2LTD)
        run_paged_sequence(a, PAGE_SHAPE, torch.bfloat16, MemoryFormat.KV_2LTD, 64)
    else:
        run_general_sequence(TensorMemoryAllocator(buf), total)


@pytest.mark.parametrize("alloc_cls", ALLOCATORS)
@pytest.mark.parametrize("use_paging", [False, True])
def test_device_allocators(alloc_cls, use_paging):
    total = 128 << 20
    a = alloc_cls(total, use_paging=use_paging, shape=PAGE_SHAPE, dtype=torch.bfloat16,
                  fmt=MemoryFormat.KV_2LTD)
    if use_paging:
        run_paged_sequence(a, PAGE_SHAPE, torch.bfloat16, MemoryFormat.KV_2LTD, 64)
    else:
        run_general_sequence(a, total)


@pytest.mark.parametrize("alloc_cls", ALLOCATORS)
def test_inplace_modification(alloc_cls):
    a = alloc_cls(1024)
    d = a.allocate([10], torch.float)
    assert d is not None and d.tensor.shape == (10,)
    d.tensor.fill_(1.0)
    assert torch.all(d.tensor == 1.0)
    d.tensor[1] = 2.0
    assert d.tensor[1] == 2.0
    a.close()


@pytest.mark.parametrize("alloc_cls", ALLOCATORS)
def test_boundary_alloc(alloc_cls):
    a = alloc_cls(1 << 25)
    d1 = a.allocate([512, 10], torch.float)
    a.allocate([512, 10], torch.float)
    a.free(d1)
    a.allocate([512, 10], torch.float)  # takes d1's block exactly: no empty block remains
    assert len(free_list(a)) == 1
    a.close()


@pytest.mark.parametrize("alloc_cls", ALLOCATORS)
def test_batched_alloc(alloc_cls):
    n = 32
    a = alloc_cls(n * 100 * 2 * 1024 * 2)  # exactly n objects
    objs = a.batched_allocate([100, 2, 1024], torch.bfloat16, n, MemoryFormat.KV_T2D)
    assert len(objs) == n
    for o in objs:
        assert o.tensor.dtype == torch.bfloat16 and o.tensor.shape == (100, 2, 1024)
        assert o.metadata.fmt == MemoryFormat.KV_T2D
    a.batched_free(objs)
    assert len(free_list(a)) == 1
    a.close()


@pytest.mark.gpu
def test_mixed_alloc():
    a = MixedMemoryAllocator(1 << 25)
    d1 = a.allocate([512, 0], None, MemoryFormat.BINARY_BUFFER)
    a.allocate([512, 10], torch.float)
    a.free(d1)
    assert len(a.pin_allocator.explicit_list) == 1
    assert isinstance(d1, BytesBufferMemoryObj)
    assert len(d1.byte_array) == 512
    a.close()


# --- beyond the reference's checks -------------------------------------------


def test_metadata_and_ref_count_return_the_block():
    a = TensorMemoryAllocator(torch.zeros(1 << 20, dtype=torch.uint8))
    o = a.allocate([4, 2, 8], torch.bfloat16, MemoryFormat.KV_T2D)
    assert o.metadata.fmt == MemoryFormat.KV_T2D and o.metadata.shape == (4, 2, 8)
    assert o.metadata.dtype == torch.bfloat16 and o.metadata.phy_size == ALIGN
    assert o.get_ref_count() == 1
    o.ref_count_up()
    o.ref_count_down()
    assert o.tensor is not None and len(a.explicit_list) == 1
    o.ref_count_down()  # the last reference frees the block
    assert o.tensor is None and a.explicit_list[0].start == 0
    assert a.memcheck()


def test_alignment_and_coalescing():
    buf = torch.zeros(1 << 20, dtype=torch.uint8)
    a = TensorMemoryAllocator(buf)
    objs = [a.allocate([7], torch.bfloat16) for _ in range(10)]
    assert all((o.tensor.data_ptr() - buf.data_ptr()) % ALIGN == 0 for o in objs)
    assert all(o.metadata.phy_size == ALIGN for o in objs)
    for o in objs[::2]:
        a.free(o)
    assert a.memcheck() and len(a.explicit_list) == 6
    for o in objs[1::2]:
        a.free(o)
    assert a.memcheck() and a._free == [(0, 1 << 20)]


def test_views_share_the_arena():
    buf = torch.zeros(4096, dtype=torch.uint8)
    a = TensorMemoryAllocator(buf)
    o = a.allocate([2, 4], torch.int32)
    o.tensor.fill_(-1)
    off = o.metadata.address
    assert (buf[off: off + 32] == 255).all()


def test_paged_pages_are_reused_and_bounded():
    page = torch.Size([2, 4, 8, 64])
    a = PagedTensorMemoryAllocator(torch.zeros(8 * page.numel() * 2, dtype=torch.uint8), page,
                                   torch.bfloat16, MemoryFormat.KV_2LTD)
    assert a.num_pages == 8
    objs = a.batched_allocate(page, torch.bfloat16, 8)
    assert a.allocate(page, torch.bfloat16) is None
    starts = sorted(o.metadata.address for o in objs)
    assert starts == [i * a.page_bytes for i in range(8)]
    assert a.allocate(torch.Size([2, 4, 8, 65]), torch.bfloat16) is None  # larger than a page
    freed_at = objs[3].metadata.address
    a.free(objs[3])
    assert objs[3].tensor is None
    again = a.allocate([1, 4, 8, 64], torch.bfloat16)  # a smaller object takes the freed page
    assert again.metadata.address == freed_at and again.tensor.shape == (1, 4, 8, 64)
    assert a.memcheck()
