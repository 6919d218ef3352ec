"""CPU tests of the arena sub-allocator, mirroring the checks of LMCache-Ascend
tests/v1/test_memory_management.py:22-67 (check_allocator)."""

import torch

from lmcache_b200.v1.memory_management import ALIGN, TensorMemoryAllocator


def check_allocator(allocator, max_size):
    data1 = allocator.allocate([512, 512], torch.float)
    assert data1 is not None and data1.tensor.dtype == torch.float
    assert data1.tensor.shape == (512, 512)
    data2 = allocator.allocate([1024, 1024], dtype=torch.bfloat16)
    assert data2 is not None and data2.tensor.shape == (1024, 1024)
    data3 = allocator.allocate([2048, 2048], dtype=torch.int8)
    assert data3 is not None and data3.tensor.dtype == torch.int8
    allocator.free(data2)
    assert data2.tensor is None
    assert allocator.memcheck()
    allocator.free(data1)
    assert data1.tensor is None
    assert allocator.memcheck()
    allocator.free(data2)  # must not crash
    data4 = allocator.allocate([3, 5, 7], dtype=torch.half)
    assert data4 is not None and data4.tensor.shape == (3, 5, 7)
    assert allocator.allocate([max_size], dtype=torch.float) is None
    assert allocator.memcheck()
    for d in (data1, data2, data3, data4):
        allocator.free(d)
    assert allocator.memcheck()
    allocator.close()


def test_tensor_allocator():
    total = 128 << 20
    check_allocator(TensorMemoryAllocator(torch.zeros(total, dtype=torch.uint8)), total)


def test_alignment_and_coalescing():
    buf = torch.zeros(1 << 20, dtype=torch.uint8)
    a = TensorMemoryAllocator(buf)
    objs = [a.allocate([7], torch.bfloat16) for _ in range(10)]
    assert all((o.tensor.data_ptr() - buf.data_ptr()) % ALIGN == 0 for o in objs)
    assert all(o.nbytes == ALIGN for o in objs)
    for o in objs[::2]:
        a.free(o)
    assert a.memcheck() and len(a._free) == 6
    for o in objs[1::2]:
        a.free(o)
    assert a.memcheck() and a._free == [(0, 1 << 20)]


def test_views_share_the_arena():
    buf = torch.zeros(4096, dtype=torch.uint8)
    a = TensorMemoryAllocator(buf)
    o = a.allocate([2, 4], torch.int32)
    o.tensor.fill_(-1)
    assert (buf[o.offset : o.offset + 32] == 255).all()
