"""GPU tests of the pinned-host side: the host registry (host_register /
get_kernel_ptr semantics of csrc/managed_mem.cpp and csrc/mem_kernels.cpp:11-26),
zero-copy and staged (DMA) retrieval from pinned-host objects, and the C ABI
called directly (ctypes) against the oracle."""

import ctypes

import numpy as np
import pytest
import torch

from lmcache_b200 import abi, c_ops
from lmcache_b200 import workloads as wl
from lmcache_b200.v1.memory_management import PinMemoryAllocator, TensorMemoryAllocator
from oracle import kv_transfer as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bits(t):
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.detach().cpu().contiguous().view(view).numpy()


def test_host_register_records_pinned_tensor():
    buf = torch.empty(1 << 20, dtype=torch.uint8, pin_memory=True)
    cap = c_ops.host_register(buf)
    assert cap is not None
    dev = c_ops.get_device_ptr(buf.data_ptr())
    assert dev != 0
    # interior addresses map with the same offset
    assert c_ops.get_device_ptr(buf.data_ptr() + 4096) == dev + 4096
    # one past the end is not registered
    assert c_ops.get_device_ptr(buf.data_ptr() + (1 << 20)) == 0
    # registering twice returns the same record
    c_ops.host_register(buf)
    lib = abi.load()
    assert lib.lmcb_host_record_size(ctypes.c_void_p(buf.data_ptr())) == 1 << 20
    c_ops.host_unregister(buf)
    assert c_ops.get_device_ptr(buf.data_ptr()) == 0


def test_host_register_pageable_memory_through_abi():
    """The C ABI pins and maps pageable memory (cudaHostRegister) and unpins it
    on unregister."""
    lib = abi.load()
    arr = np.zeros(1 << 16, dtype=np.uint8)
    dev = ctypes.c_void_p()
    abi.call("lmcb_host_register", arr.ctypes.data, arr.nbytes, ctypes.byref(dev))
    assert dev.value
    assert lib.lmcb_host_get_device_ptr(arr.ctypes.data) == dev.value
    abi.call("lmcb_host_unregister", arr.ctypes.data)
    assert lib.lmcb_host_get_device_ptr(arr.ctypes.data) is None


def test_host_register_rejects_device_memory():
    t = torch.empty(1024, device=DEV)
    lib = abi.load()
    dev = ctypes.c_void_p()
    st = lib.lmcb_host_register(t.data_ptr(), 4096, ctypes.byref(dev))
    assert st == abi.LMCB_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("mode", ["zerocopy", "dma"])
@pytest.mark.parametrize("name", ["c1", "c5"])
def test_pinned_retrieve_paths(mode, name, monkeypatch):
    """Retrieve from a pinned-host object through both host paths; the staged
    path copies the whole object into a device buffer and scatters on the
    GPU. Skipped slots must leave paged rows untouched in both."""
    monkeypatch.setenv("LMCB_HOST_RETRIEVE", mode)
    spec = wl.SPECS[name]
    kv = wl.make_kv_caches(spec, DEV, seed=3)
    slots = wl.make_slot_mapping(spec, seed=3)
    sc = wl.chunks(slots, spec.chunk_size)[0]
    sc[5] = -1
    arena = PinMemoryAllocator(64 << 20)
    obj = arena.allocate(spec.memobj_shape(len(sc)), torch.bfloat16).tensor
    obj.copy_(torch.randn(obj.shape).to(torch.bfloat16))
    before = [bits(t) for t in kv]
    c_ops.multi_layer_kv_transfer(obj, wl.pointer_tensor(kv, DEV), sc.to(DEV), kv[0].device,
                                  spec.page_buffer_size, False, False)
    torch.cuda.synchronize()
    oracle.multi_layer_kv_transfer(bits(obj), before, sc.numpy(), spec.page_buffer_size, False, False)
    for got, want in zip(kv, before):
        assert np.array_equal(bits(got), want)
    arena.close()


@pytest.mark.parametrize("mode", ["zerocopy", "dma"])
@pytest.mark.parametrize("name", ["c1", "c4", "c5"])
def test_pinned_store_paths(mode, name, monkeypatch):
    """Store into a pinned-host object through both host paths. The staged
    path gathers into a device buffer and copies it back with one DMA; rows
    of skipped slots must still keep the object's previous contents."""
    monkeypatch.setenv("LMCB_HOST_STORE", mode)
    spec = wl.SPECS[name]
    kv = wl.make_kv_caches(spec, DEV, seed=6)
    slots = wl.make_slot_mapping(spec, seed=6)
    sc = wl.chunks(slots, spec.chunk_size)[0].clone()
    sc[7] = -1
    sc[200] = -1
    arena = PinMemoryAllocator(64 << 20)
    obj = arena.allocate(spec.memobj_shape(len(sc)), torch.bfloat16).tensor
    obj.copy_(torch.randn(obj.shape).to(torch.bfloat16))  # previous contents
    want = bits(obj).copy()
    c_ops.multi_layer_kv_transfer(obj, wl.pointer_tensor(kv, DEV), sc.to(DEV), kv[0].device,
                                  spec.page_buffer_size, True, spec.use_mla)
    torch.cuda.synchronize()
    oracle.multi_layer_kv_transfer(want, [bits(t) for t in kv], sc.numpy(),
                                   spec.page_buffer_size, True, spec.use_mla)
    assert np.array_equal(bits(obj), want)
    arena.close()


def test_staged_retrieve_through_abi_and_capacity_error():
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=4)
    slots = wl.make_slot_mapping(spec, seed=4)
    host = torch.randn(spec.memobj_shape(len(slots))).to(torch.bfloat16).pin_memory()
    nbytes = host.numel() * 2
    staging = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    ptrs = wl.pointer_tensor(kv, DEV)
    sd = slots.to(DEV)
    stream = torch.cuda.current_stream().cuda_stream
    before = [bits(t) for t in kv]
    lib = abi.load()
    # too small a staging buffer is refused before any copy
    st = lib.lmcb_multi_layer_kv_retrieve_staged(
        abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, stream, ptrs.data_ptr(), host.data_ptr(),
        staging.data_ptr(), nbytes - 16, sd.data_ptr(), spec.hidden, 2, spec.num_layers,
        spec.page_buffer_size, len(slots))
    assert st == abi.LMCB_ERR_CAPACITY
    abi.call("lmcb_multi_layer_kv_retrieve_staged", abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64,
             stream, ptrs.data_ptr(), host.data_ptr(), staging.data_ptr(), nbytes, sd.data_ptr(),
             spec.hidden, 2, spec.num_layers, spec.page_buffer_size, len(slots))
    torch.cuda.synchronize()
    oracle.multi_layer_kv_transfer(bits(host), before, slots.numpy(), spec.page_buffer_size, False,
                                   False)
    for got, want in zip(kv, before):
        assert np.array_equal(bits(got), want)


@pytest.mark.parametrize("path", ["vector", "bulk"])
def test_abi_direct_store_matches_oracle(path, monkeypatch):
    """The C ABI called directly with raw device pointers and the current
    stream (what a non-Python host would bind)."""
    monkeypatch.setenv("LMCB_TRANSFER_PATH", path)
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=5)
    slots = wl.make_slot_mapping(spec, seed=5).to(torch.int32)
    obj = torch.zeros(spec.memobj_shape(len(slots)), dtype=torch.bfloat16, device=DEV)
    ptrs = wl.pointer_tensor(kv, DEV)
    sd = slots.to(DEV)
    abi.call("lmcb_multi_layer_kv_transfer_kernel", abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT32,
             torch.cuda.current_stream().cuda_stream, ptrs.data_ptr(), obj.data_ptr(),
             sd.data_ptr(), spec.hidden, 2, spec.num_layers, spec.page_buffer_size, len(slots), 1)
    torch.cuda.synchronize()
    want = np.zeros(obj.shape, dtype=np.int16)
    oracle.multi_layer_kv_transfer(want, [bits(t) for t in kv], slots.numpy(),
                                   spec.page_buffer_size, True, False)
    assert np.array_equal(bits(obj), want)


def test_pinned_allocator_reference_checks():
    """The allocator checks of LMCache-Ascend tests/v1/test_memory_management.py:22-67
    on the pinned, registered arena."""
    a = PinMemoryAllocator(16 << 20)
    d1 = a.allocate([512, 512], torch.float)
    assert d1.tensor.shape == (512, 512) and d1.tensor.dtype == torch.float
    assert c_ops.get_device_ptr(d1.tensor.data_ptr()) != 0
    d2 = a.allocate([1024, 1024], torch.bfloat16)
    d3 = a.allocate([2048, 2048], torch.int8)
    a.free(d2)
    assert d2.tensor is None and a.memcheck()
    a.free(d1)
    assert a.memcheck()
    a.free(d2)  # double free is harmless
    d4 = a.allocate([3, 5, 7], torch.half)
    assert d4.tensor.shape == (3, 5, 7)
    assert a.allocate([16 << 20], torch.float) is None
    for d in (d1, d2, d3, d4):
        a.free(d)
    assert a.memcheck()
    assert isinstance(a.allocator, TensorMemoryAllocator)
    a.close()
