"""CPU tests of the native boundary: the C ABI library loads and exports every
symbol include/*.h declares, argument errors are reported without touching a
GPU, and the c_ops module mirrors the reference's pybind surface
(csrc/pybind.cpp:13-26) including its error behaviour."""

import ctypes
import glob
import os
import re
import sys

import pytest
import torch

from lmcache_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REFERENCE_NAMES = [
    "host_register",
    "multi_layer_kv_transfer",
    "single_layer_kv_transfer",
    "multi_layer_kv_transfer_unilateral",
    "load_and_reshape_flash",
    "reshape_and_cache_back_flash",
    "encode_fast_new",
    "decode_fast_new",
    "decode_fast_prefsum",
    "calculate_cdf",
    "rotary_embedding_k_fused",
]


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        with open(h) as f:
            text = f.read()
        names.update(re.findall(r"LMCB_API\s+[\w\s\*]+?\b(lmcb_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "lmcb_multi_layer_kv_transfer_kernel" in names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    # and the ctypes signature table covers them all
    assert set(declared_symbols()) == set(abi.SIGNATURES)


def test_version_and_status_strings():
    lib = abi.load()
    assert lib.lmcb_version().decode().count(".") == 2
    assert lib.lmcb_status_string(abi.LMCB_OK) == b"LMCB_OK"
    assert lib.lmcb_status_string(abi.LMCB_ERR_CAPACITY) == b"LMCB_ERR_CAPACITY"
    assert [lib.lmcb_dtype_size(d) for d in range(5)] == [4, 2, 2, 8, 4]
    assert lib.lmcb_dtype_size(42) == 0


def test_argument_errors_need_no_gpu():
    lib = abi.load()
    # unsupported element type
    st = lib.lmcb_multi_layer_kv_transfer_kernel(42, abi.LMCB_DTYPE_INT64, None, 8, 8, 8, 1024, 2,
                                                 1, 16, 4, 1)
    assert st == abi.LMCB_ERR_UNSUPPORTED_DTYPE
    assert b"ScalarType not supported" in lib.lmcb_last_error()
    # bad slot type
    st = lib.lmcb_multi_layer_kv_transfer_kernel(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_FP32, None, 8,
                                                 8, 8, 1024, 2, 1, 16, 4, 1)
    assert st == abi.LMCB_ERR_UNSUPPORTED_DTYPE
    # kvs must be 1 or 2
    st = lib.lmcb_multi_layer_kv_transfer_kernel(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None,
                                                 8, 8, 8, 1024, 3, 1, 16, 4, 1)
    assert st == abi.LMCB_ERR_INVALID_ARGUMENT
    # K/V caches need a page buffer size
    st = lib.lmcb_multi_layer_kv_transfer_kernel(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None,
                                                 8, 8, 8, 1024, 2, 1, 0, 4, 1)
    assert st == abi.LMCB_ERR_INVALID_ARGUMENT
    # zero tokens is a no-op that succeeds without a device
    st = lib.lmcb_multi_layer_kv_transfer_kernel(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None,
                                                 None, None, None, 1024, 2, 4, 16, 0, 1)
    assert st == abi.LMCB_OK
    # NULL pointers with work to do
    st = lib.lmcb_single_layer_kv_transfer_kernel(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None,
                                                  None, None, None, None, 1024, 4, 1, 1, 0, 0, 0)
    assert st == abi.LMCB_ERR_INVALID_ARGUMENT
    # flash: layer index out of range
    st = lib.lmcb_load_and_reshape_flash_kernel(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None,
                                                8, 8, 8, 8, 1024, 10, 16, 4, 2, 5, 1, 0)
    assert st == abi.LMCB_ERR_INVALID_ARGUMENT
    # staged retrieve: staging buffer too small
    st = lib.lmcb_multi_layer_kv_retrieve_staged(abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None,
                                                 8, 8, 8, 100, 8, 1024, 2, 2, 16, 4)
    assert st == abi.LMCB_ERR_CAPACITY
    # codec argument checks
    assert lib.lmcb_calculate_cdf(8, 8, 1, 4, 4, 0, None) == abi.LMCB_ERR_INVALID_ARGUMENT
    assert lib.lmcb_calculate_cdf(8, 8, 1, 4, 4, 257, None) == abi.LMCB_ERR_INVALID_ARGUMENT
    assert lib.lmcb_encode(8, 8, 8, 8, 1, 4, 4, 16, 0, None) == abi.LMCB_ERR_INVALID_ARGUMENT
    assert lib.lmcb_decode_prefsum(8, 8, -1, 8, 8, 1, 4, 4, 16, None) == abi.LMCB_ERR_INVALID_ARGUMENT
    # rotary: odd rotary width, unsupported dtype
    assert lib.lmcb_rotary_embedding_k_fused(8, 8, abi.LMCB_DTYPE_INT64, 8, abi.LMCB_DTYPE_BF16,
                                             4, 2, 64, 128, 8, abi.LMCB_DTYPE_FP32, 63, 100, 1,
                                             None) == abi.LMCB_ERR_INVALID_ARGUMENT
    assert lib.lmcb_rotary_embedding_k_fused(8, 8, abi.LMCB_DTYPE_INT64, 8, abi.LMCB_DTYPE_INT32,
                                             4, 2, 64, 128, 8, abi.LMCB_DTYPE_FP32, 64, 100, 1,
                                             None) == abi.LMCB_ERR_UNSUPPORTED_DTYPE
    # batched transfer: negative object count
    assert lib.lmcb_multi_layer_kv_transfer_batched_kernel(
        abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None, 8, 8, 8, 8, -1, 1, 8, 1024, 2, 4, 16,
        4, 1) == abi.LMCB_ERR_INVALID_ARGUMENT
    # batched transfer: the object table is host memory and checked before any
    # launch (token offsets that do not add up, a descending range, a NULL
    # object holding tokens)
    ptrs = (ctypes.c_uint64 * 2)(4096, 8192)
    starts = (ctypes.c_int64 * 2)(0, 3)
    for offs, total in (((0, 3, 5), 4), ((0, 3, 2), 2), ((0, 3, 5), 5)):
        o = (ctypes.c_int64 * 3)(*offs)
        p = ptrs if offs != (0, 3, 5) or total != 5 else (ctypes.c_uint64 * 2)(4096, 0)
        assert lib.lmcb_multi_layer_kv_transfer_batched_kernel(
            abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, None, 8, p, o, starts, 2, 1, 8, 1024, 2,
            4, 16, total, 1) == abi.LMCB_ERR_INVALID_ARGUMENT, offs
    # host registry
    assert lib.lmcb_host_register(None, 16, None) == abi.LMCB_ERR_INVALID_ARGUMENT
    assert lib.lmcb_host_get_device_ptr(None) is None
    assert lib.lmcb_host_record_size(None) == 0
    assert lib.lmcb_host_unregister(None) == abi.LMCB_ERR_INVALID_ARGUMENT


def test_c_ops_surface_matches_reference():
    from lmcache_b200 import c_ops

    for name in REFERENCE_NAMES:
        assert callable(getattr(c_ops, name)), name
    # installed as lmcache.c_ops (lmcache_ascend/__init__.py:8)
    assert sys.modules["lmcache.c_ops"] is c_ops


def test_c_ops_rotary_rejects_cpu_tensors():
    """The reference's rotary_embedding_k_fused is a stub; here it is
    implemented for CUDA tensors and rejects anything else."""
    from lmcache_b200 import c_ops

    t = torch.zeros(4)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        c_ops.rotary_embedding_k_fused(t, t, t, 4, t, True)


def test_c_ops_errors_match_reference_messages():
    from lmcache_b200 import c_ops

    # managed_mem.cpp:296-301
    with pytest.raises(RuntimeError, match="Device must be CPU and tensor must be pinned"):
        c_ops.host_register(torch.zeros(16))
    # utils.h:36
    with pytest.raises(RuntimeError, match="ScalarType not supported"):
        c_ops.multi_layer_kv_transfer(torch.zeros(2, 1, 4, 8, dtype=torch.uint8),
                                      torch.zeros(1, dtype=torch.int64),
                                      torch.zeros(4, dtype=torch.int64), torch.device("cpu"), 16,
                                      True, False)
    with pytest.raises(RuntimeError, match="ScalarType not supported"):
        c_ops.multi_layer_kv_transfer(torch.zeros(2, 1, 4, 8, dtype=torch.bfloat16),
                                      torch.zeros(1, dtype=torch.int64),
                                      torch.zeros(4, dtype=torch.float32), torch.device("cpu"), 16,
                                      True, False)
    # the paged cache must be on a CUDA device
    with pytest.raises(RuntimeError, match="must be a CUDA device"):
        c_ops.multi_layer_kv_transfer(torch.zeros(2, 1, 4, 8, dtype=torch.bfloat16),
                                      torch.zeros(1, dtype=torch.int64),
                                      torch.zeros(4, dtype=torch.int64), torch.device("cpu"), 16,
                                      True, False)
    # shape checks come before any device work
    with pytest.raises(RuntimeError, match="smaller than"):
        c_ops.multi_layer_kv_transfer(torch.zeros(2, 1, 2, 8, dtype=torch.bfloat16),
                                      torch.zeros(1, dtype=torch.int64),
                                      torch.zeros(4, dtype=torch.int64), torch.device("cpu"), 16,
                                      True, False)
