"""ctypes binding of the C ABI in include/lmcache_b200.h.

The C ABI takes plain pointers, sizes and enums; this module declares the
argument types of every entry point so that Python callers (tests, benchmarks,
other FFI hosts) can call the library without the PyTorch extension. Pointers
are passed as Python ints (for example ``tensor.data_ptr()``) and streams as
``torch.cuda.current_stream().cuda_stream``.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_char_p, c_int, c_int32, c_int64, c_size_t, c_uint32, c_void_p

LIBRARY_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "liblmcache_b200.so")

# lmcb_status
LMCB_OK = 0
LMCB_ERR_INVALID_ARGUMENT = 1
LMCB_ERR_UNSUPPORTED_DTYPE = 2
LMCB_ERR_CUDA = 3
LMCB_ERR_NOT_REGISTERED = 4
LMCB_ERR_NOT_IMPLEMENTED = 5
LMCB_ERR_CAPACITY = 6

# lmcb_dtype
LMCB_DTYPE_FP32 = 0
LMCB_DTYPE_BF16 = 1
LMCB_DTYPE_FP16 = 2
LMCB_DTYPE_INT64 = 3
LMCB_DTYPE_INT32 = 4

LMCB_DEVICE_FLAG_SLOT_OUT_OF_RANGE = 0x1
LMCB_DEVICE_FLAG_SYMBOL_OUT_OF_RANGE = 0x2
LMCB_DEVICE_FLAG_STREAM_OVERFLOW = 0x4
LMCB_DEVICE_FLAG_WAIT_TIMEOUT = 0x8
LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE = 0x10

LMCB_NOALLOC_STAGING_BYTES = 64 << 20

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "lmcb_version": (c_char_p, []),
    "lmcb_last_error": (c_char_p, []),
    "lmcb_status_string": (c_char_p, [c_int]),
    "lmcb_dtype_size": (c_int, [c_int]),
    "lmcb_multi_layer_kv_transfer_kernel": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32,
         c_int64, c_int32, c_int],
    ),
    "lmcb_multi_layer_kv_transfer_unilateral_kernel": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
         c_int64, c_int32, c_int],
    ),
    "lmcb_multi_layer_kv_transfer_batched_kernel": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int,
         c_void_p, c_int64, c_int32, c_int32, c_int64, c_int32, c_int],
    ),
    "lmcb_single_layer_kv_transfer_batched_kernel": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int, c_void_p,
         c_void_p, c_void_p, c_int64, c_int32, c_int, c_int, c_int64, c_int64],
    ),
    "lmcb_single_layer_kv_transfer_kernel": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
         c_int, c_int, c_int, c_int64, c_int64],
    ),
    "lmcb_load_and_reshape_flash_kernel": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
         c_int32, c_int32, c_int32, c_int32, c_int, c_int64],
    ),
    "lmcb_multi_layer_kv_retrieve_staged": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_int64,
         c_int32, c_int32, c_int64, c_int32],
    ),
    "lmcb_multi_layer_kv_store_staged": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p,
         c_int64, c_int32, c_int32, c_int64, c_int32],
    ),
    "lmcb_multi_layer_kv_retrieve_staged_noalloc": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32,
         c_int64, c_int32],
    ),
    "lmcb_device_status": (c_int, [c_int, ctypes.POINTER(c_uint32)]),
    "lmcb_host_register": (c_int, [c_void_p, c_size_t, ctypes.POINTER(c_void_p)]),
    "lmcb_host_unregister": (c_int, [c_void_p]),
    "lmcb_host_get_device_ptr": (c_void_p, [c_void_p]),
    "lmcb_host_record_size": (c_size_t, [c_void_p]),
    "lmcb_host_unregister_all": (c_int, []),
    "lmcb_calculate_cdf": (
        c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "lmcb_encode": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int64,
         c_void_p],
    ),
    "lmcb_decode": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int64,
         c_void_p],
    ),
    "lmcb_decode_prefsum": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
         c_void_p],
    ),
    "lmcb_rotary_embedding_k_fused": (
        c_int,
        [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int64, c_int64, c_int64, c_int64,
         c_void_p, c_int, c_int64, c_int64, c_int, c_void_p],
    ),
}


class LmcbError(RuntimeError):
    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} -> {status}: {message}")
        self.status = status


_LIB = None


def load(path: str = LIBRARY_PATH) -> ctypes.CDLL:
    """Loads the library once and declares every entry point's signature."""
    global _LIB
    if _LIB is None:
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def call(name: str, *args) -> int:
    """Calls a status-returning entry point and raises LmcbError on failure."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != LMCB_OK:
        raise LmcbError(name, status, lib.lmcb_last_error().decode())
    return status


def torch_dtype_code(dtype) -> int:
    import torch

    return {
        torch.float32: LMCB_DTYPE_FP32,
        torch.bfloat16: LMCB_DTYPE_BF16,
        torch.float16: LMCB_DTYPE_FP16,
        torch.int64: LMCB_DTYPE_INT64,
        torch.int32: LMCB_DTYPE_INT32,
    }[dtype]
