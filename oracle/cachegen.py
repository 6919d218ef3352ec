"""numpy wrappers of the C CacheGen oracle (oracle/cachegen_ref.c).

Test infrastructure only. The format (CDF definition and range coder) is
documented at the top of cachegen_ref.c.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import native

_P = ctypes.c_void_p


def _lib():
    lib = native.load()
    if not getattr(lib, "_cg_declared", False):
        lib.oracle_calculate_cdf.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, _P]
        lib.oracle_calculate_cdf.restype = ctypes.c_int
        lib.oracle_encode.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, _P, ctypes.c_int64, _P]
        lib.oracle_encode.restype = ctypes.c_int
        lib.oracle_decode.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int64, _P]
        lib.oracle_decode.restype = None
        lib.oracle_decode_prefsum.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, _P]
        lib.oracle_decode_prefsum.restype = None
        lib._cg_declared = True
    return lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def calculate_cdf(sym: np.ndarray, max_bins: int) -> np.ndarray:
    """sym [L, T, C] (int8/uint8) -> cdf [L, C, max_bins + 1] as int16 bit patterns."""
    s = np.ascontiguousarray(sym).view(np.uint8)
    L, T, C = s.shape
    cdf = np.zeros((L, C, max_bins + 1), dtype=np.uint16)
    _lib().oracle_calculate_cdf(_ptr(s), L, T, C, max_bins, _ptr(cdf))
    return cdf.view(np.int16)


def encode(cdf: np.ndarray, sym: np.ndarray, cap: int) -> tuple[np.ndarray, np.ndarray]:
    """-> (bytestreams uint8 [L, C, cap], lengths int32 [L, C])."""
    s = np.ascontiguousarray(sym).view(np.uint8)
    c = np.ascontiguousarray(cdf).view(np.uint16)
    L, T, C = s.shape
    out = np.zeros((L, C, cap), dtype=np.uint8)
    lengths = np.zeros((L, C), dtype=np.int32)
    _lib().oracle_encode(_ptr(c), _ptr(s), L, T, C, c.shape[-1] - 1, _ptr(out), cap,
                         _ptr(lengths))
    return out, lengths


def decode(cdf: np.ndarray, streams: np.ndarray, lengths: np.ndarray, num_tokens: int) -> np.ndarray:
    """-> symbols uint8 [L, T, C]."""
    c = np.ascontiguousarray(cdf).view(np.uint16)
    st = np.ascontiguousarray(streams).view(np.uint8)
    ln = np.ascontiguousarray(lengths).astype(np.int32)
    L, C, cap = st.shape
    out = np.zeros((L, num_tokens, C), dtype=np.uint8)
    _lib().oracle_decode(_ptr(c), _ptr(st), _ptr(ln), L, num_tokens, C, c.shape[-1] - 1, cap,
                         _ptr(out))
    return out


def decode_prefsum(cdf: np.ndarray, concat: np.ndarray, ends: np.ndarray, num_tokens: int) -> np.ndarray:
    c = np.ascontiguousarray(cdf).view(np.uint16)
    st = np.ascontiguousarray(concat).view(np.uint8)
    e = np.ascontiguousarray(ends).astype(np.int64)
    L, C = c.shape[0], c.shape[1]
    out = np.zeros((L, num_tokens, C), dtype=np.uint8)
    _lib().oracle_decode_prefsum(_ptr(c), _ptr(st), _ptr(e), L, num_tokens, C, c.shape[-1] - 1,
                                 _ptr(out))
    return out


def concat_streams(streams: np.ndarray, lengths: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[L, C, cap] + lengths -> (concatenated bytes, inclusive end offsets [L*C])."""
    L, C, _ = streams.shape
    ln = lengths.reshape(-1).astype(np.int64)
    parts = [streams.reshape(L * C, -1)[i, : ln[i]] for i in range(L * C)]
    ends = np.cumsum(ln)
    return (np.concatenate(parts) if parts else np.zeros(0, np.uint8)), ends
