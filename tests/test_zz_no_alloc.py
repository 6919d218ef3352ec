"""GPU test of lmcb_multi_layer_kv_retrieve_staged_noalloc, the staged retrieve
for callers that cannot allocate device memory when they retrieve (an engine
that reserved nearly all HBM for its KV cache, or a native host where a
cudaMalloc / cudaFree per chunk would synchronise the device).

It is called through the C ABI and must produce exactly what the existing
entry point, lmcb_multi_layer_kv_retrieve_staged with a caller-allocated
staging buffer, produces (the path is a pure copy, so "within tolerance" here
means bit-identical), on two calls in a row.

The first call fills the built-in staging area with a sentinel bit pattern
(a full c2 chunk whose every element is the sentinel). The second retrieves a
smaller object whose slot mapping skips some rows; the sentinel must appear
nowhere in its result, so bytes an earlier call left in the area never reach
the caches. Objects larger than the area, and calls with invalid arguments,
are refused before any work is queued. This file is collected last and also
passes on its own.
"""

import numpy as np
import pytest
import torch

from lmcache_b200 import abi
from lmcache_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = "cuda"
# bf16 bit pattern 0x7F7B (about 3.3e38): never drawn by the seeded N(0, 1) generators
SENTINEL = 0x7F7B


def _call_staged(fn_name, extra, spec, kv, host, slots):
    """Calls one of the two staged-retrieve entry points on the current stream;
    returns its status."""
    stream = torch.cuda.current_stream().cuda_stream
    ptrs = wl.pointer_tensor(kv, DEV)
    sd = slots.to(DEV)
    common = (abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, stream, ptrs.data_ptr(),
              host.data_ptr())
    tail = (sd.data_ptr(), spec.hidden, spec.kv, spec.num_layers, spec.page_buffer_size,
            len(slots))
    st = getattr(abi.load(), fn_name)(*common, *extra, *tail)
    torch.cuda.synchronize()
    return st


def _fill_area_with_sentinel():
    """A noalloc retrieve of a full c2 chunk whose every element is SENTINEL:
    afterwards the first 32 MiB of the staging area hold the sentinel."""
    spec = wl.SPECS["c2"]
    kv = wl.make_kv_caches(spec, DEV, seed=40)
    slots = wl.make_slot_mapping(spec, seed=40)[: spec.chunk_size].clone()
    host = torch.full(spec.memobj_shape(len(slots)), SENTINEL, dtype=torch.int16)
    host = host.view(torch.bfloat16).pin_memory()
    st = _call_staged("lmcb_multi_layer_kv_retrieve_staged_noalloc", (), spec, kv, host, slots)
    assert st == abi.LMCB_OK, abi.load().lmcb_last_error().decode()
    valid = slots[slots >= 0].to(DEV)
    rows = kv[0].view(2, -1, spec.hidden)[:, valid].view(torch.int16)
    assert bool((rows == SENTINEL).all())  # the area really held the sentinel
    del kv
    torch.cuda.empty_cache()


def _one_call(spec, seed, n_skipped):
    """Retrieves one seeded object into two identical copies of seeded caches,
    once per entry point; returns the base caches, both results and the slots."""
    base = wl.make_kv_caches(spec, DEV, seed=seed)
    slots = wl.make_slot_mapping(spec, seed=seed)[: spec.chunk_size].clone()
    slots[3: 3 + 5 * n_skipped: 5] = -1  # skipped rows must stay untouched
    g = torch.Generator().manual_seed(seed)
    host = torch.randn(spec.memobj_shape(len(slots)), generator=g).to(torch.bfloat16)
    host = host.pin_memory()
    nbytes = host.numel() * host.element_size()
    assert nbytes <= abi.LMCB_NOALLOC_STAGING_BYTES

    ref_kv = [t.clone() for t in base]
    staging = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    st = _call_staged("lmcb_multi_layer_kv_retrieve_staged", (staging.data_ptr(), nbytes), spec,
                      ref_kv, host, slots)
    assert st == abi.LMCB_OK, abi.load().lmcb_last_error().decode()

    new_kv = [t.clone() for t in base]
    st = _call_staged("lmcb_multi_layer_kv_retrieve_staged_noalloc", (), spec, new_kv, host,
                      slots)
    assert st == abi.LMCB_OK, abi.load().lmcb_last_error().decode()
    return base, ref_kv, new_kv, slots


def test_noalloc_retrieve_matches_staged_retrieve_twice():
    _fill_area_with_sentinel()
    # Two calls in a row after the sentinel fill: a full c2 chunk (32 MiB),
    # then a smaller c1 object (4 MiB), both with skipped rows.
    for name, seed, n_skipped in (("c2", 31, 4), ("c1", 32, 6)):
        spec = wl.SPECS[name]
        base, ref_kv, new_kv, slots = _one_call(spec, seed, n_skipped)
        for a, b in zip(ref_kv, new_kv):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
            assert not bool((b.view(torch.int16) == SENTINEL).any())
        # the retrieve did write the rows (the comparison is not vacuous) ...
        valid = slots[slots >= 0].to(DEV)
        changed = (ref_kv[0].view(2, -1, spec.hidden)[:, valid] !=
                   base[0].view(2, -1, spec.hidden)[:, valid])
        assert bool(changed.any())
        # ... and the skipped rows kept their values
        full = wl.make_slot_mapping(spec, seed=seed)[: spec.chunk_size]
        skipped = full[(slots < 0) & (full >= 0)].to(DEV)
        assert skipped.numel() > 0
        for a, b in zip(new_kv, base):
            assert torch.equal(a.view(2, -1, spec.hidden)[:, skipped],
                               b.view(2, -1, spec.hidden)[:, skipped])
        del base, ref_kv, new_kv
        torch.cuda.empty_cache()


def test_noalloc_rejects_objects_larger_than_the_staging_area():
    lib = abi.load()
    spec = wl.SPECS["c3"]  # 2 x 64 layers x 256 tokens x 1024 x 2 B = 64 MiB
    tokens = 300  # 75 MiB object
    st = lib.lmcb_multi_layer_kv_retrieve_staged_noalloc(
        abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, torch.cuda.current_stream().cuda_stream,
        8, 8, 8, spec.hidden, 2, spec.num_layers, spec.page_buffer_size, tokens)
    assert st == abi.LMCB_ERR_CAPACITY
    assert b"staging area holds" in lib.lmcb_last_error()
    assert np.isclose(2 * spec.num_layers * tokens * spec.hidden * 2 / 2**20, 75.0)
    # a hidden size whose byte count wraps 64 bits is refused as well
    st = lib.lmcb_multi_layer_kv_retrieve_staged_noalloc(
        abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, torch.cuda.current_stream().cuda_stream,
        8, 8, 8, 1 << 62, 2, 1, 16, 1)
    assert st == abi.LMCB_ERR_CAPACITY


@pytest.mark.parametrize("bad", ["slot_dtype", "page_buffer_size", "null_pointers", "kvs"])
def test_staged_retrieve_with_bad_arguments_queues_no_copy(bad):
    """The staged retrieve checks every argument before it queues the copy
    into the staging buffer: a refused call leaves the buffer as it was."""
    spec = wl.SPECS["c1"]
    kv = wl.make_kv_caches(spec, DEV, seed=41)
    slots = wl.make_slot_mapping(spec, seed=41)
    host = torch.randn(spec.memobj_shape(len(slots))).to(torch.bfloat16).pin_memory()
    nbytes = host.numel() * host.element_size()
    staging = torch.full((nbytes,), 0x5A, dtype=torch.uint8, device=DEV)
    ptrs = wl.pointer_tensor(kv, DEV)
    sd = slots.to(DEV)
    slot_type, pbs, kvs = abi.LMCB_DTYPE_INT64, spec.page_buffer_size, spec.kv
    ptr_arg = ptrs.data_ptr()
    if bad == "slot_dtype":
        slot_type = abi.LMCB_DTYPE_FP32
    elif bad == "page_buffer_size":
        pbs = 0
    elif bad == "null_pointers":
        ptr_arg = None
    else:
        kvs = 3
    st = abi.load().lmcb_multi_layer_kv_retrieve_staged(
        abi.LMCB_DTYPE_BF16, slot_type, torch.cuda.current_stream().cuda_stream, ptr_arg,
        host.data_ptr(), staging.data_ptr(), nbytes, sd.data_ptr(), spec.hidden, kvs,
        spec.num_layers, pbs, len(slots))
    torch.cuda.synchronize()
    assert st != abi.LMCB_OK
    assert bool((staging == 0x5A).all())
