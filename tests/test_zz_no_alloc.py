"""GPU test of lmcb_multi_layer_kv_retrieve_staged_noalloc, the staged retrieve
for callers that cannot allocate device memory when they retrieve (an engine
that reserved nearly all HBM for its KV cache, or a native host where a
cudaMalloc / cudaFree per chunk would synchronise the device).

It is called through the C ABI and must produce exactly what the existing
entry point, lmcb_multi_layer_kv_retrieve_staged with a caller-allocated
staging buffer, produces (the path is a pure copy, so "within tolerance" here
means bit-identical), on two calls in a row: the second call uses a smaller
object, so bytes the first call left in the built-in staging area must not
leak into its result. Objects larger than the area are refused before any
work is queued. This file is collected last and also passes on its own.
"""

import numpy as np
import pytest
import torch

from lmcache_b200 import abi
from lmcache_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _call_staged(fn_name, extra, spec, kv, host, slots):
    """Calls one of the two staged-retrieve entry points on the current stream."""
    stream = torch.cuda.current_stream().cuda_stream
    ptrs = wl.pointer_tensor(kv, DEV)
    sd = slots.to(DEV)
    common = (abi.LMCB_DTYPE_BF16, abi.LMCB_DTYPE_INT64, stream, ptrs.data_ptr(),
              host.data_ptr())
    tail = (sd.data_ptr(), spec.hidden, spec.kv, spec.num_layers, spec.page_buffer_size,
            len(slots))
    abi.call(fn_name, *common, *extra, *tail)
    torch.cuda.synchronize()


def _one_call(spec, seed):
    """Retrieves one seeded object into two identical copies of seeded caches,
    once per entry point; returns both sets of caches."""
    base = wl.make_kv_caches(spec, DEV, seed=seed)
    slots = wl.make_slot_mapping(spec, seed=seed)[: spec.chunk_size].clone()
    slots[3] = -1  # a skipped row must stay untouched
    g = torch.Generator().manual_seed(seed)
    host = torch.randn(spec.memobj_shape(len(slots)), generator=g).to(torch.bfloat16)
    host = host.pin_memory()
    nbytes = host.numel() * host.element_size()
    assert nbytes <= abi.LMCB_NOALLOC_STAGING_BYTES

    ref_kv = [t.clone() for t in base]
    staging = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    _call_staged("lmcb_multi_layer_kv_retrieve_staged", (staging.data_ptr(), nbytes), spec,
                 ref_kv, host, slots)

    new_kv = [t.clone() for t in base]
    _call_staged("lmcb_multi_layer_kv_retrieve_staged_noalloc", (), spec, new_kv, host, slots)
    return base, ref_kv, new_kv, slots


def test_noalloc_retrieve_matches_staged_retrieve_twice():
    # First call: a full c2 chunk (32 MiB object); second: a smaller c1 object.
    for name, seed in (("c2", 31), ("c1", 32)):
        spec = wl.SPECS[name]
        base, ref_kv, new_kv, slots = _one_call(spec, seed)
        for a, b in zip(ref_kv, new_kv):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        # the retrieve did write the rows (the comparison is not vacuous) ...
        valid = slots[slots >= 0].to(DEV)
        changed = (ref_kv[0].view(2, -1, spec.hidden)[:, valid] !=
                   base[0].view(2, -1, spec.hidden)[:, valid])
        assert bool(changed.any())
        # ... and the skipped row kept its value
        skipped = int(wl.make_slot_mapping(spec, seed=seed)[3])
        if skipped >= 0:
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
