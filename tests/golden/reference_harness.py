"""Runs LMCache-Ascend's own transfer tests, unmodified, on the CPU oracle.

Test infrastructure. The reference's tests/v1/test_mem_kernels.py (with its
helpers tests/v1/utils.py) is imported from the reference checkout and its
four test functions -- test_extract_and_load_back, test_multi_layer_kernel,
test_multi_layer_kernel_use_mla and test_single_layer_kernel -- are called as
they are. Only what this container lacks is stood in for:

  * ``lmcache.c_ops`` -> OracleCOps: the reference's op names and positional
    arguments, computed by the numpy oracle (oracle/kv_transfer.py) on CPU
    tensors. Pointer arrays (``kv_cache[i].data_ptr()``) are resolved through
    a registry of the tensors the test created.
  * ``lmcache_ascend.v1.memory_management.AscendPinMemoryAllocator`` ->
    RecordingAllocator: zero-filled CPU objects, recorded in allocation order.
  * ``lmcache.config`` / ``lmcache.utils`` / ``lmcache_ascend.v1.npu_connector``
    -> the names tests/v1/utils.py imports at module level (unused by the four
    tests).
  * ``device="cuda"`` -> CPU: torch.rand / torch.tensor / torch.empty drop the
    device and pin_memory arguments, Tensor.cuda() returns the tensor,
    torch.cuda.Event and torch.cuda.synchronize are no-ops (the tests only
    print the timings).

Every test is seeded here (``random.seed`` and ``torch.manual_seed`` before the
call); the reference file is not edited. The reference's own assertions
(check_mem_obj_equal, check_paged_kv_cache_equal, the MLA per-token loop
comparison) then check the oracle. ``run_case`` also returns SHA-256 digests
of the inputs the test drew, of every object it allocated (in order: where a
test fills its first objects with its own torch expressions, they come first)
and of the tensors it created, after the test: make_reference_digests.py
stores them as fixtures for the GPU parity test, which cannot read the
reference.

The reference checkout is found at $LMCB_REFERENCE_ROOT, default
/root/reference.
"""

from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import os
import random
import sys
import types

import numpy as np
import torch

from oracle import kv_transfer as oracle

REFERENCE_ROOT = os.environ.get("LMCB_REFERENCE_ROOT", "/root/reference")
REFERENCE_TESTS = os.path.join(REFERENCE_ROOT, "tests", "v1")
TEST_FILE = os.path.join(REFERENCE_TESTS, "test_mem_kernels.py")

# test function -> its parameter names (tests/v1/test_mem_kernels.py)
TESTS = {
    "test_extract_and_load_back": ("num_tokens",),
    "test_multi_layer_kernel": ("num_tokens",),
    "test_multi_layer_kernel_use_mla": ("num_tokens",),
    "test_single_layer_kernel": ("num_tokens", "token_major"),
}
NUM_TOKENS = (256, 500, 1024, 8000)
# One seed per test function, whatever its parameters: the paged caches a
# test draws are then the same for every num_tokens, and the GPU test
# regenerates them once per function.
SEEDS = {
    "test_extract_and_load_back": 1001,
    "test_multi_layer_kernel": 1002,
    "test_multi_layer_kernel_use_mla": 1003,
    "test_single_layer_kernel": 1004,
}


def available() -> bool:
    return os.path.isfile(TEST_FILE) and os.path.isfile(os.path.join(REFERENCE_TESTS, "utils.py"))


def bits(t: torch.Tensor) -> np.ndarray:
    """Bit view of a CPU tensor as a numpy integer array (shares memory)."""
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.detach().view(view).numpy()


def sha256_of(t: torch.Tensor) -> str:
    return hashlib.sha256(np.ascontiguousarray(bits(t))).hexdigest()


class TensorRegistry:
    """Tensors created through the patched torch.rand, by data_ptr, plus a
    running digest of their values at creation."""

    def __init__(self):
        self.by_ptr: dict[int, torch.Tensor] = {}
        self.created: list[torch.Tensor] = []
        self.input_hash = hashlib.sha256()
        self.c_ops = None

    def add(self, t: torch.Tensor) -> None:
        self.by_ptr[t.data_ptr()] = t
        self.created.append(t)
        self.input_hash.update(np.ascontiguousarray(bits(t)))

    def lookup(self, ptr: int) -> torch.Tensor:
        try:
            return self.by_ptr[int(ptr)]
        except KeyError as exc:
            raise RuntimeError(f"pointer {ptr:#x} names no tensor the test created") from exc


class OracleCOps(types.ModuleType):
    """The reference's c_ops surface (csrc/pybind.cpp:13-26) for the four
    transfer ops the tests call, computed by the numpy oracle."""

    def __init__(self, registry: TensorRegistry):
        super().__init__("lmcache.c_ops")
        self.registry = registry
        self.lmc_buffers: list[torch.Tensor] = []  # single-layer buffers, first-use order

    def multi_layer_kv_transfer(self, key_value, key_value_ptrs, slot_mapping, device,
                                page_buffer_size, direction, use_mla):
        layers = [bits(self.registry.lookup(p)) for p in key_value_ptrs.tolist()]
        oracle.multi_layer_kv_transfer(bits(key_value), layers, slot_mapping.numpy(),
                                       int(page_buffer_size), bool(direction), bool(use_mla))

    def single_layer_kv_transfer(self, lmc_kv, key_cache, value_cache, slot_mapping, direction,
                                 token_major):
        if not any(b is lmc_kv for b in self.lmc_buffers):
            self.lmc_buffers.append(lmc_kv)
        oracle.single_layer_kv_transfer(bits(lmc_kv), bits(key_cache), bits(value_cache),
                                        slot_mapping.numpy(), bool(direction), bool(token_major))

    def load_and_reshape_flash(self, key_value, key_cache, value_cache, slot_mapping, layer_idx):
        oracle.load_and_reshape_flash(bits(key_value), bits(key_cache), bits(value_cache),
                                      slot_mapping.numpy(), int(layer_idx))

    def reshape_and_cache_back_flash(self, key_value, key_cache, value_cache, slot_mapping,
                                     layer_idx):
        oracle.reshape_and_cache_back_flash(bits(key_value), bits(key_cache), bits(value_cache),
                                            slot_mapping.numpy(), int(layer_idx))


class _MemoryObj:
    def __init__(self, tensor: torch.Tensor):
        self.tensor = tensor


class RecordingAllocator:
    """Stands in for AscendPinMemoryAllocator(size): zero-filled CPU objects,
    every allocation recorded in order (class-wide, cleared per case)."""

    allocations: list = []

    def __init__(self, size: int):
        self.size = size

    def allocate(self, shape, dtype):
        obj = _MemoryObj(torch.zeros(list(shape), dtype=dtype))
        RecordingAllocator.allocations.append(obj)
        return obj

    def close(self):
        pass


class _Event:
    def __init__(self, *args, **kwargs):
        pass

    def record(self, *args, **kwargs):
        pass

    def elapsed_time(self, other):
        return 0.0


class _Stub:
    def __init__(self, *args, **kwargs):
        self.args, self.kwargs = args, kwargs


def _module(name: str, **attrs) -> types.ModuleType:
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    return m


@contextlib.contextmanager
def reference_environment(registry: TensorRegistry):
    """Installs the stand-ins and the CPU device mapping; restores everything
    on exit."""
    c_ops = OracleCOps(registry)
    registry.c_ops = c_ops
    fake = {
        "lmcache": _module("lmcache", c_ops=c_ops),
        "lmcache.c_ops": c_ops,
        "lmcache.config": _module("lmcache.config", LMCacheEngineMetadata=_Stub),
        "lmcache.utils": _module("lmcache.utils", CacheEngineKey=_Stub),
        "lmcache_ascend": _module("lmcache_ascend"),
        "lmcache_ascend.v1": _module("lmcache_ascend.v1"),
        "lmcache_ascend.v1.memory_management": _module(
            "lmcache_ascend.v1.memory_management", AscendPinMemoryAllocator=RecordingAllocator),
        "lmcache_ascend.v1.npu_connector": _module(
            "lmcache_ascend.v1.npu_connector", VLLMPagedMemNPUConnectorV2=_Stub),
    }
    saved_modules = {k: sys.modules.get(k) for k in list(fake) + ["utils"]}
    real = {"rand": torch.rand, "tensor": torch.tensor, "empty": torch.empty,
            "cuda": torch.Tensor.cuda, "Event": torch.cuda.Event,
            "synchronize": torch.cuda.synchronize}

    def rand(*size, dtype=None, device=None, **kw):
        t = real["rand"](*size, dtype=dtype, **kw)
        registry.add(t)
        return t

    def tensor(data, *args, device=None, **kw):
        return real["tensor"](data, *args, **kw)

    def empty(*size, device=None, pin_memory=False, **kw):
        return real["empty"](*size, **kw)

    sys.modules.update(fake)
    sys.modules.pop("utils", None)
    torch.rand, torch.tensor, torch.empty = rand, tensor, empty
    torch.Tensor.cuda = lambda self, *a, **k: self
    torch.cuda.Event = _Event
    torch.cuda.synchronize = lambda *a, **k: None
    sys.path.insert(0, REFERENCE_TESTS)
    try:
        yield
    finally:
        sys.path.remove(REFERENCE_TESTS)
        torch.rand, torch.tensor, torch.empty = real["rand"], real["tensor"], real["empty"]
        torch.Tensor.cuda = real["cuda"]
        torch.cuda.Event = real["Event"]
        torch.cuda.synchronize = real["synchronize"]
        for k, v in saved_modules.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def _load_reference_module():
    spec = importlib.util.spec_from_file_location("_reference_test_mem_kernels", TEST_FILE)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_case(test: str, num_tokens: int, token_major: bool | None = None) -> dict:
    """Runs one parametrisation of a reference test on the oracle (its own
    assertions raise on a mismatch) and returns the digests described in the
    module docstring."""
    registry = TensorRegistry()
    RecordingAllocator.allocations = []
    seed = SEEDS[test]
    block_size = 64 if test == "test_multi_layer_kernel_use_mla" else 16
    with reference_environment(registry):
        mod = _load_reference_module()
        fn = getattr(mod, test)
        # the slots the test will draw: random.sample is its only use of `random`
        random.seed(seed)
        slots = random.sample(range(0, 1000 * block_size), num_tokens)
        random.seed(seed)
        torch.manual_seed(seed)
        if token_major is None:
            fn(num_tokens)
        else:
            fn(num_tokens, token_major)
    final = hashlib.sha256()
    for t in registry.created:
        final.update(np.ascontiguousarray(bits(t)))
    out = {
        "test": test,
        "num_tokens": num_tokens,
        "seed": seed,
        "inputs_sha256": registry.input_hash.hexdigest(),
        "num_created": len(registry.created),
        "slots_sha256": hashlib.sha256(np.asarray(slots, dtype=np.int64).tobytes()).hexdigest(),
        "objects_sha256": [sha256_of(o.tensor) for o in RecordingAllocator.allocations],
        "created_after_sha256": final.hexdigest(),
        "buffers_after_sha256": [sha256_of(b) for b in registry.c_ops.lmc_buffers],
    }
    if token_major is not None:
        out["token_major"] = token_major
    RecordingAllocator.allocations = []
    return out


def all_cases():
    for test, params in TESTS.items():
        for n in NUM_TOKENS:
            if "token_major" in params:
                for tm in (True, False):
                    yield test, n, tm
            else:
                yield test, n, None
