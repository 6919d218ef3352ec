"""Timed CPU baseline of the transfer path (test/benchmark infrastructure).

The reference's own transfer kernels are AscendC code that is absent from its
tree and cannot run here; its tests check them against torch indexing
(tests/v1/test_mem_kernels.py:84-101). This module times that
reference-semantics CPU path: ``index_select`` from the flattened paged
buffer ``[kv * page_buffer_size, H]`` into the LMCache object for a store,
``index_copy_`` back for a retrieve, skipped (-1) slots masked out, on host
tensors with every available host thread.

Only the benchmark's CPU-baseline / reference legs use it.
"""

from __future__ import annotations

import dataclasses
import importlib.util
import os
import sys
import time
from typing import Dict, List

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKLOADS_PY = os.path.join(ROOT, "lmcache-ascend_b200", "lmcache_b200", "workloads.py")


def load_workloads():
    """The workload definitions (shapes and seeded slot generator), loaded
    from their file without importing the lmcache_b200 package: the package's
    __init__ loads the CUDA extension, and the CPU legs must map none of the
    product's native libraries."""
    name = "_lmcb_workload_specs"
    mod = sys.modules.get(name)
    if mod is None:
        spec = importlib.util.spec_from_file_location(name, WORKLOADS_PY)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod  # dataclasses resolve annotations through sys.modules
        spec.loader.exec_module(mod)
    return mod


def mapped_product_libraries() -> list[str]:
    """Shared objects of the lmcache_b200 package mapped into this process."""
    found = set()
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                path = line.rstrip("\n").split(None, 5)[-1]
                if "lmcache_b200" in path and path.endswith(".so"):
                    found.add(os.path.relpath(path, ROOT))
    except OSError:
        pass
    return sorted(found)


def available_host_bytes() -> int:
    try:
        import psutil

        return int(psutil.virtual_memory().available)
    except Exception:  # pragma: no cover
        return int(os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE"))


def fitting_blocks(spec, max_blocks: int) -> int:
    """Blocks per layer for the host-resident buffers: ``max_blocks`` when
    positive, else the full count when the paged buffers and objects take at
    most half of the available host memory, else the largest power of two
    that does (never fewer than the sequence needs)."""
    if max_blocks > 0:
        return min(spec.num_blocks, max_blocks)
    budget = available_host_bytes() // 2
    per_block = spec.num_layers * spec.kv * spec.block_size * spec.hidden * 2
    objects = spec.num_layers * spec.kv * spec.num_tokens * spec.hidden * 2
    if spec.num_blocks * per_block + objects <= budget:
        return spec.num_blocks
    need = -(-spec.num_tokens // spec.block_size)
    blocks = 1 << max(0, ((budget - objects) // per_block).bit_length() - 1)
    return max(min(blocks, spec.num_blocks), need)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class CpuTransfer:
    """Host-resident paged buffers + LMCache objects for one workload spec.

    ``spec`` follows lmcache_b200/workloads.py's Spec. The number of blocks
    per layer is ``fitting_blocks(spec, max_blocks)``: the full workload when
    host RAM allows, else reduced, keeping every per-chunk shape; slots are
    then drawn for the reduced buffer with the same generator. With the full
    count the slots are exactly the GPU benchmark's.
    """

    def __init__(self, spec, max_blocks: int = 0, seed: int = 0, threads: int | None = None):
        wl = load_workloads()

        self.threads = threads or host_threads()
        torch.set_num_threads(self.threads)
        blocks = fitting_blocks(spec, max_blocks)
        self.spec = dataclasses.replace(spec, num_blocks=blocks)
        self.full_blocks = spec.num_blocks
        s = self.spec
        self.slots = wl.make_slot_mapping(s, seed=seed)
        self.chunks = wl.chunks(self.slots, s.chunk_size)
        # Seeded random bit patterns: one 64 MiB block, tiled into every layer
        # with a per-layer XOR (the copy rate does not depend on the values,
        # and drawing tens of GiB of random numbers would take a minute).
        g = torch.Generator().manual_seed(seed)
        pattern = torch.empty(32 << 20, dtype=torch.int16)
        pattern.random_(-32768, 32767, generator=g)
        self.caches: List[torch.Tensor] = []
        for layer in range(s.num_layers):
            t = torch.empty(s.layer_shape, dtype=torch.bfloat16)
            flat = t.view(-1).view(torch.int16)
            for i in range(0, flat.numel(), pattern.numel()):
                n = min(pattern.numel(), flat.numel() - i)
                torch.bitwise_xor(pattern[:n], layer, out=flat[i:i + n])
            self.caches.append(t)
        self.flat = [t.view(-1, s.hidden) for t in self.caches]
        self.objs = [torch.empty(s.memobj_shape(len(c)), dtype=torch.bfloat16) for c in self.chunks]
        # Per chunk: valid token positions and per-kv flat rows.
        self.index: List[Dict] = []
        pbs = 0 if s.use_mla else s.page_buffer_size
        for c in self.chunks:
            t_valid = torch.nonzero(c >= 0).flatten()
            slots = c[t_valid]
            rows = [k * pbs + slots for k in range(s.kv)]
            self.index.append({"all": len(t_valid) == len(c), "t": t_valid, "rows": rows})

    def store_chunk(self, ci: int) -> None:
        s, ix, obj = self.spec, self.index[ci], self.objs[ci]
        for layer in range(s.num_layers):
            src = self.flat[layer]
            for k in range(s.kv):
                if ix["all"]:
                    torch.index_select(src, 0, ix["rows"][k], out=obj[k, layer])
                else:
                    obj[k, layer].index_copy_(0, ix["t"], src.index_select(0, ix["rows"][k]))

    def retrieve_chunk(self, ci: int) -> None:
        s, ix, obj = self.spec, self.index[ci], self.objs[ci]
        for layer in range(s.num_layers):
            dst = self.flat[layer]
            for k in range(s.kv):
                vals = obj[k, layer] if ix["all"] else obj[k, layer].index_select(0, ix["t"])
                dst.index_copy_(0, ix["rows"][k], vals)

    def chunk_payload(self, ci: int) -> int:
        s = self.spec
        return len(self.index[ci]["t"]) * s.num_layers * s.kv * s.hidden * 2

    def run_step(self, n_chunks: int) -> tuple[int, float]:
        """Stores then retrieves the first ``n_chunks`` chunks; returns
        (payload bytes moved, seconds)."""
        t0 = time.perf_counter()
        for ci in range(n_chunks):
            self.store_chunk(ci)
        for ci in range(n_chunks):
            self.retrieve_chunk(ci)
        dt = time.perf_counter() - t0
        return 2 * sum(self.chunk_payload(ci) for ci in range(n_chunks)), dt

    def measure(self, budget_s: float = 15.0) -> dict:
        """Times whole steps (all chunks, both directions) within about
        ``budget_s`` seconds, after one warm-up chunk; returns GB/s and the
        sample description."""
        self.run_step(1)
        n_chunks = len(self.chunks)
        # Size the sample: one full step if it fits in the budget, else fewer chunks.
        b, dt = self.run_step(1)
        per_chunk = max(dt, 1e-6)
        n = max(1, min(n_chunks, int(budget_s / 2 / per_chunk)))
        total_b, total_t, steps = 0, 0.0, 0
        while total_t < budget_s / 2 or steps == 0:
            b, dt = self.run_step(n)
            total_b += b
            total_t += dt
            steps += 1
        return {
            "gbps": total_b / total_t / 1e9,
            "chunks_per_step": n,
            "steps": steps,
            "seconds": total_t,
            "bytes": total_b,
            "threads": self.threads,
            "blocks_per_layer": self.spec.num_blocks,
            "full_blocks_per_layer": self.full_blocks,
        }
