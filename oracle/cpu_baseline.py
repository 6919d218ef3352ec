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
import os
import time
from typing import Dict, List

import torch


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class CpuTransfer:
    """Host-resident paged buffers + LMCache objects for one workload spec.

    ``spec`` follows lmcache_b200.workloads.Spec. The number of blocks per
    layer is reduced to ``max_blocks`` (host RAM), keeping every per-chunk
    shape; slots are drawn for the reduced buffer with the same generator.
    """

    def __init__(self, spec, max_blocks: int, seed: int = 0, threads: int | None = None):
        from lmcache_b200 import workloads as wl  # shapes and slot generator only

        self.threads = threads or host_threads()
        torch.set_num_threads(self.threads)
        blocks = min(spec.num_blocks, max_blocks)
        self.spec = dataclasses.replace(spec, num_blocks=blocks)
        self.full_blocks = spec.num_blocks
        s = self.spec
        self.slots = wl.make_slot_mapping(s, seed=seed)
        self.chunks = wl.chunks(self.slots, s.chunk_size)
        self.caches: List[torch.Tensor] = []
        for _ in range(s.num_layers):
            t = torch.empty(s.layer_shape, dtype=torch.bfloat16)
            t.view(torch.int16).random_(-32768, 32767)
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
