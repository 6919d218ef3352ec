"""Seeded synthetic KV-transfer workloads with the shapes of the reference's
deployment targets, shared by the benchmark and the tests.

Each workload is a paged KV cache (one tensor per layer, vLLM layout), a token
sequence split into chunks with a slot mapping per chunk, and the shape of the
LMCache object ([kv, L, chunk, H]) each chunk is stored to. Values are drawn
from a seeded generator on the target device; slot mappings from a seeded CPU
generator, so every run sees the same slots.

  c1  CPU-sized: 4 layers, [2, 64 blocks, 16, 8, 128] bf16 ~N(0,1), one
      256-token chunk of distinct random slots with 16 set to -1.
  c2  Llama-3-8B: 32 layers, 8 x 128 heads, block_size 16, 8192 blocks per
      layer; 8192 tokens in 32 chunks of 256, each chunk 16 random distinct
      blocks of 16 consecutive slots.
  c3  Qwen3-32B: 64 layers, 8 x 128, block_size 128, 2048 blocks per layer;
      8192 tokens = 64 random distinct blocks x 128 slots, 32 chunks of 256.
  c4  DeepSeek-V3 MLA: 61 layers, one [4096 blocks, 64, 576] buffer per layer,
      values ~N(0, 0.5); 4096 random distinct slots in 16 chunks of 256.
  c5  Llama-3-70B TP=8 shard: 80 layers, 1 x 128, block_size 16, 4096 blocks
      per layer; 16384 tokens = 1024 random distinct blocks x 16, 64 chunks.
"""

from __future__ import annotations

import dataclasses
from typing import List

import torch


@dataclasses.dataclass
class Spec:
    name: str
    description: str
    num_layers: int
    num_blocks: int
    block_size: int
    num_heads: int
    head_size: int
    num_tokens: int
    chunk_size: int
    use_mla: bool = False
    std: float = 1.0
    run: int = 0          # consecutive slots per block run (0: random slots)
    neg_slots: int = 0    # slots set to -1 (c1 only)

    @property
    def kv(self) -> int:
        return 1 if self.use_mla else 2

    @property
    def hidden(self) -> int:
        return self.num_heads * self.head_size

    @property
    def page_buffer_size(self) -> int:
        return self.num_blocks * self.block_size

    @property
    def layer_shape(self) -> list:
        if self.use_mla:
            return [self.num_blocks, self.block_size, self.head_size]
        return [2, self.num_blocks, self.block_size, self.num_heads, self.head_size]

    def memobj_shape(self, tokens: int) -> list:
        return [self.kv, self.num_layers, tokens, self.hidden]

    def paged_bytes(self, elem: int = 2) -> int:
        return self.num_layers * self.kv * self.page_buffer_size * self.hidden * elem


SPECS = {
    "c1": Spec("c1", "CPU-sized 4-layer, 256 tokens with 16 skipped slots",
               4, 64, 16, 8, 128, 256, 256, neg_slots=16),
    "c2": Spec("c2", "Llama-3-8B KV, block_size 16, 8192 blocks/layer, 8192 tokens",
               32, 8192, 16, 8, 128, 8192, 256, run=16),
    "c3": Spec("c3", "Qwen3-32B KV, block_size 128, 2048 blocks/layer, 8192 tokens",
               64, 2048, 128, 8, 128, 8192, 256, run=128),
    "c4": Spec("c4", "DeepSeek-V3 MLA latent 576, block_size 64, 4096 blocks/layer, 4096 tokens",
               61, 4096, 64, 1, 576, 4096, 256, use_mla=True, std=0.5),
    "c5": Spec("c5", "Llama-3-70B TP8 shard (1 KV head), block_size 16, 4096 blocks/layer",
               80, 4096, 16, 1, 128, 16384, 256, run=16),
}


def make_slot_mapping(spec: Spec, seed: int = 0) -> torch.Tensor:
    """Seeded int64 slot mapping of spec.num_tokens tokens (CPU)."""
    g = torch.Generator().manual_seed(seed)
    if spec.run > 0:
        n_runs = spec.num_tokens // spec.run
        blocks_per_run = spec.run // spec.block_size if spec.run >= spec.block_size else 1
        if spec.run >= spec.block_size:
            # runs of whole blocks: pick n_runs * blocks_per_run distinct blocks
            blocks = torch.randperm(spec.num_blocks, generator=g)[: n_runs * blocks_per_run]
            offs = torch.arange(spec.block_size)
            slots = (blocks[:, None] * spec.block_size + offs[None, :]).reshape(-1)
        else:
            starts = torch.randperm(spec.num_blocks, generator=g)[:n_runs] * spec.block_size
            slots = (starts[:, None] + torch.arange(spec.run)[None, :]).reshape(-1)
        return slots[: spec.num_tokens].to(torch.int64)
    slots = torch.randperm(spec.page_buffer_size, generator=g)[: spec.num_tokens].to(torch.int64)
    if spec.neg_slots:
        pos = torch.randperm(spec.num_tokens, generator=g)[: spec.neg_slots]
        slots[pos] = -1
    return slots


def make_kv_caches(spec: Spec, device, seed: int = 0, dtype=torch.bfloat16) -> List[torch.Tensor]:
    """One paged buffer per layer, values ~N(0, spec.std^2) from a seeded generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    caches = []
    for _ in range(spec.num_layers):
        t = torch.empty(spec.layer_shape, dtype=dtype, device=device)
        t.normal_(0.0, spec.std, generator=g)
        caches.append(t)
    return caches


def pointer_tensor(caches: List[torch.Tensor], device) -> torch.Tensor:
    """Device int64 array of per-layer base addresses, as the connector builds it
    (lmcache_ascend/v1/npu_connector.py:24-33)."""
    ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64)
    return ptrs.to(device)


def chunks(slots: torch.Tensor, chunk_size: int) -> List[torch.Tensor]:
    return list(torch.split(slots, chunk_size))


def payload_bytes(spec: Spec, slots: torch.Tensor, elem: int = 2) -> int:
    """KV payload moved by one direction over `slots` (skipped slots excluded)."""
    n_valid = int((slots >= 0).sum())
    return n_valid * spec.num_layers * spec.kv * spec.hidden * elem
