"""fp32 reference of rotary_embedding_k_fused (test infrastructure).

The reference op is a stub (csrc/pos_kernels.cpp:7-14); its semantics are
those of the unfused path in lmcache_ascend/v1/blend/positional_encoding.py:
DummyFusedRope (:80-101) undoes the rotary embedding at the old positions
(BasicReverseRope, :20-54: shuffle the pair halves, rotate, shuffle back,
i.e. rotate by the negative angle) and applies it at the new positions. The
rotation itself is vLLM's rotary embedding with a [max_position, rot_dim]
cache laid out [cos | sin]: neox style rotates (x[i], x[i + rot/2]), GPT-J
style rotates (x[2i], x[2i+1]); dims beyond rot_dim pass through.
Everything here runs in float32 on the CPU.
"""

from __future__ import annotations

import torch


def rotate(k: torch.Tensor, positions: torch.Tensor, cos_sin_cache: torch.Tensor,
           is_neox: bool, inverse: bool = False) -> torch.Tensor:
    """k [T, heads, head_size] float32 -> rotated copy (by -angle if inverse)."""
    cache = cos_sin_cache.float()
    rot = cache.shape[1]
    half = rot // 2
    cos = cache[positions.long(), :half][:, None, :]
    sin = cache[positions.long(), half:][:, None, :]
    if inverse:
        sin = -sin
    out = k.clone()
    if is_neox:
        x1, x2 = k[..., :half], k[..., half:rot]
        out[..., :half] = x1 * cos - x2 * sin
        out[..., half:rot] = x2 * cos + x1 * sin
    else:
        x1, x2 = k[..., 0:rot:2], k[..., 1:rot:2]
        out[..., 0:rot:2] = x1 * cos - x2 * sin
        out[..., 1:rot:2] = x2 * cos + x1 * sin
    return out


def rotary_embedding_k_fused(old_positions, new_positions, key, head_size, cos_sin_cache,
                             is_neox) -> torch.Tensor:
    """Returns the re-rotated key (float32, [T, heads, head_size])."""
    k = key.detach().cpu().float().reshape(key.shape[0], -1, head_size)
    k = rotate(k, old_positions.cpu(), cos_sin_cache.cpu(), is_neox, inverse=True)
    return rotate(k, new_positions.cpu(), cos_sin_cache.cpu(), is_neox)
