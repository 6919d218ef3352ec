"""GPU tests of rotary_embedding_k_fused against the fp32 reference of the
unfused path (undo the rotary embedding at the old positions, apply it at the
new ones; lmcache_ascend/v1/blend/positional_encoding.py:80-101)."""

import math

import pytest
import torch

from lmcache_b200 import abi, c_ops
from oracle import rotary as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"

# One rounding of the fp32 result to the key's type: half an ulp, relative.
RTOL = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11, torch.float32: 1e-5}


def cos_sin_cache(max_pos, rot, base=10000.0, dtype=torch.float32):
    inv = 1.0 / (base ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    t = torch.arange(max_pos, dtype=torch.float64)
    freqs = torch.outer(t, inv)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1).to(dtype)


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("key_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("cache_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("pos_dtype", [torch.int64, torch.int32])
def test_matches_fp32_reference(is_neox, key_dtype, cache_dtype, pos_dtype):
    g = torch.Generator().manual_seed(7)
    T, heads, hd, max_pos = 500, 8, 128, 4096
    key = torch.randn(T, heads * hd, generator=g).to(key_dtype).to(DEV)
    old = torch.randint(0, max_pos, (T,), generator=g).to(pos_dtype).to(DEV)
    new = torch.randint(0, max_pos, (T,), generator=g).to(pos_dtype).to(DEV)
    cache = cos_sin_cache(max_pos, hd, dtype=cache_dtype).to(DEV)
    want = ref.rotary_embedding_k_fused(old, new, key, hd, cache, is_neox)
    k = key.view(T, -1, hd)  # as FusedRope passes it (positional_encoding.py:65)
    c_ops.rotary_embedding_k_fused(old, new, k, hd, cache, is_neox)
    got = k.float().cpu()
    # The fp32 reference rounds the cache to cache_dtype first, as the kernel does.
    torch.testing.assert_close(got, want, rtol=RTOL[key_dtype], atol=1e-5)


def test_partial_rotary_dims_and_same_position_identity():
    g = torch.Generator().manual_seed(8)
    T, heads, hd, rot, max_pos = 64, 4, 128, 64, 1024
    key = torch.randn(T, heads, hd, generator=g).to(DEV)
    pos = torch.randint(0, max_pos, (T,), generator=g).to(DEV)
    cache = cos_sin_cache(max_pos, rot).to(DEV)
    k = key.clone()
    c_ops.rotary_embedding_k_fused(pos, pos, k, hd, cache, True)  # identity rotation
    torch.testing.assert_close(k, key, rtol=1e-6, atol=1e-6)
    new = (pos + 37) % max_pos
    c_ops.rotary_embedding_k_fused(pos, new, k, hd, cache, True)
    want = ref.rotary_embedding_k_fused(pos, new, key, hd, cache, True)
    torch.testing.assert_close(k.cpu(), want, rtol=1e-5, atol=1e-5)
    assert torch.equal(k[..., rot:], key[..., rot:])  # dims beyond rot_dim untouched
    # norms are preserved by a rotation
    torch.testing.assert_close(k.norm(dim=-1), key.norm(dim=-1), rtol=1e-5, atol=1e-5)


def test_out_of_range_positions_are_skipped_and_flagged():
    T, heads, hd, max_pos = 8, 2, 64, 100
    key = torch.randn(T, heads, hd, device=DEV)
    old = torch.arange(T, device=DEV)
    new = old + 10
    new[3] = max_pos  # out of range
    new[5] = -1  # out of range
    cache = cos_sin_cache(max_pos, hd).to(DEV)
    k = key.clone()
    c_ops.device_status(torch.cuda.current_device())
    c_ops.rotary_embedding_k_fused(old, new, k, hd, cache, False)
    torch.cuda.synchronize()
    flags = c_ops.device_status(torch.cuda.current_device())
    assert flags & abi.LMCB_DEVICE_FLAG_POSITION_OUT_OF_RANGE
    assert torch.equal(k[3], key[3])
    assert torch.equal(k[5], key[5])
    ok = [t for t in range(T) if t not in (3, 5)]
    want = ref.rotary_embedding_k_fused(old[ok], new[ok], key[ok], hd, cache, False)
    torch.testing.assert_close(k[ok].cpu(), want, rtol=1e-5, atol=1e-5)
    assert math.isfinite(float(k.abs().max()))


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("case", ["rot_dim_6", "misaligned_key"])
def test_scalar_fallback_shapes(is_neox, case):
    """Shapes the two-pair vector kernel cannot take (rot_dim not a multiple
    of 4; a key base off its vector alignment) run the one-pair kernel, with
    the same results."""
    g = torch.Generator().manual_seed(9)
    T, max_pos = 300, 512
    if case == "rot_dim_6":
        heads, hd, rot = 4, 6, 6
        key = torch.randn(T, heads, hd, generator=g).to(torch.bfloat16).to(DEV)
    else:
        heads, hd, rot = 4, 64, 64
        buf = torch.randn(T * heads * hd + 1, generator=g).to(torch.bfloat16).to(DEV)
        key = buf[1:].view(T, heads, hd)  # base 2 bytes past a 4-byte boundary
    old = torch.randint(0, max_pos, (T,), generator=g).to(DEV)
    new = torch.randint(0, max_pos, (T,), generator=g).to(DEV)
    cache = cos_sin_cache(max_pos, rot).to(DEV)
    want = ref.rotary_embedding_k_fused(old, new, key.clone(), hd, cache, is_neox)
    c_ops.rotary_embedding_k_fused(old, new, key, hd, cache, is_neox)
    torch.testing.assert_close(key.float().cpu(), want, rtol=RTOL[torch.bfloat16], atol=1e-5)


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("key_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rot", [128, 64, 24, 12])
def test_the_three_kernels_agree_bit_for_bit(is_neox, key_dtype, rot, monkeypatch):
    """The 16-byte vector kernel (default where aligned), the two-pair kernel
    and the one-pair kernel do the same fp32 arithmetic per pair: forcing each
    (LMCB_ROPE_KERNEL) gives identical bits. rot 24 and 12 leave the 16-byte
    kernel for bf16 neox keys (it needs rot_dim % 16 == 0) and exercise the
    fallbacks under the default choice."""
    g = torch.Generator().manual_seed(10)
    T, heads, hd, max_pos = 777, 4, 128, 2048
    key = torch.randn(T, heads, hd, generator=g).to(key_dtype).to(DEV)
    old = torch.randint(0, max_pos, (T,), generator=g).to(DEV)
    new = torch.randint(0, max_pos, (T,), generator=g).to(DEV)
    cache = cos_sin_cache(max_pos, rot).to(DEV)
    outs = {}
    for kernel in ("default", "v16", "vec2", "pair"):
        if kernel == "default":
            monkeypatch.delenv("LMCB_ROPE_KERNEL", raising=False)
        else:
            monkeypatch.setenv("LMCB_ROPE_KERNEL", kernel)
        k = key.clone()
        c_ops.rotary_embedding_k_fused(old, new, k, hd, cache, is_neox)
        outs[kernel] = k
    for kernel in ("v16", "vec2", "pair"):
        assert torch.equal(outs[kernel], outs["default"]), kernel
    want = ref.rotary_embedding_k_fused(old, new, key, hd, cache, is_neox)
    torch.testing.assert_close(outs["default"].float().cpu(), want, rtol=RTOL[key_dtype],
                               atol=1e-5)
    assert torch.equal(outs["default"][..., rot:], key[..., rot:])
