"""Decode-step RoPE(q, k) + paged K/V append reference.

Composes triton_agent/ops/rope/reference.py:17-25 (NeoX rotation, here with
cos/sin rows selected by each token's position), rope_kv_append/reference.py:
33-35 (k rotated before it is stored) and paged_kv/reference.py:18-25 (slot ->
block, offset; invalid slots skipped).  Rotation in fp32 with every product
and sum rounded separately, then one rounding to the storage dtype.
Returns (q_out, k_cache', v_cache') as new tensors.
"""

import math

import torch


def _rot(x, c, s):
    h = x.shape[-1] // 2
    xf = x.float()
    return torch.cat((xf[..., :h] * c - xf[..., h:] * s, xf[..., h:] * c + xf[..., :h] * s), dim=-1).to(x.dtype)


def rope_kv_append_paged(q, k, v, positions, cos, sin, slot_mapping, k_cache, v_cache):
    D = k.shape[-1]
    h = D // 2
    c = cos[positions.long(), :h].float().unsqueeze(1)
    s = sin[positions.long(), :h].float().unsqueeze(1)
    q_out = _rot(q, c, s)
    k_rot = _rot(k, c, s)
    nb, bs = k_cache.shape[:2]
    k_out, v_out = k_cache.clone(), v_cache.clone()
    for t in range(k.shape[0]):
        slot = int(slot_mapping[t])
        if 0 <= slot < nb * bs:
            k_out[slot // bs, slot % bs] = k_rot[t]
            v_out[slot // bs, slot % bs] = v[t]
    return q_out, k_out, v_out


def generate_test_inputs(T: int = 64, Hq: int = 32, Hkv: int = 8, D: int = 128, num_blocks: int = 65536,
                         block_size: int = 16, max_pos: int = 4096, theta: float = 1e4,
                         dtype: torch.dtype = torch.bfloat16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(T, Hq, D, generator=g, device=device).to(dtype)
    k = torch.randn(T, Hkv, D, generator=g, device=device).to(dtype)
    v = torch.randn(T, Hkv, D, generator=g, device=device).to(dtype)
    positions = torch.randint(0, max_pos, (T,), generator=g, device=device)
    j = torch.arange(0, D, 2, dtype=torch.float32, device=device)
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32, device=device), 1.0 / theta ** (j / D))
    cos = torch.cat((ang.cos(), ang.cos()), dim=-1).contiguous()
    sin = torch.cat((ang.sin(), ang.sin()), dim=-1).contiguous()
    slots = torch.randperm(num_blocks * block_size, generator=g, device=device)[:T].contiguous()
    k_cache = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device=device).to(dtype)
    v_cache = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device=device).to(dtype)
    return q, k, v, positions, cos, sin, slots, k_cache, v_cache
