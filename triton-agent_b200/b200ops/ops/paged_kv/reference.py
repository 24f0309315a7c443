"""Paged KV-cache append reference (semantics of triton_agent/ops/paged_kv/reference.py:6-40).

Global slot s maps to block s // block_size, offset s % block_size; rows whose
block is outside [0, num_blocks) are skipped; later (b, t) overwrite earlier
ones.  Returns new tensors; the CUDA variant writes the caches in place.
"""

import torch


def paged_kv(k_cache, v_cache, k_new, v_new, slot_mapping):
    nb, bs, H, D = k_cache.shape
    k_out, v_out = k_cache.clone(), v_cache.clone()
    flat_k = k_new.reshape(-1, H, D)
    flat_v = v_new.reshape(-1, H, D)
    slots = slot_mapping.reshape(-1)
    blk = torch.div(slots, bs, rounding_mode="floor")
    off = slots - blk * bs
    for i in range(slots.numel()):  # sequential: the last writer wins
        if 0 <= int(blk[i]) < nb:
            k_out[blk[i], off[i]] = flat_k[i]
            v_out[blk[i], off[i]] = flat_v[i]
    return k_out, v_out


def generate_test_inputs(B: int = 4, H: int = 32, num_blocks: int = 256, block_size: int = 16, T_new: int = 1,
                         D: int = 128, dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    k_cache = torch.randn(num_blocks, block_size, H, D, generator=g, device=device).to(dtype)
    v_cache = torch.randn(num_blocks, block_size, H, D, generator=g, device=device).to(dtype)
    k_new = torch.randn(B, T_new, H, D, generator=g, device=device).to(dtype)
    v_new = torch.randn(B, T_new, H, D, generator=g, device=device).to(dtype)
    slot_mapping = torch.randperm(num_blocks * block_size, generator=g, device=device)[: B * T_new].reshape(B, T_new)
    return k_cache, v_cache, k_new, v_new, slot_mapping
