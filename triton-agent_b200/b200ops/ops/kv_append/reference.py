"""Contiguous KV-cache append reference (semantics of triton_agent/ops/kv_append/reference.py:10-52).

For every (b, t) in order, row slot = slot_mapping[b, t] of k_cache[b, :, :, :]
and v_cache[b, :, :, :] receives k_new[b, :, t] and v_new[b, :, t]; slots
outside [0, L) are skipped and a later (b, t) overwrites an earlier one.
Returns new tensors; the CUDA variant writes the caches in place.
"""

import torch


def kv_append(k_cache, v_cache, k_new, v_new, slot_mapping):
    B, H, L, D = k_cache.shape
    k_out, v_out = k_cache.clone(), v_cache.clone()
    T_new = k_new.shape[2]
    slots = slot_mapping.reshape(B, T_new)
    for t in range(T_new):  # t order: later tokens overwrite earlier ones
        s = slots[:, t]
        ok = (s >= 0) & (s < L)
        b_idx = torch.nonzero(ok).flatten()
        if b_idx.numel():
            k_out[b_idx, :, s[b_idx]] = k_new[b_idx, :, t]
            v_out[b_idx, :, s[b_idx]] = v_new[b_idx, :, t]
    return k_out, v_out


def generate_test_inputs(B: int = 4, H: int = 32, L: int = 4096, T_new: int = 1, D: int = 128,
                         dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    k_cache = torch.randn(B, H, L, D, generator=g, device=device).to(dtype)
    v_cache = torch.randn(B, H, L, D, generator=g, device=device).to(dtype)
    k_new = torch.randn(B, H, T_new, D, generator=g, device=device).to(dtype)
    v_new = torch.randn(B, H, T_new, D, generator=g, device=device).to(dtype)
    # distinct slots per sequence: the result does not depend on write order
    slot_mapping = torch.stack([torch.randperm(L, generator=g, device=device)[:T_new] for _ in range(B)])
    return k_cache, v_cache, k_new, v_new, slot_mapping
