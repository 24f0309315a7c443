"""RoPE + contiguous K-cache append reference (semantics of
triton_agent/ops/rope_kv_append/reference.py:10-59): rotate k_new [B,H,T_new,D]
with cos/sin [T_new, D] (NeoX halves, fp32), then store token t of sequence b
at row slot_mapping[b, t] of k_cache[b]; slots outside [0, L) skipped.
"""

import torch


def rope_kv_append(k_new, cos, sin, k_cache, slot_mapping):
    h = k_new.shape[-1] // 2
    kf = k_new.float()
    c, s = cos[..., :h].float(), sin[..., :h].float()
    rot = torch.cat((kf[..., :h] * c - kf[..., h:] * s, kf[..., h:] * c + kf[..., :h] * s), dim=-1).to(k_new.dtype)
    B, H, L, D = k_cache.shape
    out = k_cache.clone()
    slots = slot_mapping.reshape(B, -1)
    for t in range(rot.shape[2]):
        st = slots[:, t]
        ok = (st >= 0) & (st < L)
        b_idx = torch.nonzero(ok).flatten()
        if b_idx.numel():
            out[b_idx, :, st[b_idx]] = rot[b_idx, :, t]
    return out


def generate_test_inputs(B: int = 4, H: int = 32, L: int = 4096, T_new: int = 1, D: int = 128,
                         dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    k_new = torch.randn(B, H, T_new, D, generator=g, device=device).to(dtype)
    cos = torch.randn(T_new, D, generator=g, device=device).to(dtype)
    sin = torch.randn(T_new, D, generator=g, device=device).to(dtype)
    k_cache = torch.randn(B, H, L, D, generator=g, device=device).to(dtype)
    slot_mapping = torch.stack([torch.randperm(L, generator=g, device=device)[:T_new] for _ in range(B)])
    return k_new, cos, sin, k_cache, slot_mapping
