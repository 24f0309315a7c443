"""Scaled dot-product attention reference (semantics of
triton_agent/ops/flash_attn_like/reference.py:7-41): softmax(q k^T / sqrt(D)
[+ causal mask: key s > query t removed, T == S]) v, fp32 softmax, chunked
over query rows so the score matrix never exceeds 1024 rows.
"""

import math

import torch


def flash_attn_like(q, k, v, causal: bool = False):
    B, H, T, D = q.shape
    S = k.shape[2]
    out = torch.empty(B, H, T, D, dtype=torch.float32, device=q.device)
    kf, vf = k.float(), v.float()
    for t0 in range(0, T, 1024):
        t1 = min(T, t0 + 1024)
        sc = torch.einsum("bhtd,bhsd->bhts", q[:, :, t0:t1].float(), kf) / math.sqrt(D)
        if causal:
            mask = torch.arange(S, device=q.device)[None, :] > torch.arange(t0, t1, device=q.device)[:, None]
            sc = sc.masked_fill(mask, float("-inf"))
        out[:, :, t0:t1] = torch.einsum("bhts,bhsd->bhtd", torch.softmax(sc, dim=-1), vf)
    return out.to(q.dtype)


def generate_test_inputs(B: int = 4, H: int = 32, T: int = 2048, S: int = 2048, D: int = 64,
                         dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, H, T, D, generator=g, device=device).to(dtype)
    k = torch.randn(B, H, S, D, generator=g, device=device).to(dtype)
    v = torch.randn(B, H, S, D, generator=g, device=device).to(dtype)
    return q, k, v
