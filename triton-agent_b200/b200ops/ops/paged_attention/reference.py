"""Paged-attention decode reference (semantics of
triton_agent/ops/paged_attention/reference.py:10-68).

For sequence b: take the first ceil(ctx/block_size) entries of its block
table, drop ids outside [0, num_blocks), concatenate those blocks' tokens and
keep the first ctx; out = softmax(q[b] K^T / sqrt(D)) V in fp32.  The
reference writes q[b:b+1] into a 2-D einsum and fails; here the query row is
q[b].  Query head h reads kv head h // (H / H_kv) (grouped-query attention;
with H == H_kv this is the reference).  A sequence with no tokens gives zeros.
"""

import math

import torch


def paged_attention(q, k_cache, v_cache, block_table, context_len):
    B, H, D = q.shape
    nb, bs, Hkv, _ = k_cache.shape
    group = H // Hkv
    out = torch.zeros(B, H, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        ctx = int(context_len[b])
        if ctx <= 0:
            continue
        ids = block_table[b, : (ctx + bs - 1) // bs].long()
        ids = ids[(ids >= 0) & (ids < nb)]
        if ids.numel() == 0:
            continue
        keys = k_cache[ids].reshape(-1, Hkv, D)[:ctx].float().transpose(0, 1).repeat_interleave(group, 0)
        vals = v_cache[ids].reshape(-1, Hkv, D)[:ctx].float().transpose(0, 1).repeat_interleave(group, 0)
        w = torch.softmax(torch.einsum("hd,hld->hl", q[b].float(), keys) / math.sqrt(D), dim=-1)
        out[b] = torch.einsum("hl,hld->hd", w, vals)
    return out.to(q.dtype)


def generate_test_inputs(B: int = 8, H: int = 32, D: int = 128, num_blocks: int = 256, block_size: int = 16,
                         max_blocks: int = 32, ctx_len: int = 512, H_kv: int = 0,
                         dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    Hkv = H_kv or H
    q = torch.randn(B, H, D, generator=g, device=device).to(dtype)
    k_cache = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device=device).to(dtype)
    v_cache = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device=device).to(dtype)
    block_table = torch.randint(0, num_blocks, (B, max_blocks), generator=g, device=device)
    context_len = torch.full((B,), ctx_len, dtype=torch.long, device=device)
    return q, k_cache, v_cache, block_table, context_len
