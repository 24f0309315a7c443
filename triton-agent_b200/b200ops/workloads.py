"""Seeded synthetic inputs at the benchmark shapes of the operator hot path.

Shapes and distributions (seed 0 unless given):
  rmsnorm         x f32 [8, 2048, 4096] ~ N(0,1); weight [4096] ~ N(1, 0.1); eps 1e-6
  decode append   64 tokens; q [64,32,128], k/v [64,8,128] bf16 ~ N(0,1);
                  positions ~ U{0..4095}; RoPE theta 1e4; paged caches
                  [65536, 16, 8, 128] bf16; slot_mapping = 64 distinct random slots
  paged decode    q [64,32,128] bf16; same caches ~ N(0,1); context_len ~ U{512..8192};
                  block_table rows = consecutive slices of a random permutation of
                  the 65536 physical blocks; scale 1/sqrt(128)
  int8 GEMM       A [M,4096], W [N,4096] int8 ~ U{-127..127}; scales f32 ~ U(0.001, 0.02);
                  M in {16, 4096}, N in {4096, 14336}
  causal prefill  q, k, v bf16 [4, 32, 4096, 128] ~ N(0,1)
Everything is generated on the target device with a torch.Generator, so a
4 GiB cache costs milliseconds, not a host-side fill and copy.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def rope_tables(max_pos: int, D: int, theta: float = 1e4, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin tables [max_pos, D]: angle(p, j) = p * theta^(-2j/D) for
    j < D/2, second half repeating the first (NeoX layout), indexed by
    position like a serving engine's cos/sin cache."""
    j = torch.arange(0, D, 2, dtype=torch.float32)
    inv_freq = 1.0 / (theta ** (j / D))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv_freq)
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1).contiguous().to(device)
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1).contiguous().to(device)
    return cos, sin


def rmsnorm_inputs(B=8, T=2048, D=4096, dtype=torch.float32, device="cuda", seed=0):
    g = _gen(device, seed)
    x = torch.randn(B, T, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    w = (1.0 + 0.1 * torch.randn(D, generator=g, device=device, dtype=torch.float32)).to(dtype)
    return x, w


@dataclass
class PagedCache:
    k_cache: torch.Tensor  # [num_blocks, block_size, Hkv, D]
    v_cache: torch.Tensor

    @property
    def num_blocks(self) -> int:
        return self.k_cache.shape[0]

    @property
    def block_size(self) -> int:
        return self.k_cache.shape[1]


def paged_cache(num_blocks=65536, block_size=16, Hkv=8, D=128, dtype=torch.bfloat16, device="cuda", seed=0):
    g = _gen(device, seed + 1000)
    kc = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device=device, dtype=dtype)
    vc = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device=device, dtype=dtype)
    return PagedCache(kc, vc)


def decode_append_inputs(cache: PagedCache, n_tok=64, Hq=32, max_pos=4096, theta=1e4, device="cuda", seed=0):
    """Inputs of one decode-step RoPE + paged append."""
    Hkv, D = cache.k_cache.shape[2:]
    g = _gen(device, seed + 2000)
    dt = cache.k_cache.dtype
    q = torch.randn(n_tok, Hq, D, generator=g, device=device, dtype=torch.float32).to(dt)
    k = torch.randn(n_tok, Hkv, D, generator=g, device=device, dtype=torch.float32).to(dt)
    v = torch.randn(n_tok, Hkv, D, generator=g, device=device, dtype=torch.float32).to(dt)
    positions = torch.randint(0, max_pos, (n_tok,), generator=g, device=device, dtype=torch.int64)
    slots = torch.randperm(cache.num_blocks * cache.block_size, generator=g, device=device)[:n_tok].contiguous()
    cos, sin = rope_tables(max_pos, D, theta, device)
    return dict(q=q, k=k, v=v, positions=positions, cos=cos, sin=sin, slot_mapping=slots)


def context_lengths(n_seq: int, ctx_lo=512, ctx_hi=8192, seed=0) -> torch.Tensor:
    """Context lengths ~ U{ctx_lo..ctx_hi} of a global batch of sequences
    (host int64), drawn once so that every rank shards the same batch."""
    g = torch.Generator().manual_seed(seed + 6000)
    return torch.randint(ctx_lo, ctx_hi + 1, (n_seq,), generator=g, dtype=torch.int64)


def decode_attention_inputs(cache: PagedCache, B=64, Hq=32, ctx_lo=512, ctx_hi=8192, device="cuda", seed=0,
                            index_dtype=torch.int32, context_len: torch.Tensor | None = None):
    """Inputs of one paged-attention decode step over `cache`.  With
    `context_len` (this rank's share of a global batch) B is its length and
    the lengths are used as given."""
    Hkv, D = cache.k_cache.shape[2:]
    bs = cache.block_size
    g = _gen(device, seed + 3000)
    dt = cache.k_cache.dtype
    if context_len is not None:
        B = int(context_len.numel())
    q = torch.randn(B, Hq, D, generator=g, device=device, dtype=torch.float32).to(dt)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (B,), generator=g, device=device, dtype=torch.int64)
    if context_len is not None:
        ctx = context_len.to(device=device, dtype=torch.int64)
    max_blocks = (ctx_hi + bs - 1) // bs
    if B * max_blocks > cache.num_blocks:
        raise ValueError("cache too small for disjoint block tables")
    perm = torch.randperm(cache.num_blocks, generator=g, device=device)
    table = perm[: B * max_blocks].reshape(B, max_blocks).to(index_dtype).contiguous()
    return dict(q=q, block_table=table, context_len=ctx.to(index_dtype), scale=1.0 / math.sqrt(D))


def decode_bytes(context_len: torch.Tensor, Hq: int, Hkv: int, D: int, block_size: int, elem: int = 2,
                 index_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one paged decode launch: every surviving K and
    V row once, q and out once, the used block-table entries and ctx once."""
    ctx = context_len.detach().to("cpu", torch.int64)
    tok = int(ctx.clamp(min=0).sum())
    blocks = int(((ctx.clamp(min=0) + block_size - 1) // block_size).sum())
    B = ctx.numel()
    return tok * Hkv * D * elem * 2 + 2 * B * Hq * D * elem + blocks * index_bytes + B * index_bytes


def append_bytes(n_tok: int, Hq: int, Hkv: int, D: int, elem: int = 2) -> int:
    """Algorithmic bytes of the decode-step append: read q,k,v, write q_out and
    the k,v cache rows, read positions and slots, read cos/sin rows."""
    rows = n_tok * (Hq + 2 * Hkv) * D * elem
    return 2 * rows + 2 * n_tok * 8 + 2 * n_tok * D * 4


def int8_gemm_inputs(M, N, K, device="cuda", seed=0):
    g = _gen(device, seed + 4000)
    A = torch.randint(-127, 128, (M, K), generator=g, device=device, dtype=torch.int8)
    W = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int8)
    sA = torch.empty(M, device=device, dtype=torch.float32).uniform_(0.001, 0.02, generator=g)
    sW = torch.empty(N, device=device, dtype=torch.float32).uniform_(0.001, 0.02, generator=g)
    return A, W, sA, sW


def flash_inputs(B=4, H=32, T=4096, D=128, dtype=torch.bfloat16, device="cuda", seed=0):
    g = _gen(device, seed + 5000)
    q = torch.randn(B, H, T, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    k = torch.randn(B, H, T, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    v = torch.randn(B, H, T, D, generator=g, device=device, dtype=torch.float32).to(dtype)
    return q, k, v


def causal_flops(B, H, T, D) -> int:
    """QK^T and PV FLOPs of causal attention with the diagonal included."""
    return 4 * B * H * D * (T * (T + 1) // 2)
