"""Symmetric INT8 matmul reference (semantics of
triton_agent/ops/quant_matmul/reference.py:6-37).

a [..., M, K] is quantised per row and b [K, N] per column:
scale = max|x| / 127 (zero -> 1e-6), code = clamp(round(x / scale), -127, 127);
c = (codes_a @ codes_b) * scale_a * scale_b in fp32.  The product of codes is
accumulated exactly in integers (the reference's fp32 matmul of codes is
exact only while partial sums stay below 2^24).
"""

import torch


def _quant(x, dim):
    scale = x.abs().amax(dim=dim, keepdim=True) / 127.0
    scale[scale == 0] = 1e-6
    return (x / scale).round().clamp(-127, 127).to(torch.int8), scale


def quant_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    qa, sa = _quant(a, -1)
    qb, sb = _quant(b, 0)
    acc = torch.matmul(qa.cpu().to(torch.int64), qb.cpu().to(torch.int64)).to(a.device)
    return acc.float() * sa * sb


def generate_test_inputs(B: int = 8, M: int = 256, K: int = 4096, N: int = 4096,
                         dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn(B, M, K, generator=g, device=device).to(dtype)
    b = torch.randn(K, N, generator=g, device=device).to(dtype)
    return a, b
