"""Matmul + bias + GELU reference (semantics of
triton_agent/ops/matmul_epilogue/reference.py:6-18): c = a @ b + bias, then
0.5 c (1 + tanh(0.7978845608028654 (c + 0.044715 c^3))), evaluated in fp32
and returned in a's dtype."""

import torch


def matmul_epilogue(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    c = a.float() @ b.float() + bias.float()
    return (0.5 * c * (1.0 + torch.tanh(0.7978845608028654 * (c + 0.044715 * c.pow(3))))).to(a.dtype)


def generate_test_inputs(B: int = 8, M: int = 256, K: int = 4096, N: int = 4096,
                         dtype: torch.dtype = torch.float16, device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn(B, M, K, generator=g, device=device).to(dtype)
    b = torch.randn(K, N, generator=g, device=device).to(dtype)
    bias = torch.randn(N, generator=g, device=device).to(dtype)
    return a, b, bias


def generate_boundary_inputs(device: str = "cuda"):
    cases = []
    for B, M, K, N in ((1, 1, 64, 64), (4, 128, 2048, 2048)):
        a, b, bias = generate_test_inputs(B, M, K, N, torch.float16, device)
        cases.append((a, b, bias, {}))
    return cases
