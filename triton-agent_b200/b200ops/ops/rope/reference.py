"""NeoX rotate-half RoPE reference (semantics of triton_agent/ops/rope/reference.py:6-40).

With h = D/2: y[..., :h] = x1*c - x2*s and y[..., h:] = x2*c + x1*s where
x1, x2 are the halves of x and c, s the first h columns of cos, sin [T, D].
Computed in fp32, returned in x's dtype.
"""

import torch


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    xf = x.float()
    c = cos[..., :h].float()
    s = sin[..., :h].float()
    lo, hi = xf[..., :h], xf[..., h:]
    return torch.cat((lo * c - hi * s, hi * c + lo * s), dim=-1).to(x.dtype)


def generate_test_inputs(B: int = 4, H: int = 32, T: int = 2048, D: int = 128, dtype: torch.dtype = torch.float16,
                         device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(B, H, T, D, generator=g, device=device).to(dtype)
    cos = torch.randn(T, D, generator=g, device=device).to(dtype)
    sin = torch.randn(T, D, generator=g, device=device).to(dtype)
    return x, cos, sin
