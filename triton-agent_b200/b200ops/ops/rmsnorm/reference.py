"""RMSNorm reference (semantics of triton_agent/ops/rmsnorm/reference.py:6-27).

y = x * rsqrt(mean(x^2, -1) + eps) * weight, evaluated in fp32 and returned
in x's dtype.  generate_test_inputs draws x ~ N(0,1) and weight ~ N(1, 0.1).
"""

import torch


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    inv_rms = torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)
    return (xf * inv_rms * weight.float()).to(x.dtype)


def generate_test_inputs(B: int = 8, T: int = 2048, D: int = 4096, dtype: torch.dtype = torch.float16,
                         device: str = "cuda", seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(B, T, D, generator=g, device=device).to(dtype)
    w = (1.0 + 0.1 * torch.randn(D, generator=g, device=device)).to(dtype)
    return x, w


def generate_boundary_inputs(device: str = "cuda"):
    cases = []
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        for B, T, D in ((1, 1, 64), (8, 2048, 4096), (32, 1, 128), (3, 5, 100)):
            x, w = generate_test_inputs(B, T, D, dtype, device)
            cases.append((x, w, {"eps": 1e-6}))
    cases.append((torch.zeros(1, 1, 64, device=device), torch.ones(64, device=device), {"eps": 1e-6}))
    return cases
