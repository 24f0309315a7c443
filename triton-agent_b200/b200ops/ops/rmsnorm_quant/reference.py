"""rmsnorm + INT8 activation quantiser reference: the composition of
triton_agent/ops/rmsnorm/reference.py:17-18 (evaluated in fp32, cast to x's
dtype) and the row quantiser of triton_agent/ops/quant_matmul/reference.py:16-19
(scale = max|y| / 127 in y's dtype, zero -> 1e-6, codes = clamp(round(y /
scale), -127, 127)).  Returns (codes int8 [B, T, D], scale [B, T, 1]).
"""

import torch

from b200ops.ops.rmsnorm.reference import generate_test_inputs as _rms_inputs
from b200ops.ops.rmsnorm.reference import rmsnorm as _rmsnorm


def rmsnorm_quant(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    y = _rmsnorm(x, weight, eps)
    scale = y.abs().amax(dim=-1, keepdim=True) / 127.0
    scale[scale == 0] = 1e-6
    q = (y / scale).round().clamp(-127, 127).to(torch.int8)
    return q, scale.float()


def generate_test_inputs(B: int = 8, T: int = 2048, D: int = 4096, dtype: torch.dtype = torch.bfloat16,
                         device: str = "cuda", seed: int = 0):
    return _rms_inputs(B, T, D, dtype, device, seed)


def generate_boundary_inputs(device: str = "cuda"):
    cases = []
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        for B, T, D in ((1, 1, 64), (2, 16, 4096), (3, 5, 128)):
            x, w = generate_test_inputs(B, T, D, dtype, device)
            cases.append((x, w, {"eps": 1e-6}))
    return cases
