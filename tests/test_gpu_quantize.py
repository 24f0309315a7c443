"""GPU parity: int8 quantisation codes and scales are bit-identical to the
oracle restatement of quant_matmul/reference.py:16-24."""

import pytest
import torch

import oracle.ops as O
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(7, 64), (33, 130), (1, 4096), (300, 17)])
@pytest.mark.parametrize("by_column", [False, True])
def test_quantize_codes_exact(dtype, shape, by_column, cuda_device):
    g = torch.Generator().manual_seed(shape[0] * 7 + shape[1])
    x = (torch.randn(*shape, generator=g) * 3).to(dtype)
    x[0] = 0  # zero row: scale -> 1e-6
    x[:, 0] = 0
    q, s = K.quantize_int8(x.to(cuda_device), by_column=by_column)
    eq, es = O.quantize_int8(x, by_column=by_column)
    assert torch.equal(q.cpu(), eq)
    assert torch.equal(s.cpu(), es.float())
