"""GPU parity on the reference's own boundary cases for rmsnorm
(rmsnorm/reference.py:30-44: shapes (1,1,64), (8,2048,4096), (32,1,128) in
fp16/bf16/fp32 with N(0,1) weights, and an all-zero input with unit weights),
for rmsnorm and for rmsnorm fused with the INT8 quantiser.  An all-zero row
normalises to zeros, gets the reference's 1e-6 fallback scale (rounded to the
dtype) and zero codes."""

import pytest
import torch

import oracle.ops as O
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


def tol(dt):
    return dict(rtol=1e-5, atol=1e-5) if dt == torch.float32 else dict(rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 1, 64), (8, 2048, 4096), (32, 1, 128)])
def test_rmsnorm_reference_boundary_shapes(dtype, shape, cuda_device):
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).to(dtype)
    w = torch.randn(shape[-1], generator=g).to(dtype)  # N(0, 1) weights, negative ones included
    y = K.rmsnorm(x.to(cuda_device), w.to(cuda_device), 1e-6)
    if shape[0] * shape[1] > 4096:  # the oracle on a row sample at the large shape
        rows = torch.arange(0, shape[0] * shape[1], 97)
        x2, y2 = x.reshape(-1, shape[-1])[rows], y.reshape(-1, shape[-1])[rows]
        torch.testing.assert_close(y2.cpu().float(), O.rmsnorm(x2, w, 1e-6).float(), **tol(dtype))
    else:
        torch.testing.assert_close(y.cpu().float(), O.rmsnorm(x, w, 1e-6).float(), **tol(dtype))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_all_zero_rows(dtype, cuda_device):
    x = torch.zeros(3, 64, dtype=dtype, device=cuda_device)
    w = torch.ones(64, dtype=dtype, device=cuda_device)
    y = K.rmsnorm(x, w, 1e-6)
    assert torch.count_nonzero(y) == 0
    q, s, yq = K.rmsnorm_quant_int8(x, w, 1e-6, want_y=True)
    torch.cuda.synchronize()
    assert torch.count_nonzero(q) == 0 and torch.count_nonzero(yq) == 0
    expect = torch.tensor(1e-6, dtype=dtype).float().item()  # the fallback scale, rounded to the dtype
    assert torch.all(s.cpu() == expect)
    qo, so = O.rmsnorm_quant_int8(x.cpu(), w.cpu(), 1e-6)
    assert torch.equal(q.cpu(), qo) and torch.allclose(s.cpu(), so.reshape(-1).float())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rmsnorm_quant_negative_weights(dtype, cuda_device):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(32, 128, generator=g).to(dtype)
    w = torch.randn(128, generator=g).to(dtype)
    q, s, y = K.rmsnorm_quant_int8(x.to(cuda_device), w.to(cuda_device), 1e-6, want_y=True)
    q_ref, s_ref = K.quantize_int8(y)
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref.reshape(-1).float())
    qo, so = O.rmsnorm_quant_int8(x, w, 1e-6)
    d = (q.cpu().int() - qo.int()).abs()
    assert int(d.max()) <= 1
