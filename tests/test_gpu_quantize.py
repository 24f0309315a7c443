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


# the packed 16-bit paths: warp rows (widths of at most 4096, multiples of 8)
# and 64-column strips (rows a multiple of 16) over a cluster of eight CTAs
# holding their rows in shared memory (up to 4096 rows; 32 and 16 rows leave
# CTAs of the cluster without rows) or, above, of four CTAs reading x twice
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape,by_column", [((16, 64), True), ((32, 128), True), ((1040, 320), True),
                                             ((4096, 1024), True), ((4112, 128), True), ((8192, 64), True),
                                             ((5, 8), False), ((9, 4088), False), ((4100, 2048), False)])
def test_packed_paths_codes_exact(dtype, shape, by_column, cuda_device):
    g = torch.Generator().manual_seed(shape[0] + 3 * shape[1])
    x = (torch.randn(*shape, generator=g) * torch.exp2(torch.randint(-6, 6, (shape[0], 1), generator=g).float()))
    x = x.to(dtype)
    x[0] = 0
    x[:, 1] = 0  # a zero column: scale -> 1e-6
    q, s = K.quantize_int8(x.to(cuda_device), by_column=by_column)
    torch.cuda.synchronize()
    eq, es = O.quantize_int8(x, by_column=by_column)
    assert torch.equal(s.cpu(), es.float().reshape(-1))
    assert torch.equal(q.cpu(), eq)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_codes_exact_at_scale_and_ties(dtype, cuda_device):
    """2048 rows x 4096: random rows of many magnitudes, and rows whose scale
    is a power of two with entries on the half-integer ties of x / scale
    (round half to even) and just beside them -- the codes must match the
    reference rounding everywhere."""
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2048, 4096, generator=g) * torch.exp2(torch.randint(-12, 8, (2048, 1), generator=g).float())
    k = torch.randint(-127, 127, (512, 4096), generator=g).float() + 0.5
    e = torch.exp2(torch.randint(-10, 4, (512, 1), generator=g).float())
    ties = k * e
    ties[:, 0] = 127 * e[:, 0]  # row max: scale = e exactly
    nudge = torch.where(torch.rand(512, 4096, generator=g) < 0.5, 1 - 2.0 ** -7, 1 + 2.0 ** -7)
    x[:512] = ties
    x[512:1024] = ties * nudge
    x = x.to(dtype)
    q, s = K.quantize_int8(x.to(cuda_device))
    eq, es = O.quantize_int8(x)
    assert torch.equal(s.cpu(), es.float().reshape(-1))
    assert torch.equal(q.cpu(), eq)
    # the same values as columns (4096 rows x 2048 columns: the strip path for 16-bit types)
    xt = x.t().contiguous()
    q, s = K.quantize_int8(xt.to(cuda_device), by_column=True)
    eq, es = O.quantize_int8(xt, by_column=True)
    assert torch.equal(s.cpu(), es.float().reshape(-1))
    assert torch.equal(q.cpu(), eq)
