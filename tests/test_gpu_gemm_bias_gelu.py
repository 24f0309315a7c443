"""GPU parity: bf16/fp16 GEMM + bias + GELU (matmul_epilogue) on the tcgen05
CTA-pair kernel against the fp32 oracle, within one rounding of the output
dtype relative to |c| (1e-2), on tails of M, N and K and the default shape."""

import pytest
import torch

import oracle.ops as O
from b200ops.runtime import lib as L
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


def check(Bt, M, Kd, N, dtype, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    a = (torch.randn(Bt, M, Kd, generator=g, device=dev) / 8).to(dtype)
    b = torch.randn(Kd, N, generator=g, device=dev).to(dtype)
    bias = torch.randn(N, generator=g, device=dev).to(dtype)
    c = K.gemm_bias_gelu(a, b, bias)
    torch.cuda.synchronize()
    assert K.read_device_error() == 0
    exp = O.matmul_epilogue(a, b, bias)
    torch.testing.assert_close(c.cpu().float(), exp, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Bt,M,Kd,N", [(1, 256, 512, 256), (2, 300, 1000, 264), (1, 1, 64, 64),
                                       (3, 130, 4104, 520), (1, 1024, 2048, 4096)])
def test_shapes(Bt, M, Kd, N, dtype, cuda_device):
    check(Bt, M, Kd, N, dtype, cuda_device)


def test_reference_default_shape_sampled(cuda_device):
    """[8,256,4096] x [4096,4096] fp16: full run, oracle on sampled rows."""
    g = torch.Generator(device=cuda_device).manual_seed(1)
    a = (torch.randn(8, 256, 4096, generator=g, device=cuda_device) / 8).half()
    b = torch.randn(4096, 4096, generator=g, device=cuda_device).half()
    bias = torch.randn(4096, generator=g, device=cuda_device).half()
    c = K.gemm_bias_gelu(a, b, bias)
    rows = a.reshape(-1, 4096)[::97]
    exp = O.matmul_epilogue(rows, b, bias)
    torch.testing.assert_close(c.reshape(-1, 4096)[::97].cpu().float(), exp, rtol=1e-2, atol=1e-2)


def test_rejects_unaligned_widths(cuda_device):
    a = torch.randn(4, 100, device=cuda_device).half()
    b = torch.randn(100, 64, device=cuda_device).half()
    with pytest.raises(L.B200OpsError):
        K.gemm_bias_gelu(a, b, torch.zeros(64, device=cuda_device).half())
