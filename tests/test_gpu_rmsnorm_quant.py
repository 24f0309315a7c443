"""GPU parity: rmsnorm fused with the row INT8 quantiser.

Bit-exact means: the codes and scales equal the oracle's quantiser
(quant_matmul/reference.py:16-19, evaluated on the CPU) applied to the
normalised rows y the kernel produced, element for element; and y itself is
the oracle rmsnorm within the rmsnorm tolerance (1e-5 fp32, 1e-2 rel
bf16/fp16).  The one freedom is the order of the fp32 sum of squares, which
can move y by one unit in its last place and so, rarely, a code by one step
against the oracle's own y; that end-to-end composition is bounded
separately."""

import pytest
import torch

import oracle.ops as O
from b200ops.runtime import lib as L
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


def inputs(rows, D, dtype, wdtype, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(rows, D, generator=g, device=dev).to(dtype)
    w = (1.0 + 0.1 * torch.randn(D, generator=g, device=dev)).to(wdtype)
    return x, w


@pytest.mark.parametrize("rows,D,dtype,wdtype", [
    (16, 4096, torch.bfloat16, torch.bfloat16), (37, 4104, torch.bfloat16, torch.float32),
    (64, 4096, torch.float16, torch.float16), (9, 1000, torch.float32, torch.float32),
    (8 * 2048, 4096, torch.bfloat16, torch.bfloat16), (5, 64, torch.float16, torch.float32),
])
# default (warp rows with the next row prefetched into shared memory for
# 16-bit D = 4096, else the persistent CTA kernel or the row kernel) / warp
# rows without the prefetch (flags 4) / the persistent CTA kernel (flags 2) /
# one CTA per row (flags 1) / b200_rmsnorm's CTA size for D=4096, with 1, 2
# and 4 rows per CTA
@pytest.mark.parametrize("cfg", [None, {"flags": 4}, {"flags": 2}, {"flags": 1}, {"threads": 256},
                                 {"threads": 256, "flags": 1}, {"rows_per_cta": 4},
                                 {"threads": 128, "rows_per_cta": 2}])
def test_bit_identical_to_unfused(rows, D, dtype, wdtype, cfg, cuda_device):
    x, w = inputs(rows, D, dtype, wdtype, cuda_device)
    q, s, y = K.rmsnorm_quant_int8(x, w, 1e-6, want_y=True, cfg=cfg)
    torch.cuda.synchronize()
    # the codes and scales are exactly the oracle quantiser's on the y this kernel produced
    q_o, s_o = O.quantize_int8(y.cpu().reshape(rows, D))
    assert torch.equal(q.cpu(), q_o)
    assert torch.equal(s.cpu(), s_o.reshape(-1).float())
    # and the GPU quantiser agrees with both
    q_ref, s_ref = K.quantize_int8(y)
    assert torch.equal(q, q_ref)
    assert torch.equal(s, s_ref.reshape(-1).float())
    # y is the oracle's rmsnorm within the rmsnorm tolerance
    tol_o = 1e-5 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(y.cpu().float(), O.rmsnorm(x.cpu(), w.cpu(), 1e-6).float(), rtol=tol_o, atol=tol_o)
    # y is b200_rmsnorm's output up to the order of the fp32 sum of squares
    # (identical when both reduce in the same order: one CTA per row of the
    # same size)
    y_ref = K.rmsnorm(x, w, 1e-6)
    if cfg is not None and cfg.get("threads") == 256 and cfg.get("flags", 0) & 1:
        assert torch.equal(y, y_ref)
    else:
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        torch.testing.assert_close(y.float(), y_ref.float(), rtol=tol, atol=tol)
    q2, s2 = K.rmsnorm_quant_int8(x, w, 1e-6, cfg=cfg)  # without y
    assert torch.equal(q2, q) and torch.equal(s2, s)


@pytest.mark.parametrize("rows,D", [(1, 4096), (7, 8192), (300, 1024), (2048, 4104), (2048, 4096),
                                    (5000, 1024), (3001, 2048), (4099, 4096)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cfg", [None, {"flags": 2}, {"flags": 4}])
def test_row_loops_and_tails(rows, D, dtype, cfg, cuda_device):
    """The row loops of the warp-row kernel (with and without the shared-
    memory prefetch; several rows per warp group once rows exceed the
    resident groups, which the larger cases force) and of the persistent CTA
    kernel (fewer CTAs than rows, the next row prefetched in registers);
    partial last vectors (D not a multiple of the CTA's vectors), widths
    whose codes land on +-127 and rows that are all zero: codes exactly the
    oracle quantiser's on the kernel's y, and equal to the one-CTA-per-row
    kernel's."""
    x, w = inputs(rows, D, dtype, dtype, cuda_device, seed=rows)
    x[0, :] = 0
    if rows > 3:
        x[3, :] = x[3, :].abs()  # one-signed row: the maximum lands exactly on 127
    q, s, y = K.rmsnorm_quant_int8(x, w, 1e-6, want_y=True, cfg=cfg)
    q1, s1, y1 = K.rmsnorm_quant_int8(x, w, 1e-6, want_y=True, cfg={"flags": 1})
    torch.cuda.synchronize()
    q_o, s_o = O.quantize_int8(y.cpu())
    assert torch.equal(q.cpu(), q_o) and torch.equal(s.cpu(), s_o.reshape(-1).float())
    torch.testing.assert_close(y.float(), y1.float(), rtol=1e-2, atol=1e-2)
    if torch.equal(y, y1):
        assert torch.equal(q, q1) and torch.equal(s, s1)
    assert int(q.abs().max()) <= 127 and int(q[0].abs().max()) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_against_oracle_composition(dtype, cuda_device):
    x, w = inputs(24, 4096, dtype, dtype, cuda_device, seed=3)
    q, s = K.rmsnorm_quant_int8(x, w, 1e-6)
    qo, so = O.rmsnorm_quant_int8(x.cpu(), w.cpu(), 1e-6)
    d = (q.cpu().int() - qo.int()).abs()
    assert int(d.max()) <= 1
    assert float((d == 0).float().mean()) > 0.99
    torch.testing.assert_close(s.cpu(), so.reshape(-1).float(), rtol=1e-2, atol=0)


def test_zero_rows_and_misaligned_width(cuda_device):
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device=cuda_device)
    w = torch.ones(256, dtype=torch.bfloat16, device=cuda_device)
    q, s = K.rmsnorm_quant_int8(x, w)
    torch.cuda.synchronize()
    assert int(q.abs().max()) == 0
    assert torch.equal(s.cpu(), torch.full((4,), O.quantize_int8(torch.zeros(1, 8, dtype=torch.bfloat16))[1].float().item()))
    xb, wb = inputs(4, 4100, torch.bfloat16, torch.bfloat16, cuda_device)
    with pytest.raises(L.B200OpsError):
        K.rmsnorm_quant_int8(xb, wb)
