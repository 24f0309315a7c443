"""GPU parity: tcgen05 INT8 GEMM.  int32 accumulators are bit-exact against
the oracle's exact integer GEMM; the dequantised output is bit-exact too
(same fp32 product order, one final rounding); the reference-API path
(quantise a and b, GEMM, rescale) matches the reference's fp32 output."""

import numpy as np
import pytest
import torch

import oracle.ops as O
from b200ops import workloads as WL
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


def check(M, N, K_, cuda_device, out_dtype=torch.float16, cfg=None, seed=0, with_acc=True, sw_offset=0):
    """Dequantised output bit-exact against the oracle; with_acc also returns
    the raw int32 accumulators (which routes the tile kernels' epilogue
    through per-row stores; without them 16-bit and fp32 outputs go through
    the staged epilogue).  sw_offset shifts sW by that many floats in its
    buffer (unaligned scales also take the per-row path)."""
    A, W, sA, sW = WL.int8_gemm_inputs(M, N, K_, device=cuda_device, seed=seed)
    if sw_offset:
        buf = torch.empty(N + sw_offset, dtype=torch.float32, device=cuda_device)
        buf[sw_offset:] = sW
        sW = buf[sw_offset:]
    acc = torch.empty(M, N, dtype=torch.int32, device=cuda_device) if with_acc else None
    C = K.int8_gemm(A, W, sA, sW, out_dtype=out_dtype, acc_out=acc, cfg=cfg)
    torch.cuda.synchronize()
    assert K.read_device_error() == 0
    exp_acc = O.int8_gemm_acc(A.cpu(), W.cpu())
    if with_acc:
        assert np.array_equal(acc.cpu().numpy().astype(np.int64), exp_acc)
    exp = O.dequant(exp_acc, sA.cpu(), sW.cpu(), out_dtype)
    assert torch.equal(C.cpu(), exp)


# the staged epilogue (no raw accumulators): groups of 256-byte rows (128
# columns of a 16-bit output, 64 of fp32) staged in shared memory and written
# as whole row runs, ragged edges by rows
@pytest.mark.parametrize("cfg", [None, {"tile_n": 128}, {"tile_n": 224}, {"flags": 2}, {"flags": 2, "tile_n": 128}])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,N,K_", [(600, 1000, 640), (512, 4096, 1024), (300, 448, 256), (4096, 1280, 128)])
def test_int8_gemm_staged_epilogue(cfg, out_dtype, M, N, K_, cuda_device):
    for seed in (0, 1):
        check(M, N, K_, cuda_device, out_dtype=out_dtype, cfg=cfg, seed=seed, with_acc=False)


# the CTA-pair kernel's last partial wave split into half-width items (on 74
# CTA pairs: 256, 84, 80 and 896 tiles leave 34, 10, 6 and 8 for the last
# wave); flags bit 3 keeps whole tiles
@pytest.mark.parametrize("cfg", [None, {"flags": 8}])
@pytest.mark.parametrize("M,N,K_", [(4096, 4096, 256), (1024, 5184, 384), (1024, 5120, 128), (4096, 14336, 128)])
@pytest.mark.parametrize("with_acc", [True, False])
def test_int8_gemm_last_wave_halves(cfg, M, N, K_, with_acc, cuda_device):
    check(M, N, K_, cuda_device, cfg=cfg, with_acc=with_acc)
    if not with_acc:
        check(M, N, K_, cuda_device, out_dtype=torch.float32, cfg=cfg, with_acc=False)


def test_int8_gemm_unaligned_scales_take_the_row_path(cuda_device):
    check(600, 1000, 640, cuda_device, with_acc=False, sw_offset=1)
    check(600, 1000, 640, cuda_device, out_dtype=torch.float32, with_acc=False, sw_offset=1)


@pytest.mark.parametrize("M,N,K_", [(128, 256, 128), (256, 512, 1024), (130, 200, 48), (1, 8, 16),
                                    (300, 1000, 4096), (16, 4096, 4096)])
def test_int8_gemm_exact(M, N, K_, cuda_device):
    check(M, N, K_, cuda_device)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_int8_gemm_out_dtypes(out_dtype, cuda_device):
    check(200, 384, 512, cuda_device, out_dtype=out_dtype)


# flags bit 1 selects the one-SM persistent kernel over the CTA-pair kernel
# (the default for M > 128); tile_n is the tile width of either
@pytest.mark.parametrize("cfg", [{"flags": 2, "tile_n": 128}, {"flags": 2, "tile_n": 256}, {"split": 4},
                                 {"stages": 2}, {"flags": 2, "stages": 3}, {"tile_n": 128, "split": 3, "stages": 3}])
def test_int8_gemm_configs(cfg, cuda_device):
    check(256, 768, 2048, cuda_device, cfg=cfg)


# small M: the streaming kernel (default; W cut into one k-range per SM) and
# the split-grid kernel (flags bit 2), with ragged N and K and repeated calls
# (the partial-sum workspace must come back to zero)
@pytest.mark.parametrize("cfg", [None, {"flags": 4}, {"stages": 3}, {"flags": 4, "split": 3}, {"tile_k": 128},
                                 {"tile_k": 1024, "stages": 2}])
@pytest.mark.parametrize("M,N,K_", [(1, 300, 4096), (16, 1000, 1008), (33, 4096, 640), (64, 2000, 8192)])
def test_int8_gemm_skinny_kernels(cfg, M, N, K_, cuda_device):
    for seed in (0, 1):
        check(M, N, K_, cuda_device, cfg=cfg, seed=seed)


# CTA-pair tile widths (tile_n 128..256, each CTA loading tile_n / 2 W rows;
# the default picks the width whose tiles fill whole waves of CTA pairs), on
# ragged N and M, and the streaming kernel's grid size (tile_m)
@pytest.mark.parametrize("cfg", [{"tile_n": 128}, {"tile_n": 160}, {"tile_n": 192}, {"tile_n": 224}, {"tile_n": 256}])
@pytest.mark.parametrize("M,N,K_", [(600, 1000, 640), (512, 4096, 1024), (300, 448, 256)])
def test_int8_gemm_pair_tile_widths(cfg, M, N, K_, cuda_device):
    check(M, N, K_, cuda_device, cfg=cfg)


@pytest.mark.parametrize("cfg", [{"tile_m": 7}, {"tile_m": 64}, {"tile_m": 112}, {"tile_m": 148}, {"tile_m": 1000}])
def test_int8_gemm_streaming_grid_sizes(cfg, cuda_device):
    for seed in (0, 1):
        check(16, 3000, 4096, cuda_device, cfg=cfg, seed=seed)


@pytest.mark.parametrize("M,N,K_", [(600, 1000, 640), (257, 300, 128), (129, 256, 4128), (1024, 4096, 48)])
def test_int8_gemm_pair_kernel_tails(M, N, K_, cuda_device):
    """CTA-pair kernel: several 256 x 256 tiles per pair, ragged M, N and K."""
    check(M, N, K_, cuda_device)


def test_int8_gemm_baseline_shapes_checksum(cuda_device):
    """Full-size shapes (4096 x 4096, 4096 x 14336 and 16 x 14336, K = 4096): exact integer checks that do not need a full
    CPU GEMM -- column sums of the accumulator equal (1^T A) W^T and row sums
    equal A (W^T 1), both in int64, plus a sampled block compared exactly."""
    for M, N in [(4096, 4096), (4096, 14336), (16, 14336)]:
        K_ = 4096
        A, W, sA, sW = WL.int8_gemm_inputs(M, N, K_, device=cuda_device)
        acc = torch.empty(M, N, dtype=torch.int32, device=cuda_device)
        C = K.int8_gemm(A, W, sA, sW, acc_out=acc)
        col = acc.to(torch.int64).sum(0).cpu()
        row = acc.to(torch.int64).sum(1).cpu()
        a64 = A.cpu().numpy().astype(np.int64)
        w64 = W.cpu().numpy().astype(np.int64)
        assert np.array_equal(col.numpy(), a64.sum(0) @ w64.T)
        assert np.array_equal(row.numpy(), a64 @ w64.sum(0))
        r0, c0 = M // 3, N // 5
        blk = O.int8_gemm_acc(A[r0:r0 + 16].cpu(), W[c0:c0 + 64].cpu())
        assert np.array_equal(acc[r0:r0 + 16, c0:c0 + 64].cpu().numpy().astype(np.int64), blk)
        exp = O.dequant(blk, sA[r0:r0 + 16].cpu(), sW[c0:c0 + 64].cpu(), torch.float16)
        assert torch.equal(C[r0:r0 + 16, c0:c0 + 64].cpu(), exp)


def test_quant_matmul_reference_api_golden(golden_dir, cuda_device):
    """quantise a per row and b per column on the GPU, int8 GEMM, fp32
    rescale -- equals the reference's quant_matmul output bit for bit."""
    for c in torch.load(golden_dir / "quant_matmul.pt"):
        a, b = c["a"].to(cuda_device), c["b"].to(cuda_device)
        lead, (M, K_) = a.shape[:-2], a.shape[-2:]
        qa, sa = K.quantize_int8(a.reshape(-1, K_))
        qb, sb = K.quantize_int8(b, by_column=True)
        if K_ % 16:
            pytest.skip("K not a multiple of 16")
        out = K.int8_gemm(qa, qb, sa, sb, out_dtype=torch.float32).reshape(*lead, M, -1)
        assert torch.equal(out.cpu(), c["c"])
