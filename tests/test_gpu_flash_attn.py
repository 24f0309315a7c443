"""GPU parity: tcgen05 flash-attention prefill vs the oracle (fp32), within
2e-2 absolute against fp32, causal and full, bf16 and fp16, tails and both
head dims of the tensor-core path, plus the generic fallback."""

import pytest
import torch

import oracle.ops as O
from b200ops import workloads as WL
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu
ATOL = 2e-2


def check(B, H, T, S, D, causal, dtype, cuda_device, rows=None, seed=0, cfg=None):
    g = torch.Generator(device=cuda_device).manual_seed(seed)
    q = torch.randn(B, H, T, D, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, H, S, D, generator=g, device=cuda_device).to(dtype)
    v = torch.randn(B, H, S, D, generator=g, device=cuda_device).to(dtype)
    lse = torch.empty(B, H, T, device=cuda_device, dtype=torch.float32)
    out = K.flash_attn(q, k, v, causal=causal, lse=lse, cfg=cfg)
    torch.cuda.synchronize()
    assert K.read_device_error() == 0
    exp = O.flash_attn(q.cpu(), k.cpu(), v.cpu(), causal, rows=rows)
    got = out.reshape(B * H, T, D)
    if rows is not None:
        got = got[rows]
    else:
        exp = exp.reshape(B * H, T, D)
    torch.testing.assert_close(got.cpu().float(), exp, rtol=0, atol=ATOL)
    return out


# launch flags: 0 three-warpgroup kernel (default); 16 persistent kernel
# (one CTA per SM taking work items); 4 two-tile kernel (+2: half its
# exponentials on the FMA pipe); 1 one-tile kernel.  split: heads per
# scheduling group.
# tile_k: exponential pairs (of every 8) on the FMA pipe in the default kernel
# (0: the default, 2; 4: none)
@pytest.mark.parametrize("cfg", [{"flags": 0}, {"flags": 0, "split": 1}, {"flags": 0, "split": 5}, {"flags": 16},
                                 {"flags": 16, "split": 3}, {"tile_k": 2}, {"tile_k": 3}, {"tile_k": 4}, {"flags": 4},
                                 {"flags": 6}, {"flags": 1}])
@pytest.mark.parametrize("causal,T,S,D", [(True, 1000, 1000, 128), (False, 130, 517, 128), (True, 700, 700, 64)])
def test_kernel_variants(cfg, causal, T, S, D, cuda_device):
    check(2, 3, T, S, D, causal, torch.bfloat16, cuda_device, cfg=cfg)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("cfg", [None, {"tile_k": 4}, {"flags": 16}])
def test_running_max_rises_across_key_tiles(causal, cfg, cuda_device):
    """Keys whose scores grow along the sequence, so the row maximum rises by
    more than the rescale threshold (2^8) from one key tile to the next: the
    softmax's P computed from the running max is redone with the new max and
    O is rescaled; every element against the fp32 oracle."""
    g = torch.Generator(device=cuda_device).manual_seed(7)
    B, H, T, D = 1, 4, 1024, 128
    q = torch.randn(B, H, T, D, generator=g, device=cuda_device)
    k = torch.randn(B, H, T, D, generator=g, device=cuda_device)
    k = k * (1.0 + torch.arange(T, device=cuda_device, dtype=torch.float32) / 128.0).view(1, 1, T, 1)
    q = (q.abs() + 0.5).bfloat16()  # positive queries against growing positive keys
    k = (k.abs()).bfloat16()
    # outputs of order 1 (a peaked softmax returns single V rows; bf16 rounds
    # an output near 4 by up to 0.016 on its own)
    v = (0.5 * torch.randn(B, H, T, D, generator=g, device=cuda_device)).bfloat16()
    out = K.flash_attn(q, k, v, causal=causal, cfg=cfg)
    torch.cuda.synchronize()
    assert K.read_device_error() == 0
    exp = O.flash_attn(q.cpu(), k.cpu(), v.cpu(), causal)
    torch.testing.assert_close(out.cpu().float(), exp, rtol=0, atol=ATOL)


def test_golden_reference_cases(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "flash_attn_like.pt"):
        q, k, v = (c[n].bfloat16().to(cuda_device) for n in ("q", "k", "v"))
        out = K.flash_attn(q, k, v, causal=c["causal"])
        torch.testing.assert_close(out.cpu().float(), c["out"], rtol=0, atol=ATOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("T", [128, 256, 384, 200, 1])
def test_tc_path_shapes(dtype, causal, T, cuda_device):
    check(2, 3, T, T, 128, causal, dtype, cuda_device)


@pytest.mark.parametrize("causal", [True, False])
def test_head_dim_64(causal, cuda_device):
    check(1, 4, 300, 300, 64, causal, torch.bfloat16, cuda_device)


def test_cross_attention_lengths(cuda_device):
    check(1, 2, 130, 517, 128, False, torch.bfloat16, cuda_device)


def test_generic_fallback_d32(cuda_device):
    check(1, 2, 40, 40, 32, True, torch.bfloat16, cuda_device)


def test_baseline_config_whole_batches(cuda_device):
    """[4,32,4096,128] causal bf16 (the prefill config): one full kernel run,
    every element of all 32 heads of the first and the last batch against the
    fp32 oracle."""
    check(4, 32, 4096, 4096, 128, True, torch.bfloat16, cuda_device, rows=slice(0, 32))
    check(4, 32, 4096, 4096, 128, True, torch.bfloat16, cuda_device, rows=slice(96, 128))
