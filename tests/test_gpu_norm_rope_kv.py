"""GPU parity: rmsnorm, RoPE and the KV-append family against the oracle and
the reference's golden outputs.

Bars: cache writes, copies and fp32 RoPE are bit-exact; rmsnorm within
1e-5 (fp32) / 1e-2 relative (bf16, fp16), the stated tolerance.
"""

import pytest
import torch

import oracle.ops as O
from b200ops import workloads as WL
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


def tol(dt):
    return dict(rtol=1e-5, atol=1e-5) if dt == torch.float32 else dict(rtol=1e-2, atol=1e-2)


# ------------------------------------------------------------------ rmsnorm
def test_rmsnorm_golden(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "rmsnorm.pt"):
        y = K.rmsnorm(c["x"].to(cuda_device), c["w"].to(cuda_device), c["eps"])
        torch.testing.assert_close(y.cpu().float(), c["y"].float(), **tol(c["x"].dtype))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(4, 7, 4096), (3, 5, 128), (2, 3, 100), (1, 1, 64), (2, 2, 8192),
                                   (1, 3, 4097), (5, 1, 24)])
def test_rmsnorm_shapes(dtype, shape, cuda_device):
    g = torch.Generator().manual_seed(hash(shape) % 1000)
    x = torch.randn(*shape, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
    y = K.rmsnorm(x.to(cuda_device), w.to(cuda_device), 1e-6)
    ref = O.rmsnorm(x, w, 1e-6)
    assert y.dtype == dtype
    torch.testing.assert_close(y.cpu().float(), ref.float(), **tol(dtype))


def test_rmsnorm_fp32_weight_with_bf16_x(cuda_device):
    x = torch.randn(3, 256).bfloat16()
    w = torch.randn(256)
    y = K.rmsnorm(x.to(cuda_device), w.to(cuda_device))
    torch.testing.assert_close(y.cpu().float(), O.rmsnorm(x, w).float(), rtol=1e-2, atol=1e-2)


def test_rmsnorm_baseline_shape(cuda_device):
    x, w = WL.rmsnorm_inputs(device=cuda_device)
    y = K.rmsnorm(x, w, 1e-6)
    ref = O.rmsnorm(x.cpu(), w.cpu(), 1e-6)
    torch.testing.assert_close(y.cpu(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("threads", [64, 128, 512, 1024])
def test_rmsnorm_launch_configs(threads, cuda_device):
    x = torch.randn(6, 4096, device=cuda_device)
    w = torch.randn(4096, device=cuda_device)
    y = K.rmsnorm(x, w, cfg={"threads": threads})
    torch.testing.assert_close(y.cpu(), O.rmsnorm(x.cpu(), w.cpu()), rtol=1e-5, atol=1e-5)


# --------------------------------------------------------------------- RoPE
def test_rope_golden_bit_exact_fp32(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "rope.pt"):
        y = K.rope(c["x"].to(cuda_device), c["cos"].to(cuda_device), c["sin"].to(cuda_device))
        if c["x"].dtype == torch.float32:
            assert torch.equal(y.cpu(), c["y"])
        else:
            torch.testing.assert_close(y.cpu().float(), c["y"].float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [128, 64, 10])
def test_rope_vs_oracle_bit_exact(dtype, D, cuda_device):
    x = torch.randn(2, 3, 5, D).to(dtype)
    cos = torch.randn(5, D).to(dtype)
    sin = torch.randn(5, D).to(dtype)
    y = K.rope(x.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device))
    assert torch.equal(y.cpu(), O.rope(x, cos, sin))


# ------------------------------------------------------------------ appends
def test_kv_append_golden_exact(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "kv_append.pt"):
        kc, vc = c["k_cache"].to(cuda_device), c["v_cache"].to(cuda_device)
        K.kv_append(kc, vc, c["k_new"].to(cuda_device), c["v_new"].to(cuda_device),
                    c["slot_mapping"].to(cuda_device))
        assert torch.equal(kc.cpu(), c["k_out"]) and torch.equal(vc.cpu(), c["v_out"])


def test_paged_kv_golden_exact(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "paged_kv.pt"):
        kc, vc = c["k_cache"].to(cuda_device), c["v_cache"].to(cuda_device)
        K.paged_kv(kc, vc, c["k_new"].to(cuda_device), c["v_new"].to(cuda_device),
                   c["slot_mapping"].to(cuda_device))
        assert torch.equal(kc.cpu(), c["k_out"]) and torch.equal(vc.cpu(), c["v_out"])


def test_rope_kv_append_golden_exact(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "rope_kv_append.pt"):
        kc = c["k_cache"].to(cuda_device)
        K.rope_kv_append(c["k_new"].to(cuda_device), c["cos"].to(cuda_device), c["sin"].to(cuda_device), kc,
                         c["slot_mapping"].to(cuda_device))
        assert torch.equal(kc.cpu(), c["k_out"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T_new", [1, 5, 40])
def test_kv_family_random_with_collisions(dtype, T_new, cuda_device):
    g = torch.Generator().manual_seed(T_new)
    B, H, Lc, D = 3, 4, 24, 64
    kc = torch.randn(B, H, Lc, D, generator=g).to(dtype)
    vc = torch.randn(B, H, Lc, D, generator=g).to(dtype)
    kn = torch.randn(B, H, T_new, D, generator=g).to(dtype)
    vn = torch.randn(B, H, T_new, D, generator=g).to(dtype)
    sm = torch.randint(-3, Lc + 3, (B, T_new), generator=g)
    ek, ev = O.kv_append(kc, vc, kn, vn, sm)
    gk, gv = kc.to(cuda_device), vc.to(cuda_device)
    K.kv_append(gk, gv, kn.to(cuda_device), vn.to(cuda_device), sm.to(cuda_device))
    assert torch.equal(gk.cpu(), ek) and torch.equal(gv.cpu(), ev)
    # rope variant on the same data
    cos = torch.randn(T_new, D, generator=g).to(dtype)
    sin = torch.randn(T_new, D, generator=g).to(dtype)
    ek2 = O.rope_kv_append(kn, cos, sin, kc, sm)
    gk2 = kc.to(cuda_device)
    K.rope_kv_append(kn.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device), gk2, sm.to(cuda_device))
    assert torch.equal(gk2.cpu(), ek2)
    # paged layout
    nb, bs = 5, 4
    pk = torch.randn(nb, bs, H, D, generator=g).to(dtype)
    pv = torch.randn(nb, bs, H, D, generator=g).to(dtype)
    pkn = torch.randn(B, T_new, H, D, generator=g).to(dtype)
    pvn = torch.randn(B, T_new, H, D, generator=g).to(dtype)
    psm = torch.randint(-5, nb * bs + 5, (B, T_new), generator=g)
    ek3, ev3 = O.paged_kv(pk, pv, pkn, pvn, psm)
    gk3, gv3 = pk.to(cuda_device), pv.to(cuda_device)
    K.paged_kv(gk3, gv3, pkn.to(cuda_device), pvn.to(cuda_device), psm.to(cuda_device))
    assert torch.equal(gk3.cpu(), ek3) and torch.equal(gv3.cpu(), ev3)


def _check_fused_append(cache, inp, cuda_device):
    kc0, vc0 = cache.k_cache.clone(), cache.v_cache.clone()
    q_out = K.rope_kv_append_paged(inp["q"], inp["k"], inp["v"], inp["positions"], inp["cos"], inp["sin"],
                                   inp["slot_mapping"], cache.k_cache, cache.v_cache)
    nslots = cache.num_blocks * cache.block_size
    eq, ek, ev, keep = O.rope_kv_append_paged(inp["q"], inp["k"], inp["v"], inp["positions"], inp["cos"],
                                              inp["sin"], inp["slot_mapping"], nslots)
    assert torch.equal(q_out.cpu(), eq)
    Hkv, D = cache.k_cache.shape[2:]
    sl = inp["slot_mapping"].cpu()[keep]
    blk, off = sl // cache.block_size, sl % cache.block_size
    exp_k, exp_v = kc0, vc0
    exp_k[blk.to(cuda_device), off.to(cuda_device)] = ek[keep].to(cuda_device)
    exp_v[blk.to(cuda_device), off.to(cuda_device)] = ev[keep].to(cuda_device)
    # whole-cache comparison on the device: touched rows match the oracle,
    # every other row is untouched
    assert torch.equal(cache.k_cache, exp_k)
    assert torch.equal(cache.v_cache, exp_v)


def test_fused_decode_append_baseline_config(cuda_device):
    cache = WL.paged_cache(device=cuda_device)
    inp = WL.decode_append_inputs(cache, device=cuda_device)
    _check_fused_append(cache, inp, cuda_device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_decode_append_edge_cases(dtype, cuda_device):
    cache = WL.paged_cache(num_blocks=32, block_size=16, Hkv=2, D=128, dtype=dtype, device=cuda_device)
    inp = WL.decode_append_inputs(cache, n_tok=9, Hq=8, max_pos=64, device=cuda_device)
    sm = inp["slot_mapping"]
    sm[1] = -1                       # skipped
    sm[2] = 32 * 16                  # one past the end: skipped
    sm[5] = sm[3]                    # collision: token 5 wins
    _check_fused_append(cache, inp, cuda_device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_append_prefill_slot_owner_table(dtype, cuda_device):
    """More than 512 new tokens take the slot-ownership table path: later
    tokens win collisions (including runs of three), invalid slots are
    skipped, and a second call with another pattern sees a clean table."""
    cache = WL.paged_cache(num_blocks=256, block_size=16, Hkv=2, D=128, dtype=dtype, device=cuda_device)
    for seed in (0, 1):
        inp = WL.decode_append_inputs(cache, n_tok=2000, Hq=4, max_pos=4096, device=cuda_device, seed=seed)
        sm = inp["slot_mapping"]
        sm[10] = -5
        sm[11] = 256 * 16
        sm[100] = sm[50]
        sm[1500] = sm[50]              # three writers of one slot: token 1500 wins
        sm[1999] = sm[0]
        sm[7 + seed] = sm[900]         # token 900 wins over the earlier one
        _check_fused_append(cache, inp, cuda_device)


@pytest.mark.parametrize("cfg_rows", [None, 2, 3, 6, 12])
def test_fused_append_prefill_bench_shape(cfg_rows, cuda_device):
    """The prefill-size append at the bench shape (16384 tokens, 32 q / 8 kv
    heads, 48 rows per token -> the rows-per-thread kernel, two tokens per
    CTA at the default), with collisions, invalid slots and out-of-table
    positions, bit-exact against the oracle over the whole cache."""
    cache = WL.paged_cache(num_blocks=16384, block_size=16, Hkv=8, D=128, device=cuda_device, seed=9)
    inp = WL.decode_append_inputs(cache, n_tok=16384, Hq=32, device=cuda_device, seed=9)
    sm, pos = inp["slot_mapping"], inp["positions"]
    sm[5] = -1
    sm[6] = 16384 * 16
    sm[16383] = sm[100]            # the last token wins
    sm[9000] = sm[8999]
    pos[77] = -3                   # out of the cos/sin table: the token's rows stay untouched
    cfg = {"rows_per_cta": cfg_rows} if cfg_rows else None
    kc0, vc0 = cache.k_cache.clone(), cache.v_cache.clone()
    q_out = K.rope_kv_append_paged(inp["q"], inp["k"], inp["v"], pos, inp["cos"], inp["sin"], sm,
                                   cache.k_cache, cache.v_cache, cfg=cfg)
    nslots = cache.num_blocks * cache.block_size
    eq, ek, ev, keep = O.rope_kv_append_paged(inp["q"], inp["k"], inp["v"], pos, inp["cos"], inp["sin"], sm, nslots)
    keep = keep.clone()
    keep[77] = False               # its slot is unique, so the cache keeps the old row there
    got_q = q_out.cpu()
    ok_rows = (pos.cpu() >= 0)
    assert torch.equal(got_q[ok_rows], eq[ok_rows])
    sl = sm.cpu()[keep]
    blk, off = sl // cache.block_size, sl % cache.block_size
    kc0[blk.to(cuda_device), off.to(cuda_device)] = ek[keep].to(cuda_device)
    vc0[blk.to(cuda_device), off.to(cuda_device)] = ev[keep].to(cuda_device)
    assert torch.equal(cache.k_cache, kc0)
    assert torch.equal(cache.v_cache, vc0)
