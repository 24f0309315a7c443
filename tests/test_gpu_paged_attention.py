"""GPU parity: paged-attention decode vs the oracle (fp32) and the
reference's golden outputs.  Tolerance: 2e-2 absolute against fp32, checked
on every output element."""

import math

import pytest
import torch

import oracle.ops as O
from b200ops import workloads as WL
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu
ATOL = 2e-2


def run_and_check(q, kc, vc, bt, cl, cuda_device, cfg=None, sample=None):
    out = K.paged_attention(q, kc, vc, bt, cl, cfg=cfg)
    torch.cuda.synchronize()
    assert K.read_device_error() == 0
    B = q.shape[0]
    rows = range(B) if sample is None else sample
    bs = kc.shape[1]
    for b in rows:
        ctx = int(cl[b])
        nvb = max(0, min((ctx + bs - 1) // bs, bt.shape[1]))
        ids = bt[b, :nvb].long()
        nb = kc.shape[0]
        valid = (ids >= 0) & (ids < nb)
        # compact cache holding only this sequence's pages; invalid ids stay invalid
        uniq = ids[valid]
        kk = kc[uniq].cpu() if uniq.numel() else kc[:0].cpu()
        vv = vc[uniq].cpu() if uniq.numel() else vc[:0].cpu()
        remap = torch.full((nvb,), -1, dtype=torch.long)
        remap[valid.cpu()] = torch.arange(int(valid.sum()))
        exp = O.paged_attention(q[b:b + 1].cpu(), kk, vv, remap.unsqueeze(0), torch.tensor([ctx]))
        torch.testing.assert_close(out[b:b + 1].cpu().float(), exp, rtol=0, atol=ATOL)
    return out


def test_golden_reference_cases(golden_dir, cuda_device):
    for c in torch.load(golden_dir / "paged_attention.pt"):
        dt = torch.bfloat16
        q, kc, vc = (c[n].to(dt).to(cuda_device) for n in ("q", "k_cache", "v_cache"))
        out = K.paged_attention(q, kc, vc, c["block_table"].to(cuda_device), c["context_len"].to(cuda_device))
        torch.testing.assert_close(out.cpu().float(), c["out"], rtol=0, atol=ATOL)


def test_baseline_config_every_row(cuda_device):
    """The full decode config (64 sequences, ctx U[512,8192], 65536-block
    cache): every output row against the fp32 oracle, for the default
    persistent kernel and the programmatic-launch flag the decode step uses."""
    cache = WL.paged_cache(device=cuda_device)
    inp = WL.decode_attention_inputs(cache, device=cuda_device)
    for cfg in (None, {"flags": 8}):
        run_and_check(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"], cuda_device,
                      cfg=cfg)


def test_baseline_config_all_rows_vs_single_split(cuda_device):
    """Size-independent property at the full config: the split-KV result
    equals the one-split result (same math, different partition) within
    tolerance, for every sequence."""
    cache = WL.paged_cache(device=cuda_device)
    inp = WL.decode_attention_inputs(cache, device=cuda_device)
    a = K.paged_attention(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"])
    b = K.paged_attention(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"],
                          cfg={"split": 256})
    torch.testing.assert_close(a.float(), b.float(), rtol=0, atol=ATOL)
    # run-to-run determinism of the multi-split path
    c = K.paged_attention(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"])
    assert torch.equal(a, c)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("flags", [0, 1])
def test_gqa_ratios(G, dtype, flags, cuda_device):
    Hkv = 8 if G < 8 else 4
    cache = WL.paged_cache(num_blocks=256, block_size=16, Hkv=Hkv, D=128, dtype=dtype, device=cuda_device, seed=G)
    inp = WL.decode_attention_inputs(cache, B=5, Hq=Hkv * G, ctx_lo=1, ctx_hi=700, device=cuda_device, seed=G)
    run_and_check(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"], cuda_device,
                  cfg={"flags": flags})


def test_garbage_in_unused_slots_is_ignored(cuda_device):
    """Slots past the context length inside the last page may hold anything,
    including NaN; masked tokens must not leak into the output."""
    cache = WL.paged_cache(num_blocks=128, block_size=16, Hkv=8, D=128, device=cuda_device, seed=11)
    inp = WL.decode_attention_inputs(cache, B=4, Hq=32, ctx_lo=20, ctx_hi=400, device=cuda_device, seed=11)
    bt, cl = inp["block_table"], inp["context_len"]
    for b in range(4):
        ctx = int(cl[b])
        last = int(bt[b, (ctx - 1) // 16])
        off = ctx % 16
        if off:
            cache.k_cache[last, off:] = float("nan")
            cache.v_cache[last, off:] = float("nan")
    for flags in (0, 1):
        out = run_and_check(inp["q"], cache.k_cache, cache.v_cache, bt, cl, cuda_device, cfg={"flags": flags})
        assert not torch.isnan(out).any()


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("flags", [0, 1])  # 1: force the CUDA-core consumer
def test_edge_contexts_and_invalid_blocks(index_dtype, flags, cuda_device):
    cache = WL.paged_cache(num_blocks=128, block_size=16, Hkv=8, D=128, device=cuda_device, seed=3)
    B, maxb = 9, 20
    g = torch.Generator(device=cuda_device).manual_seed(5)
    bt = torch.randint(0, 128, (B, maxb), generator=g, device=cuda_device).to(index_dtype)
    cl = torch.tensor([1, 15, 16, 17, 32, 0, 319, 320, 200], device=cuda_device).to(index_dtype)
    bt[6, 3] = -1          # dropped: later blocks shift down (reference.py:40-48)
    bt[8, 0] = 128         # one past the end: dropped
    bt[8, 5] = -7
    q = torch.randn(B, 32, 128, generator=g, device=cuda_device).bfloat16()
    for split in (None, 1, 2, 3, 7):
        cfg = {"split": split or 0, "flags": flags}
        out = run_and_check(q, cache.k_cache, cache.v_cache, bt, cl, cuda_device, cfg=cfg)
        assert torch.count_nonzero(out[5]) == 0  # ctx 0 -> zero row


@pytest.mark.parametrize("bs", [8, 32])
def test_other_block_sizes(bs, cuda_device):
    cache = WL.paged_cache(num_blocks=800, block_size=bs, Hkv=8, D=128, device=cuda_device, seed=bs)
    inp = WL.decode_attention_inputs(cache, B=4, Hq=32, ctx_lo=bs - 3, ctx_hi=1500, device=cuda_device, seed=bs)
    for stages in (2, 3):
        run_and_check(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"], cuda_device,
                      cfg={"stages": stages, "split": 5})


def test_generic_path_head_dim_64(cuda_device):
    cache = WL.paged_cache(num_blocks=64, block_size=16, Hkv=4, D=64, device=cuda_device, seed=9)
    inp = WL.decode_attention_inputs(cache, B=3, Hq=12, ctx_lo=3, ctx_hi=300, device=cuda_device, seed=9)
    run_and_check(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"], cuda_device)


# Persistent kernel partitions: equal static ranges only (flags 4), and
# static ranges plus claimed chunks of tile_n pages for tile_k percent of the
# entries, on grids of tile_m CTAs.  Ranges are a fixed partition of the
# entries, so results must not depend on which CTA claimed which chunk.
@pytest.mark.parametrize("cfg", [{"flags": 4}, {}, {"tile_k": 25}, {"tile_n": 1, "tile_k": 50}, {"tile_n": 2, "tile_k": 90},
                                 {"tile_m": 16, "tile_n": 1, "tile_k": 60}, {"tile_m": 3, "tile_k": 30},
                                 {"rows_per_cta": 4, "tile_k": 40, "tile_n": 3}])
def test_persistent_claimed_chunks(cfg, cuda_device):
    cache = WL.paged_cache(num_blocks=2048, block_size=16, Hkv=8, D=128, device=cuda_device, seed=21)
    inp = WL.decode_attention_inputs(cache, B=16, Hq=32, ctx_lo=1, ctx_hi=1500, device=cuda_device, seed=21)
    bt, cl = inp["block_table"].clone(), inp["context_len"]
    bt[3, 2] = -1  # dropped entry inside a claimed range shifts later blocks
    outs = [run_and_check(inp["q"], cache.k_cache, cache.v_cache, bt, cl, cuda_device, cfg=cfg) for _ in range(2)]
    assert torch.equal(outs[0], outs[1])  # the claim counter re-armed itself; same partition, same bits
    # edge contexts (0, 1, page boundaries) with dropped ids, few entries
    cache2 = WL.paged_cache(num_blocks=128, block_size=16, Hkv=8, D=128, device=cuda_device, seed=3)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    bt2 = torch.randint(0, 128, (9, 20), generator=g, device=cuda_device).to(torch.int32)
    cl2 = torch.tensor([1, 15, 16, 17, 32, 0, 319, 320, 200], device=cuda_device, dtype=torch.int32)
    bt2[6, 3] = -1
    bt2[8, 0] = 128
    q2 = torch.randn(9, 32, 128, generator=g, device=cuda_device).bfloat16()
    out2 = run_and_check(q2, cache2.k_cache, cache2.v_cache, bt2, cl2, cuda_device, cfg=cfg)
    assert torch.count_nonzero(out2[5]) == 0


def test_append_then_decode_with_programmatic_launch(cuda_device):
    """Decode launched with programmatic dependent launch (flags bit 3)
    right after the append, with no synchronisation between them, sees every
    page the append wrote: bit-identical to append, synchronise, decode."""
    cache = WL.paged_cache(num_blocks=16384, block_size=16, Hkv=8, D=128, device=cuda_device, seed=13)
    att = WL.decode_attention_inputs(cache, B=64, Hq=32, ctx_lo=512, ctx_hi=4096, device=cuda_device, seed=13)
    app = WL.decode_append_inputs(cache, n_tok=64, Hq=32, device=cuda_device, seed=13)
    # every appended row lands in a page the decode reads (the first page of each sequence)
    app["slot_mapping"] = (att["block_table"][:, 0].long() * 16 + 5).contiguous()
    k0, v0 = cache.k_cache.clone(), cache.v_cache.clone()
    q_out = torch.empty_like(app["q"])

    def append():
        K.rope_kv_append_paged(app["q"], app["k"], app["v"], app["positions"], app["cos"], app["sin"],
                               app["slot_mapping"], cache.k_cache, cache.v_cache, q_out=q_out)

    append()
    torch.cuda.synchronize()
    ref = K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"], att["context_len"])
    torch.cuda.synchronize()
    for _ in range(3):
        cache.k_cache.copy_(k0)
        cache.v_cache.copy_(v0)
        append()
        out = K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"], att["context_len"],
                                cfg={"flags": 8})
        torch.cuda.synchronize()
        assert K.read_device_error() == 0
        assert torch.equal(out, ref)
    # the appended rows matter: without them the output differs
    cache.k_cache.copy_(k0)
    cache.v_cache.copy_(v0)
    stale = K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"], att["context_len"])
    assert not torch.equal(stale, ref)
