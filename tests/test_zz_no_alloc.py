"""Allocation-free paged attention through the C ABI.

b200_paged_attention_noalloc serves callers that cannot allocate device
memory -- a host runtime bound through a plain C FFI that holds only the
device pointers it is given, or a request path where cudaMalloc is forbidden
because it can synchronise the device -- by keeping its split-KV scratch in a
static array inside the library instead of a caller workspace.  These tests
call it directly through ctypes and compare it with the workspace entry point
and with the fp32 oracle (same tolerance as the other paged-attention tests,
2e-2 absolute), twice in a row so that the second call runs on the scratch
the first one left behind -- including a launch configuration with claimed
chunks, whose pool counter lives in that shared scratch.  The file is named
to be collected last.
"""

import ctypes

import pytest
import torch

import oracle.ops as O
from b200ops import workloads as WL
from b200ops.runtime import lib as L
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu
ATOL = 2e-2
SCRATCH_LIMIT = 16 << 20  # bytes of static scratch the library holds per device


def _check_rows_against_oracle(out, q, cache, table, ctx):
    """Every output row against the oracle on a compact copy of the row's pages."""
    bs, nb = cache.k_cache.shape[1], cache.k_cache.shape[0]
    for b in range(q.shape[0]):
        c = int(ctx[b])
        nvb = max(0, min((c + bs - 1) // bs, table.shape[1]))
        ids = table[b, :nvb].long()
        valid = (ids >= 0) & (ids < nb)
        uniq = ids[valid]
        remap = torch.full((nvb,), -1, dtype=torch.long)
        remap[valid.cpu()] = torch.arange(int(valid.sum()))
        exp = O.paged_attention(q[b:b + 1].cpu(), cache.k_cache[uniq].cpu(), cache.v_cache[uniq].cpu(),
                                remap.unsqueeze(0), torch.tensor([c]))
        torch.testing.assert_close(out[b:b + 1].cpu().float(), exp, rtol=0, atol=ATOL)


def _workspace_bytes(lib, q, cache, table, cfg):
    B, Hq, D = q.shape
    c = L.LaunchCfg.from_dict(cfg)
    return lib.b200_paged_attention_workspace_size(B, Hq, table.shape[1], cache.k_cache.shape[1], D,
                                                   ctypes.byref(c) if c is not None else None)


def _call(lib, q, cache, table, ctx, out, cfg=None):
    B, Hq, D = q.shape
    nb, bs, Hkv, _ = cache.k_cache.shape
    c = L.LaunchCfg.from_dict(cfg)
    return lib.b200_paged_attention_noalloc(
        q.data_ptr(), cache.k_cache.data_ptr(), cache.v_cache.data_ptr(), table.data_ptr(), ctx.data_ptr(),
        out.data_ptr(), B, Hq, Hkv, D, nb, bs, table.shape[1], 1.0 / D ** 0.5, K.dtype_code(q.dtype),
        K.dtype_code(table.dtype), ctypes.byref(c) if c is not None else None,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("cfg", [None, {"split": 8}])
def test_noalloc_matches_workspace_entry_point_twice(cfg, cuda_device):
    cache = WL.paged_cache(num_blocks=4096, block_size=16, Hkv=8, D=128, device=cuda_device, seed=21)
    inp = WL.decode_attention_inputs(cache, B=24, Hq=32, ctx_lo=17, ctx_hi=2500, device=cuda_device, seed=21)
    ref = K.paged_attention(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"], cfg=cfg)
    torch.cuda.synchronize()
    lib = L.load()
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        st = _call(lib, inp["q"], cache, inp["block_table"], inp["context_len"], out, cfg)
        assert st == L.OK, L.status_string(st)
        torch.cuda.synchronize()
        assert K.read_device_error() == 0
        torch.testing.assert_close(out.float(), ref.float(), rtol=0, atol=ATOL)


def test_noalloc_full_decode_config_against_oracle_twice(cuda_device):
    """The full decode config (64 sequences, ctx U[512,8192], 65536-block
    cache): every row against the oracle and the workspace entry point, on
    two calls in a row."""
    cache = WL.paged_cache(device=cuda_device)
    inp = WL.decode_attention_inputs(cache, device=cuda_device)
    lib = L.load()
    assert _workspace_bytes(lib, inp["q"], cache, inp["block_table"], None) <= SCRATCH_LIMIT
    ref = K.paged_attention(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"])
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        st = _call(lib, inp["q"], cache, inp["block_table"], inp["context_len"], out)
        assert st == L.OK, L.status_string(st)
        torch.cuda.synchronize()
        assert K.read_device_error() == 0
        torch.testing.assert_close(out.float(), ref.float(), rtol=0, atol=ATOL)
        _check_rows_against_oracle(out, inp["q"], cache, inp["block_table"], inp["context_len"])


@pytest.mark.parametrize("cfg", [{"tile_k": 25, "tile_n": 2}, {"tile_m": 16, "tile_k": 50, "tile_n": 4}])
def test_noalloc_claimed_chunks_against_oracle_twice(cfg, cuda_device):
    """Claimed chunks (cfg tile_k percent of the entries, tile_n pages each)
    take their chunks from a pool counter kept in the shared scratch; two
    calls in a row must both match the oracle and the workspace entry point."""
    cache = WL.paged_cache(num_blocks=2048, block_size=16, Hkv=8, D=128, device=cuda_device, seed=23)
    inp = WL.decode_attention_inputs(cache, B=16, Hq=32, ctx_lo=1, ctx_hi=1500, device=cuda_device, seed=23)
    lib = L.load()
    assert _workspace_bytes(lib, inp["q"], cache, inp["block_table"], cfg) <= SCRATCH_LIMIT
    ref = K.paged_attention(inp["q"], cache.k_cache, cache.v_cache, inp["block_table"], inp["context_len"], cfg=cfg)
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        st = _call(lib, inp["q"], cache, inp["block_table"], inp["context_len"], out, cfg)
        assert st == L.OK, L.status_string(st)
        torch.cuda.synchronize()
        assert K.read_device_error() == 0
        torch.testing.assert_close(out.float(), ref.float(), rtol=0, atol=ATOL)
        _check_rows_against_oracle(out, inp["q"], cache, inp["block_table"], inp["context_len"])


def test_noalloc_rejects_scratch_beyond_its_limit():
    """Sizes whose split-KV partials exceed the static scratch are refused on
    the host with a clear error (no pointers are touched, nothing launches)."""
    lib = L.load()
    st = lib.b200_paged_attention_noalloc(None, None, None, None, None, None, 4096, 64, 8, 128, 1 << 20, 16,
                                          8192, 0.0, L.BF16, L.I32, None, None)
    assert st == L.ERR_WORKSPACE
    assert "static scratch holds" in lib.b200_last_error_detail().decode()
