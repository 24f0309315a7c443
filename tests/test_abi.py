"""C ABI: the library loads, exports every entry point include/b200ops.h
declares, and rejects bad arguments / injected faults on the host without
touching a GPU."""

import ctypes
import re
from pathlib import Path

import pytest

from b200ops.runtime import lib as L

HEADER = Path(__file__).resolve().parent.parent / "include" / "b200ops.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert set(declared_symbols()) == set(L.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(L.lib_path()))
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_status_strings_and_version():
    L.load()
    assert L.status_string(0) == "ok"
    assert "injected" in L.status_string(L.ERR_INJECTED)
    assert L.version() >= 100
    names = L.kernel_names()
    for k in ("paged_decode_kernel", "int8_gemm_tcgen05_kernel", "flash_fwd_tcgen05_kernel", "rmsnorm_row_kernel"):
        assert k in names


def test_bad_arguments_rejected_on_host():
    lib = L.load()
    # negative sizes / null pointers never reach a launch
    assert lib.b200_rmsnorm(None, None, None, -1, 4096, 1e-6, L.F32, L.F32, None, None) == L.ERR_BAD_ARG
    assert lib.b200_rmsnorm(None, None, None, 4, 4096, 1e-6, L.F32, L.F32, None, None) == L.ERR_BAD_ARG
    assert lib.b200_rmsnorm(None, None, None, 0, 4096, 1e-6, L.F32, L.F32, None, None) == L.OK  # empty
    assert lib.b200_rope(None, None, None, None, 1, 1, 1, 7, L.F32, L.F32, None, None) == L.ERR_BAD_ARG  # odd D
    assert lib.b200_paged_attention(None, None, None, None, None, None, 2, 32, 6, 128, 16, 16, 4, 0.0,
                                    L.BF16, L.I32, None, 0, None, None) == L.ERR_BAD_ARG  # Hq % Hkv != 0
    assert lib.b200_int8_gemm(None, None, None, None, None, 4, 4, 40, 4, L.F16, None, None, 0, None,
                              None) == L.ERR_BAD_ARG  # null operands
    assert lib.b200_flash_attn(None, None, None, None, None, 1, 1, 8, 9, 64, 0.0, 1, L.BF16, None,
                               None) == L.ERR_BAD_ARG  # causal with T != S


def test_workspace_sizes():
    lib = L.load()
    n = lib.b200_paged_attention_workspace_size(64, 32, 512, 16, 128, None)
    # fixed ticket region + (o, m, l) per (sequence, head, split)
    assert n == 256 * 1024 + 64 * 32 * 8 * (128 + 2) * 4  # default split: 64 blocks
    cfg = L.LaunchCfg(split=16)
    assert lib.b200_paged_attention_workspace_size(64, 32, 512, 16, 128, ctypes.byref(cfg)) == \
        256 * 1024 + 64 * 32 * 32 * 130 * 4
    assert lib.b200_int8_gemm_workspace_size(4096, 4096, 4096, None) == 0  # enough tiles: no split-K
    assert lib.b200_int8_gemm_workspace_size(16, 4096, 4096, None) > 0


def test_host_fault_injection(monkeypatch):
    """B200OPS_INJECT_ERROR fails an entry point on the host, before any
    launch; the Python layer raises B200OpsError with the status."""
    lib = L.load()
    monkeypatch.setenv("B200OPS_INJECT_ERROR", "rmsnorm")
    assert lib.b200_rmsnorm(None, None, None, 4, 64, 1e-6, L.F32, L.F32, None, None) == L.ERR_INJECTED
    assert "injected" in lib.b200_last_error_detail().decode()
    with pytest.raises(L.B200OpsError) as ei:
        L.check(L.ERR_INJECTED, "rmsnorm")
    assert ei.value.code == L.ERR_INJECTED
    monkeypatch.setenv("B200OPS_INJECT_ERROR", "all")
    assert lib.b200_paged_attention(None, None, None, None, None, None, 1, 1, 1, 128, 1, 16, 1, 0.0, L.BF16, L.I32,
                                    None, 0, None, None) == L.ERR_INJECTED


def test_ops_refuse_cpu_tensors():
    """No CPU path: host tensors raise instead of computing anywhere else."""
    import torch

    from b200ops.runtime import ops as K

    with pytest.raises(L.B200OpsError) as ei:
        K.rmsnorm(torch.randn(2, 8), torch.randn(8))
    assert ei.value.code == L.ERR_NO_DEVICE


def test_decode_workspace_sizes_for_claimed_chunks():
    """Claimed chunks (cfg tile_k percent) need partial rows per chunk, so the
    workspace query grows with the percent and shrinks with the chunk size;
    the default (no claimed chunks) and equal ranges only (flags bit 2) ask
    for the same bytes, within the 16 MiB scratch of the allocation-free
    entry point at the bench shape (64 sequences, 32 heads, 512 blocks)."""
    lib = L.load()

    def ws(**kw):
        cfg = L.LaunchCfg(**kw) if kw else None
        return lib.b200_paged_attention_workspace_size(64, 32, 512, 16, 128, ctypes.byref(cfg) if cfg else None)

    base = ws()
    assert ws(flags=4) == base
    assert ws(tile_k=25) > base
    assert ws(tile_k=50) >= ws(tile_k=25)
    assert ws(tile_k=25, tile_n=16) <= ws(tile_k=25, tile_n=4)
    assert base <= 16 << 20
