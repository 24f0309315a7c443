"""ctypes binding of libb200ops.so (the C ABI declared in include/b200ops.h).

Loads the in-tree library (triton-agent_b200/lib/libb200ops.so, or the path
in B200OPS_LIB), declares every entry point's argument types, and maps a
non-zero status to B200OpsError.  Nothing here falls back to another
implementation: a missing library raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[2]
DEFAULT_LIB = PKG_ROOT / "lib" / "libb200ops.so"

# b200_status / b200_dtype values from include/b200ops.h
OK = 0
ERR_BAD_ARG = -1
ERR_UNSUPPORTED = -2
ERR_LAUNCH = -3
ERR_DEVICE_TIMEOUT = -4
ERR_WORKSPACE = -5
ERR_NO_DEVICE = -6
ERR_INJECTED = -7
ERR_ALIGNMENT = -8

F32, F16, BF16, I8, I32, I64 = 0, 1, 2, 3, 4, 5


class B200OpsError(RuntimeError):
    """A libb200ops entry point returned a non-zero status."""

    def __init__(self, code: int, op: str, detail: str = ""):
        self.code = code
        self.op = op
        msg = f"{op}: {status_string(code)} (status {code})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


class LaunchCfg(ctypes.Structure):
    """b200_launch_cfg: tuner-chosen launch/tile parameters (0 = default)."""

    _fields_ = [
        ("threads", c_int32),
        ("rows_per_cta", c_int32),
        ("stages", c_int32),
        ("split", c_int32),
        ("tile_m", c_int32),
        ("tile_n", c_int32),
        ("tile_k", c_int32),
        ("flags", c_int32),
    ]

    @classmethod
    def from_dict(cls, d: dict | None) -> "LaunchCfg | None":
        if not d:
            return None
        cfg = cls()
        for name, _ in cls._fields_:
            if name in d and d[name] is not None:
                setattr(cfg, name, int(d[name]))
        return cfg


P = c_void_p
I64_ = c_int64
PCFG = POINTER(LaunchCfg)

# name -> (restype, argtypes); the same order as include/b200ops.h
SIGNATURES = {
    "b200_status_string": (c_char_p, [c_int]),
    "b200_version": (c_int, []),
    "b200_kernel_list": (c_char_p, []),
    "b200_last_error_detail": (c_char_p, []),
    "b200_read_device_error": (c_int, [POINTER(c_int32), P]),
    "b200_query_config_space": (c_char_p, [c_char_p, I64_]),
    "b200_set_peer_wait_timeout_us": (c_int, [I64_]),
    "b200_rmsnorm": (c_int, [P, P, P, I64_, I64_, c_float, c_int32, c_int32, PCFG, P]),
    "b200_rmsnorm_quant_int8": (c_int, [P, P, P, P, P, I64_, I64_, c_float, c_int32, c_int32, PCFG, P]),
    "b200_rope": (c_int, [P, P, P, P, I64_, I64_, I64_, I64_, c_int32, c_int32, PCFG, P]),
    "b200_kv_append": (c_int, [P, P, P, P, P, I64_, I64_, I64_, I64_, I64_, c_int32, PCFG, P]),
    "b200_paged_kv": (c_int, [P, P, P, P, P, I64_, I64_, I64_, I64_, I64_, I64_, c_int32, PCFG, P]),
    "b200_rope_kv_append": (c_int, [P, P, P, P, P, I64_, I64_, I64_, I64_, I64_, c_int32, c_int32, PCFG, P]),
    "b200_rope_kv_append_paged": (
        c_int,
        [P, P, P, P, P, P, I64_, P, P, P, P, I64_, I64_, I64_, I64_, I64_, I64_, c_int32, c_int32, PCFG, P],
    ),
    "b200_rope_kv_append_paged_ws": (
        c_int,
        [P, P, P, P, P, P, I64_, P, P, P, P, I64_, I64_, I64_, I64_, I64_, I64_, c_int32, c_int32, P, I64_, PCFG,
         P],
    ),
    "b200_paged_attention_workspace_size": (c_size_t, [I64_, I64_, I64_, I64_, I64_, PCFG]),
    "b200_paged_attention": (
        c_int,
        [P, P, P, P, P, P, I64_, I64_, I64_, I64_, I64_, I64_, I64_, c_float, c_int32, c_int32, P, c_size_t,
         PCFG, P],
    ),
    "b200_paged_attention_noalloc": (
        c_int,
        [P, P, P, P, P, P, I64_, I64_, I64_, I64_, I64_, I64_, I64_, c_float, c_int32, c_int32, PCFG, P],
    ),
    "b200_int8_gemm_workspace_size": (c_size_t, [I64_, I64_, I64_, PCFG]),
    "b200_int8_gemm": (c_int, [P, P, P, P, P, I64_, I64_, I64_, I64_, c_int32, P, P, c_size_t, PCFG, P]),
    "b200_gemm_bias_gelu": (c_int, [P, P, P, P, I64_, I64_, I64_, c_int32, PCFG, P]),
    "b200_int8_gemm_allgather": (
        c_int,
        [P, P, P, P, POINTER(c_void_p), POINTER(c_void_p), c_int32, c_int32, I64_, I64_, I64_, I64_, I64_, c_int32,
         c_uint32, P, c_size_t, PCFG, P],
    ),
    "b200_ipc_handle": (c_int, [P, P, POINTER(c_int64)]),
    "b200_ipc_open": (c_int, [P, I64_, POINTER(c_void_p)]),
    "b200_ipc_close": (c_int, [P, I64_]),
    "b200_quantize_int8": (c_int, [P, P, P, I64_, I64_, c_int32, c_int32, PCFG, P]),
    "b200_flash_attn": (
        c_int, [P, P, P, P, P, I64_, I64_, I64_, I64_, I64_, c_float, c_int32, c_int32, PCFG, P]
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib_path() -> Path:
    env = os.environ.get("B200OPS_LIB")
    return Path(env) if env else DEFAULT_LIB


def load() -> ctypes.CDLL:
    """Loads libb200ops.so once; raises if it is missing or lacks a symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not path.exists():
            raise B200OpsError(ERR_NO_DEVICE, "load", f"{path} not built (run triton-agent_b200/build.py)")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)  # AttributeError if the symbol is missing
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(code: int) -> str:
    try:
        return load().b200_status_string(code).decode()
    except Exception:
        return "unknown status"


def check(status: int, op: str) -> None:
    if status != OK:
        detail = load().b200_last_error_detail().decode()
        raise B200OpsError(status, op, detail)


def kernel_names() -> list[str]:
    return [k for k in load().b200_kernel_list().decode().split("\n") if k]


def config_space(op: str, rows: int = 0) -> dict | None:
    """The launch parameters the kernel selected for `op` at `rows` rows
    reads, with their legal values (b200_query_config_space), or None for an
    op the library does not know."""
    import json

    txt = load().b200_query_config_space(op.encode(), int(rows))
    return json.loads(txt.decode()) if txt else None


def version() -> int:
    return load().b200_version()
