"""Torch-facing calls into libb200ops.so.

Each function takes CUDA tensors, checks shapes/dtypes/contiguity on the
host, allocates outputs with torch on the tensors' device, and launches the
kernel on the current CUDA stream through the C ABI.  There is no CPU path:
CPU tensors, a missing library or a non-sm_100 device raise.

Reference semantics each call reproduces are cited per function (paths
inside the reference project).
"""

from __future__ import annotations

import ctypes
import math
import threading

import torch

from . import lib as L

_DT = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16, torch.int8: L.I8,
       torch.int32: L.I32, torch.int64: L.I64}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise L.B200OpsError(L.ERR_UNSUPPORTED, "dtype", f"{dt} not supported") from None


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _cfg(cfg):
    if cfg is None:
        return None
    if isinstance(cfg, L.LaunchCfg):
        return ctypes.byref(cfg)
    c = L.LaunchCfg.from_dict(cfg)
    return ctypes.byref(c) if c is not None else None


def _need_cuda(op: str, *ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise L.B200OpsError(L.ERR_NO_DEVICE, op, "tensors must be on a CUDA device (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise L.B200OpsError(L.ERR_BAD_ARG, op, "tensors on different devices")
    return dev


def _contig(op: str, **ts):
    for name, t in ts.items():
        if t is not None and not t.is_contiguous():
            raise L.B200OpsError(L.ERR_BAD_ARG, op, f"{name} must be contiguous")


# --------------------------------------------------------------------- rmsnorm
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None,
            cfg=None) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2, -1) + eps) * weight  (rmsnorm/reference.py:17-18)."""
    dev = _need_cuda("rmsnorm", x, weight, out)
    _contig("rmsnorm", x=x, weight=weight, out=out)
    D = x.shape[-1]
    if weight.numel() != D:
        raise L.B200OpsError(L.ERR_BAD_ARG, "rmsnorm", "weight must have D elements")
    y = torch.empty_like(x) if out is None else out
    rows = x.numel() // D if D else 0
    st = L.load().b200_rmsnorm(_ptr(x), _ptr(weight), _ptr(y), rows, D, float(eps), dtype_code(x.dtype),
                               dtype_code(weight.dtype), _cfg(cfg), _stream(dev))
    L.check(st, "rmsnorm")
    return y


def rmsnorm_quant_int8(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, want_y: bool = False, cfg=None):
    """rmsnorm fused with the per-row INT8 quantiser of the next GEMM's
    activations (rmsnorm/reference.py:17-18 then quant_matmul/reference.py:16-19).
    Returns (q int8 [..., D], scale f32 [rows]) or (q, scale, y) with want_y."""
    dev = _need_cuda("rmsnorm_quant_int8", x, weight)
    _contig("rmsnorm_quant_int8", x=x, weight=weight)
    D = x.shape[-1]
    if weight.numel() != D:
        raise L.B200OpsError(L.ERR_BAD_ARG, "rmsnorm_quant_int8", "weight must have D elements")
    rows = x.numel() // D if D else 0
    q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    scale = torch.empty(rows, dtype=torch.float32, device=dev)
    y = torch.empty_like(x) if want_y else None
    st = L.load().b200_rmsnorm_quant_int8(_ptr(x), _ptr(weight), _ptr(q), _ptr(scale), _ptr(y), rows, D,
                                          float(eps), dtype_code(x.dtype), dtype_code(weight.dtype), _cfg(cfg),
                                          _stream(dev))
    L.check(st, "rmsnorm_quant_int8")
    return (q, scale, y) if want_y else (q, scale)


# ------------------------------------------------------------------------ RoPE
def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: torch.Tensor | None = None,
         cfg=None) -> torch.Tensor:
    """NeoX rotate-half over x [B,H,T,D] with cos/sin [T,D] (rope/reference.py:17-25)."""
    dev = _need_cuda("rope", x, cos, sin, out)
    _contig("rope", x=x, cos=cos, sin=sin, out=out)
    B, H, T, D = x.shape
    if tuple(cos.shape) != (T, D) or tuple(sin.shape) != (T, D) or cos.dtype != sin.dtype:
        raise L.B200OpsError(L.ERR_BAD_ARG, "rope", "cos/sin must be [T, D] of one dtype")
    y = torch.empty_like(x) if out is None else out
    st = L.load().b200_rope(_ptr(x), _ptr(cos), _ptr(sin), _ptr(y), B, H, T, D, dtype_code(x.dtype),
                            dtype_code(cos.dtype), _cfg(cfg), _stream(dev))
    L.check(st, "rope")
    return y


# ----------------------------------------------------------------- KV appends
def _slots64(slot_mapping: torch.Tensor) -> torch.Tensor:
    if slot_mapping.dtype != torch.int64:
        raise L.B200OpsError(L.ERR_UNSUPPORTED, "slot_mapping", "slot_mapping must be int64")
    return slot_mapping.contiguous()


def kv_append(k_cache, v_cache, k_new, v_new, slot_mapping, cfg=None):
    """In-place contiguous KV append (kv_append/reference.py:27-40).

    Caches [B,H,L,D]; new tokens [B,H,T_new,D]; slot_mapping [B,T_new] int64.
    Returns the (mutated) caches, as the reference's Triton launcher does.
    """
    dev = _need_cuda("kv_append", k_cache, v_cache, k_new, v_new, slot_mapping)
    _contig("kv_append", k_cache=k_cache, v_cache=v_cache, k_new=k_new, v_new=v_new)
    B, H, Lc, D = k_cache.shape
    T_new = k_new.shape[2]
    sm = _slots64(slot_mapping)
    st = L.load().b200_kv_append(_ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), _ptr(sm), B, H, Lc,
                                 T_new, D, dtype_code(k_cache.dtype), _cfg(cfg), _stream(dev))
    L.check(st, "kv_append")
    return k_cache, v_cache


def paged_kv(k_cache, v_cache, k_new, v_new, slot_mapping, cfg=None):
    """In-place paged KV append (paged_kv/reference.py:11-27).

    Caches [num_blocks, block_size, H, D]; new tokens [B, T_new, H, D].
    """
    dev = _need_cuda("paged_kv", k_cache, v_cache, k_new, v_new, slot_mapping)
    _contig("paged_kv", k_cache=k_cache, v_cache=v_cache, k_new=k_new, v_new=v_new)
    nb, bs, H, D = k_cache.shape
    B, T_new = k_new.shape[:2]
    sm = _slots64(slot_mapping)
    st = L.load().b200_paged_kv(_ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), _ptr(sm), B, T_new, H,
                                D, nb, bs, dtype_code(k_cache.dtype), _cfg(cfg), _stream(dev))
    L.check(st, "paged_kv")
    return k_cache, v_cache


def rope_kv_append(k_new, cos, sin, k_cache, slot_mapping, cfg=None):
    """In-place RoPE + contiguous K append (rope_kv_append/reference.py:26-47)."""
    dev = _need_cuda("rope_kv_append", k_new, cos, sin, k_cache, slot_mapping)
    _contig("rope_kv_append", k_new=k_new, cos=cos, sin=sin, k_cache=k_cache)
    B, H, T_new, D = k_new.shape
    Lc = k_cache.shape[2]
    sm = _slots64(slot_mapping)
    st = L.load().b200_rope_kv_append(_ptr(k_new), _ptr(cos), _ptr(sin), _ptr(k_cache), _ptr(sm), B, H, Lc,
                                      T_new, D, dtype_code(k_new.dtype), dtype_code(cos.dtype), _cfg(cfg),
                                      _stream(dev))
    L.check(st, "rope_kv_append")
    return k_cache


def rope_kv_append_paged(q, k, v, positions, cos, sin, slot_mapping, k_cache, v_cache,
                         q_out: torch.Tensor | None = None, cfg=None):
    """Decode step: rotate q and k by their positions, write k (rotated) and
    v into the paged caches at slot_mapping.  q [T,Hq,D] (or None), k/v
    [T,Hkv,D], positions/slot_mapping [T] int64, cos/sin [P, D] tables,
    caches [num_blocks, block_size, Hkv, D].  Returns q_out (or None)."""
    dev = _need_cuda("rope_kv_append_paged", q, k, v, positions, cos, sin, slot_mapping, k_cache, v_cache)
    _contig("rope_kv_append_paged", q=q, k=k, v=v, cos=cos, sin=sin, k_cache=k_cache, v_cache=v_cache)
    T, Hkv, D = k.shape
    Hq = q.shape[1] if q is not None else 0
    nb, bs = k_cache.shape[:2]
    if q is not None and q_out is None:
        q_out = torch.empty_like(q)
    pos = positions.contiguous() if positions is not None else None
    if pos is not None and pos.dtype != torch.int64:
        raise L.B200OpsError(L.ERR_UNSUPPORTED, "rope_kv_append_paged", "positions must be int64")
    sm = _slots64(slot_mapping)
    # many new tokens (prefill): slot-ownership table (zeroed once, restored by
    # every call) instead of each token scanning all later slots
    owner = WORKSPACES.get(dev, nb * bs * 4, "slot_owner") if T > OWNER_TABLE_MIN_TOKENS else None
    st = L.load().b200_rope_kv_append_paged_ws(_ptr(q), _ptr(k), _ptr(v), _ptr(pos), _ptr(cos), _ptr(sin),
                                               cos.shape[0], _ptr(sm), _ptr(q_out), _ptr(k_cache),
                                               _ptr(v_cache), T, Hq, Hkv, D, nb, bs, dtype_code(k.dtype),
                                               dtype_code(cos.dtype), _ptr(owner), nb * bs if owner is not None
                                               else 0, _cfg(cfg), _stream(dev))
    L.check(st, "rope_kv_append_paged")
    return q_out


OWNER_TABLE_MIN_TOKENS = 512


# -------------------------------------------------------------- paged decode
class _Workspaces:
    """Per-device zero-initialised scratch for split-KV partials.

    The decode kernel leaves its ticket counters at zero after every launch,
    so a buffer is zeroed once when it is (re)allocated and reused after.
    """

    def __init__(self):
        self._bufs: dict[tuple[int, str], torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


WORKSPACES = _Workspaces()


def paged_attention_workspace_size(B, Hq, max_blocks, block_size, D, cfg=None) -> int:
    return int(L.load().b200_paged_attention_workspace_size(B, Hq, max_blocks, block_size, D, _cfg(cfg)))


def paged_attention(q, k_cache, v_cache, block_table, context_len, scale: float | None = None,
                    out: torch.Tensor | None = None, workspace: torch.Tensor | None = None, cfg=None):
    """Paged decode attention (paged_attention/reference.py:26-52 with q[b] and
    grouped-query heads).  q [B,Hq,D]; caches [num_blocks, block_size, Hkv, D];
    block_table [B, max_blocks] and context_len [B] int32 or int64 (same
    dtype).  Returns out [B,Hq,D] in q's dtype."""
    dev = _need_cuda("paged_attention", q, k_cache, v_cache, block_table, context_len, out)
    _contig("paged_attention", q=q, k_cache=k_cache, v_cache=v_cache, block_table=block_table)
    B, Hq, D = q.shape
    nb, bs, Hkv, D2 = k_cache.shape
    if D2 != D or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise L.B200OpsError(L.ERR_BAD_ARG, "paged_attention", "cache shape mismatch")
    if block_table.dtype != context_len.dtype:
        context_len = context_len.to(block_table.dtype)
    cl = context_len.contiguous()
    max_blocks = block_table.shape[1]
    o = torch.empty_like(q) if out is None else out
    ws_bytes = paged_attention_workspace_size(B, Hq, max_blocks, bs, D, cfg)
    ws = workspace if workspace is not None else WORKSPACES.get(dev, ws_bytes, "paged_attention")
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    st = L.load().b200_paged_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table), _ptr(cl),
                                       _ptr(o), B, Hq, Hkv, D, nb, bs, max_blocks, sc, dtype_code(q.dtype),
                                       dtype_code(block_table.dtype), _ptr(ws), ws.numel(), _cfg(cfg),
                                       _stream(dev))
    L.check(st, "paged_attention")
    return o


# ----------------------------------------------------------------- INT8 GEMM
def int8_gemm(A: torch.Tensor, W: torch.Tensor, sA: torch.Tensor, sW: torch.Tensor,
              out_dtype: torch.dtype = torch.float16, out: torch.Tensor | None = None,
              acc_out: torch.Tensor | None = None, cfg=None) -> torch.Tensor:
    """C = out_dtype(float(A @ W^T) * sA[:,None] * sW[None,:]) with an exact
    int32 accumulator (quant_matmul/reference.py:26-27 on int8 codes).
    A [M,K] int8, W [N,K] int8, sA [M] f32, sW [N] f32."""
    dev = _need_cuda("int8_gemm", A, W, sA, sW, out, acc_out)
    _contig("int8_gemm", A=A, W=W, sA=sA, sW=sW)
    M, K = A.shape
    N = W.shape[0]
    if W.shape[1] != K or A.dtype != torch.int8 or W.dtype != torch.int8:
        raise L.B200OpsError(L.ERR_BAD_ARG, "int8_gemm", "A [M,K] and W [N,K] must be int8")
    if sA.dtype != torch.float32 or sW.dtype != torch.float32:
        raise L.B200OpsError(L.ERR_BAD_ARG, "int8_gemm", "scales must be float32")
    C = torch.empty(M, N, dtype=out_dtype, device=dev) if out is None else out
    ldc = C.stride(0)
    ws_bytes = int(L.load().b200_int8_gemm_workspace_size(M, N, K, _cfg(cfg)))
    ws = WORKSPACES.get(dev, ws_bytes, "int8_gemm") if ws_bytes else None
    st = L.load().b200_int8_gemm(_ptr(A), _ptr(W), _ptr(sA), _ptr(sW), _ptr(C), M, N, K, ldc,
                                 dtype_code(out_dtype), _ptr(acc_out), _ptr(ws), ws.numel() if ws is not None else 0,
                                 _cfg(cfg), _stream(dev))
    L.check(st, "int8_gemm")
    return C


def gemm_bias_gelu(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor, out: torch.Tensor | None = None,
                   cfg=None) -> torch.Tensor:
    """gelu_tanh(a @ b + bias) (matmul_epilogue/reference.py:6-18): a [..., M, K],
    b [K, N], bias [N], fp16 or bf16; fp32 accumulation and epilogue."""
    dev = _need_cuda("gemm_bias_gelu", a, b, bias, out)
    _contig("gemm_bias_gelu", a=a, b=b, bias=bias, out=out)
    K = a.shape[-1]
    if b.dim() != 2 or b.shape[0] != K or bias.numel() != b.shape[1] or not (a.dtype == b.dtype == bias.dtype):
        raise L.B200OpsError(L.ERR_BAD_ARG, "gemm_bias_gelu", "a [..., M, K], b [K, N], bias [N] of one dtype")
    N = b.shape[1]
    M = a.numel() // K if K else 0
    c = torch.empty(*a.shape[:-1], N, dtype=a.dtype, device=dev) if out is None else out
    st = L.load().b200_gemm_bias_gelu(_ptr(a), _ptr(b), _ptr(bias), _ptr(c), M, N, K, dtype_code(a.dtype),
                                      _cfg(cfg), _stream(dev))
    L.check(st, "gemm_bias_gelu")
    return c


def quantize_int8(x: torch.Tensor, by_column: bool = False, cfg=None):
    """Per-row (or per-column, transposed) symmetric int8 quantisation
    (quant_matmul/reference.py:16-24).  Returns (q int8, scale f32)."""
    dev = _need_cuda("quantize_int8", x)
    _contig("quantize_int8", x=x)
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    if by_column:
        q = torch.empty(cols, rows, dtype=torch.int8, device=dev)
        s = torch.empty(cols, dtype=torch.float32, device=dev)
    else:
        q = torch.empty(rows, cols, dtype=torch.int8, device=dev)
        s = torch.empty(rows, dtype=torch.float32, device=dev)
    st = L.load().b200_quantize_int8(_ptr(x), _ptr(q), _ptr(s), rows, cols, dtype_code(x.dtype),
                                     1 if by_column else 0, _cfg(cfg), _stream(dev))
    L.check(st, "quantize_int8")
    return q, s


# ------------------------------------------------------------ flash attention
def flash_attn(q, k, v, causal: bool = False, scale: float | None = None, out=None, lse=None, cfg=None):
    """softmax(q k^T * scale [+ causal mask]) v (flash_attn_like/reference.py:22-31).
    q [B,H,T,D], k/v [B,H,S,D]; returns [B,H,T,D] in q's dtype."""
    dev = _need_cuda("flash_attn", q, k, v, out, lse)
    _contig("flash_attn", q=q, k=k, v=v)
    B, H, T, D = q.shape
    S = k.shape[2]
    if causal and T != S:
        raise L.B200OpsError(L.ERR_BAD_ARG, "flash_attn", "causal requires T == S (reference.py:25-28)")
    o = torch.empty_like(q) if out is None else out
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    st = L.load().b200_flash_attn(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, H, T, S, D, sc,
                                  1 if causal else 0, dtype_code(q.dtype), _cfg(cfg), _stream(dev))
    L.check(st, "flash_attn")
    return o


# device error word codes (first failure wins)
DEV_ERR_TIMEOUT_FULL, DEV_ERR_TIMEOUT_EMPTY, DEV_ERR_TIMEOUT_MMA, DEV_ERR_TIMEOUT_COMBINE = 1, 2, 3, 4
DEV_ERR_TIMEOUT_PEER = 6


def set_peer_wait_timeout_us(us: int) -> None:
    """Limit of the cross-GPU flag waits of the fused all-gather GEMM (0 = 2 s)."""
    L.check(L.load().b200_set_peer_wait_timeout_us(int(us)), "set_peer_wait_timeout_us")


def read_device_error(device: torch.device | None = None) -> int:
    """Device error word set by bounded waits that gave up (0 = none; codes above)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    v = ctypes.c_int32(0)
    L.check(L.load().b200_read_device_error(ctypes.byref(v), _stream(dev)), "read_device_error")
    return int(v.value)
