"""CPU restatements of the reference operator math -- the oracle (test-only).

Every function names the reference lines it follows (paths inside the
reference project).  Floating-point work is done in fp32 with each product
and sum rounded separately (as eager PyTorch on the CPU evaluates the
reference formulas) and rounded once to the output dtype; integer work
(int8 GEMM accumulators, slot arithmetic) is exact in int64.
"""

from __future__ import annotations

import math

import numpy as np
import torch

__all__ = [
    "rmsnorm",
    "rope",
    "rope_cos_sin",
    "kv_append",
    "paged_kv",
    "rope_kv_append",
    "rope_kv_append_paged",
    "paged_attention",
    "quantize_int8",
    "int8_gemm_acc",
    "dequant",
    "quant_matmul",
    "flash_attn",
]


# --------------------------------------------------------------------- rmsnorm
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """triton_agent/ops/rmsnorm/reference.py:17-18, evaluated in fp32.

    rstd = rsqrt(mean(x^2, -1) + eps); y = x * rstd * w, cast to x.dtype.
    """
    xf = x.detach().to("cpu", torch.float32)
    wf = weight.detach().to("cpu", torch.float32)
    rstd = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * rstd * wf).to(x.dtype)


# ------------------------------------------------------------------------ RoPE
def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """NeoX rotate-half, triton_agent/ops/rope/reference.py:17-25 (fp32).

    x1 = x[..., :D/2], x2 = x[..., D/2:], c/s = cos/sin[..., :D/2];
    y1 = x1*c - x2*s, y2 = x2*c + x1*s.  Each product and sum is its own
    fp32 rounding (eager tensor ops), which the CUDA kernels reproduce with
    explicitly rounded multiplies and adds.
    """
    D = x.shape[-1]
    h = D // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = cos[..., :h], sin[..., :h]
    y1 = (x1 * c) - (x2 * s)
    y2 = (x2 * c) + (x1 * s)
    return torch.cat([y1, y2], dim=-1)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """triton_agent/ops/rope/reference.py:6-25.  x [B,H,T,D], cos/sin [T,D]."""
    xf = x.detach().to("cpu", torch.float32)
    return _rotate(xf, cos.detach().to("cpu", torch.float32), sin.detach().to("cpu", torch.float32)).to(x.dtype)


def rope_cos_sin(max_pos: int, D: int, theta: float = 1e4) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin tables [max_pos, D] for RoPE with base `theta`.

    The reference takes cos/sin as inputs (rope/reference.py:11-12) and uses
    their first D/2 columns.  For a decode step at integer positions they are
    inv_freq_j = theta^(-2j/D), angle = pos * inv_freq_j (j < D/2); the
    second half repeats the first (the NeoX layout), so either convention of
    "first half used" reads the same values.
    """
    j = torch.arange(0, D, 2, dtype=torch.float32)
    inv_freq = 1.0 / (theta ** (j / D))
    pos = torch.arange(max_pos, dtype=torch.float32)
    ang = torch.outer(pos, inv_freq)
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1)
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1)
    return cos.contiguous(), sin.contiguous()


# ----------------------------------------------------------------- KV appends
def _last_writer_mask(keys: np.ndarray, valid: np.ndarray) -> np.ndarray:
    """True for the entries whose destination is not written again later.

    The reference loops b outer, t inner and overwrites in order
    (kv_append/reference.py:33-38), so the last (b, t) naming a row wins.
    """
    n = keys.shape[0]
    keep = np.zeros(n, dtype=bool)
    idx = np.nonzero(valid)[0]
    if idx.size == 0:
        return keep
    rev = idx[::-1]
    _, first_in_rev = np.unique(keys[rev], return_index=True)
    keep[rev[first_in_rev]] = True
    return keep


def kv_append(k_cache, v_cache, k_new, v_new, slot_mapping):
    """triton_agent/ops/kv_append/reference.py:27-40.

    Caches [B,H,L,D], new tokens [B,H,T_new,D], slot_mapping [B,T_new];
    rows with slot outside [0, L) are skipped.  Returns updated copies.
    """
    B, H, L, D = k_cache.shape
    T_new = k_new.shape[2]
    k_out = k_cache.detach().cpu().clone()
    v_out = v_cache.detach().cpu().clone()
    slots = slot_mapping.detach().cpu().numpy().astype(np.int64).reshape(B * T_new)
    bidx = np.repeat(np.arange(B), T_new)
    tidx = np.tile(np.arange(T_new), B)
    valid = (slots >= 0) & (slots < L)
    keep = _last_writer_mask(bidx * L + slots, valid)
    kn, vn = k_new.detach().cpu(), v_new.detach().cpu()
    for i in np.nonzero(keep)[0]:
        b, t, s = int(bidx[i]), int(tidx[i]), int(slots[i])
        k_out[b, :, s, :] = kn[b, :, t, :]
        v_out[b, :, s, :] = vn[b, :, t, :]
    return k_out, v_out


def paged_kv(k_cache, v_cache, k_new, v_new, slot_mapping):
    """triton_agent/ops/paged_kv/reference.py:11-27.

    Caches [num_blocks, block_size, H, D]; new tokens [B, T_new, H, D];
    block = slot // block_size, offset = slot % block_size (floor division),
    rows whose block is outside [0, num_blocks) are skipped.
    """
    nb, bs, H, D = k_cache.shape
    B, T_new = k_new.shape[:2]
    k_out = k_cache.detach().cpu().clone()
    v_out = v_cache.detach().cpu().clone()
    slots = slot_mapping.detach().cpu().numpy().astype(np.int64).reshape(B * T_new)
    blk = np.floor_divide(slots, bs)
    off = np.mod(slots, bs)
    valid = (blk >= 0) & (blk < nb)
    keep = _last_writer_mask(slots, valid)
    kn = k_new.detach().cpu().reshape(B * T_new, H, D)
    vn = v_new.detach().cpu().reshape(B * T_new, H, D)
    sel = np.nonzero(keep)[0]
    if sel.size:
        ti = torch.from_numpy(sel)
        k_out[torch.from_numpy(blk[sel]), torch.from_numpy(off[sel])] = kn[ti]
        v_out[torch.from_numpy(blk[sel]), torch.from_numpy(off[sel])] = vn[ti]
    return k_out, v_out


def rope_kv_append(k_new, cos, sin, k_cache, slot_mapping):
    """triton_agent/ops/rope_kv_append/reference.py:26-47 (rotation in fp32)."""
    B, H, T_new, D = k_new.shape
    L = k_cache.shape[2]
    k_rot = _rotate(k_new.detach().cpu().float(), cos.detach().cpu().float(), sin.detach().cpu().float())
    k_rot = k_rot.to(k_new.dtype)
    k_out = k_cache.detach().cpu().clone()
    slots = slot_mapping.detach().cpu().numpy().astype(np.int64).reshape(B * T_new)
    bidx = np.repeat(np.arange(B), T_new)
    tidx = np.tile(np.arange(T_new), B)
    valid = (slots >= 0) & (slots < L)
    keep = _last_writer_mask(bidx * L + slots, valid)
    for i in np.nonzero(keep)[0]:
        b, t, s = int(bidx[i]), int(tidx[i]), int(slots[i])
        k_out[b, :, s, :] = k_rot[b, :, t, :]
    return k_out


def rope_kv_append_paged(q, k, v, positions, cos, sin, slot_mapping, num_slots: int):
    """Decode-step RoPE(q, k) + paged K/V append, as rows.

    Composition of rope/reference.py:17-25 (rotation of q and of new k),
    rope_kv_append/reference.py:33-35 (k rotated before it is stored) and
    paged_kv/reference.py:18-25 (slot -> block/offset, invalid slots skipped,
    last writer wins).  q [T,Hq,D], k/v [T,Hkv,D], positions [T] (row into the
    cos/sin tables), slot_mapping [T].

    Returns (q_out, k_rows, v_rows, keep) where k_rows/v_rows [T,Hkv,D] are
    what lands in the cache at slot_mapping[t] for every t with keep[t].
    """
    pos = positions.detach().cpu().long()
    c = cos.detach().cpu().float()[pos].unsqueeze(1)  # [T,1,D]
    s = sin.detach().cpu().float()[pos].unsqueeze(1)
    q_out = _rotate(q.detach().cpu().float(), c, s).to(q.dtype) if q is not None else None
    k_rows = _rotate(k.detach().cpu().float(), c, s).to(k.dtype)
    v_rows = v.detach().cpu().clone()
    slots = slot_mapping.detach().cpu().numpy().astype(np.int64).reshape(-1)
    valid = (slots >= 0) & (slots < num_slots)
    keep = _last_writer_mask(slots, valid)
    return q_out, k_rows, v_rows, torch.from_numpy(keep)


# -------------------------------------------------------------- paged decode
def gather_pages(k_cache, v_cache, block_table_row, ctx: int):
    """Token rows a sequence attends to, per paged_attention/reference.py:32-48.

    Walks the first ceil(ctx/bs) table entries, drops ids outside
    [0, num_blocks) (:40-41), concatenates the kept blocks and truncates to
    ctx tokens (:47-48).  Returns K, V as [n_tok, Hkv, D] (n_tok may be < ctx
    when blocks were dropped).
    """
    nb, bs = k_cache.shape[:2]
    nvb = (ctx + bs - 1) // bs
    ids = [int(i) for i in block_table_row[:nvb].tolist()]
    ids = [i for i in ids if 0 <= i < nb]
    if not ids:
        return None, None
    idx = torch.tensor(ids, dtype=torch.long)
    K = k_cache[idx].reshape(-1, *k_cache.shape[2:])[:ctx]
    V = v_cache[idx].reshape(-1, *v_cache.shape[2:])[:ctx]
    return K, V


def paged_attention(q, k_cache, v_cache, block_table, context_len, scale: float | None = None):
    """paged_attention/reference.py:26-52, restated with q[b] (the reference's
    q[b:b+1] at :50 makes its einsum fail) and grouped-query heads: query
    head h reads kv head h // (Hq // Hkv) (reduces to the reference when
    Hq == Hkv).  fp32 throughout; returns fp32 [B, Hq, D].  A sequence with no
    surviving token gives a zero row (the reference raises there).
    """
    B, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    G = Hq // Hkv
    if scale is None or scale <= 0:
        scale = 1.0 / math.sqrt(D)
    qf = q.detach().cpu().float()
    kc = k_cache.detach().cpu()
    vc = v_cache.detach().cpu()
    bt = block_table.detach().cpu()
    cl = context_len.detach().cpu()
    out = torch.zeros(B, Hq, D, dtype=torch.float32)
    for b in range(B):
        ctx = int(cl[b])
        if ctx <= 0:
            continue
        K, V = gather_pages(kc, vc, bt[b], ctx)
        if K is None:
            continue
        Kf = K.float().permute(1, 0, 2)  # [Hkv, n, D]
        Vf = V.float().permute(1, 0, 2)
        Kf = Kf.repeat_interleave(G, dim=0)
        Vf = Vf.repeat_interleave(G, dim=0)
        scores = torch.einsum("hd,hld->hl", qf[b], Kf) * scale
        attn = torch.softmax(scores, dim=-1)
        out[b] = torch.einsum("hl,hld->hd", attn, Vf)
    return out


# ---------------------------------------------------------------- INT8 GEMM
def quantize_int8(x: torch.Tensor, by_column: bool = False):
    """triton_agent/ops/quant_matmul/reference.py:16-24.

    scale = max|x| / 127 along the row (columns when by_column), in x's dtype,
    zero scales replaced by 1e-6; q = clamp(round(x / scale), -127, 127) with
    round-half-even and the division rounded to x's dtype, as eager PyTorch
    does.  Returns (q int8, scale in x.dtype).  Column mode returns q
    transposed, [cols, rows] (the K-major weight layout).
    """
    x = x.detach().cpu()
    dim = 0 if by_column else -1
    amax = x.abs().amax(dim=dim, keepdim=True)
    scale = amax / 127.0
    scale[scale == 0] = 1e-6
    qv = (x / scale).round().clamp(-127, 127).to(torch.int8)
    if by_column:
        return qv.t().contiguous(), scale.reshape(-1)
    return qv, scale.reshape(-1)


def int8_gemm_acc(A: torch.Tensor, W: torch.Tensor) -> np.ndarray:
    """Exact int8 x int8 -> integer accumulators: acc[m,n] = sum_k A[m,k] W[n,k].

    Replaces the reference's float matmul of int8 codes
    (quant_matmul/reference.py:26), which is exact only while every partial
    sum stays below 2^24; here the accumulation is exact in int64.
    """
    a = A.detach().cpu().numpy().astype(np.int64)
    w = W.detach().cpu().numpy().astype(np.int64)
    return a @ w.T


def dequant(acc: np.ndarray, sA: torch.Tensor, sW: torch.Tensor, out_dtype=torch.float16) -> torch.Tensor:
    """quant_matmul/reference.py:27: c = acc * a_scale * b_scale, in fp32
    (acc converted to fp32 first, then the two multiplies rounded in
    order), cast once to out_dtype."""
    accf = torch.from_numpy(acc.astype(np.float32))
    c = accf * sA.detach().cpu().float().reshape(-1, 1)
    c = c * sW.detach().cpu().float().reshape(1, -1)
    return c.to(out_dtype)


def quant_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """quant_matmul/reference.py:6-28 end to end (a [..., M, K], b [K, N]);
    returns fp32 [..., M, N] like the reference, with an exact integer GEMM."""
    lead = a.shape[:-2]
    M, K = a.shape[-2:]
    N = b.shape[1]
    a2 = a.detach().cpu().reshape(-1, K)
    qa, sa = quantize_int8(a2)
    qb, sb = quantize_int8(b.detach().cpu(), by_column=True)  # qb [N, K]
    acc = int8_gemm_acc(qa, qb)
    c = dequant(acc, sa.float(), sb.float(), torch.float32)
    return c.reshape(*lead, M, N)


# ------------------------------------------------------------ flash attention
def flash_attn(q, k, v, causal: bool = False, rows: slice | None = None, chunk: int = 1024):
    """flash_attn_like/reference.py:22-31 in fp32, chunked over query rows.

    scores = q k^T / sqrt(D); with causal, key s > query t is masked (the
    reference's tril mask assumes T == S); softmax; @ v.  `rows` limits the
    computation to a slice of the flattened (b, h) pairs.  Returns fp32.
    """
    B, H, T, D = q.shape
    S = k.shape[2]
    if causal and T != S:
        raise ValueError("causal mask requires T == S (reference.py:25-28)")
    scale = 1.0 / math.sqrt(D)
    qf = q.detach().cpu().reshape(B * H, T, D)
    kf = k.detach().cpu().reshape(B * H, S, D)
    vf = v.detach().cpu().reshape(B * H, S, D)
    sel = range(B * H)[rows] if rows is not None else range(B * H)
    out = torch.zeros(len(sel), T, D, dtype=torch.float32)
    for oi, bh in enumerate(sel):
        kb = kf[bh].float()
        vb = vf[bh].float()
        for t0 in range(0, T, chunk):
            t1 = min(T, t0 + chunk)
            sc = (qf[bh, t0:t1].float() @ kb.t()) * scale
            if causal:
                tt = torch.arange(t0, t1).unsqueeze(1)
                ss = torch.arange(S).unsqueeze(0)
                sc = sc.masked_fill(ss > tt, float("-inf"))
            out[oi, t0:t1] = torch.softmax(sc, dim=-1) @ vb
    if rows is None:
        return out.reshape(B, H, T, D)
    return out


# ---------------------------------------------------------- rmsnorm + quant
def rmsnorm_quant_int8(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """rmsnorm (triton_agent/ops/rmsnorm/reference.py:17-18, fp32, cast to
    x's dtype) followed by the row quantiser of
    triton_agent/ops/quant_matmul/reference.py:16-19.  Returns (q int8,
    scale in x's dtype [rows, 1])."""
    y = rmsnorm(x, weight, eps)
    return quantize_int8(y.reshape(-1, y.shape[-1]))


# --------------------------------------------------------- matmul epilogue
def matmul_epilogue(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """triton_agent/ops/matmul_epilogue/reference.py:6-18 in fp32:
    c = a @ b + bias; 0.5 c (1 + tanh(0.7978845608028654 (c + 0.044715 c^3)))."""
    c = a.detach().cpu().float() @ b.detach().cpu().float() + bias.detach().cpu().float()
    return 0.5 * c * (1.0 + torch.tanh(0.7978845608028654 * (c + 0.044715 * c.pow(3))))
