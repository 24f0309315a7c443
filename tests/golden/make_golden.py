"""Generates tests/golden/*.pt by running the reference project's own PyTorch
operator references on small seeded inputs.

Usage (in a container that has the reference checked out):
    python tests/golden/make_golden.py --ref <reference checkout>
    (or set TRITON_AGENT_REF to the checkout and omit --ref)

Each reference.py is imported by file path (they depend only on torch and
math), so no part of the reference package is installed or copied.  The
fixtures hold the inputs and the reference outputs; tests/test_oracle_golden.py
checks the oracle restatements against them.  The fixtures are committed so
that the GPU-side tests never need the reference.

paged_attention's reference indexes the query as q[b:b+1] and then fails in
its einsum (reference.py:50).  It is run here unmodified with the query
wrapped in a tensor subclass whose one-element slice q[b:b+1] yields q[b], so
every other line of the reference (block walk, invalid-id skip, truncation,
softmax) executes as written.
"""

from __future__ import annotations

import argparse
import os
import importlib.util
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def load_ref(ref_root: Path, op: str):
    path = ref_root / "triton_agent" / "ops" / op / "reference.py"
    spec = importlib.util.spec_from_file_location(f"_golden_ref_{op}", str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _RowQuery(torch.Tensor):
    """q whose single-row slice q[b:b+1] returns q[b] (see module docstring)."""

    def __getitem__(self, idx):
        base = self.as_subclass(torch.Tensor)
        if isinstance(idx, slice) and idx.step is None and idx.start is not None and idx.stop == idx.start + 1:
            return base[idx.start]
        return base[idx]


def gen(seed: int):
    g = torch.Generator().manual_seed(seed)
    return g


def make(ref_root: Path) -> None:
    out = {}

    # ---- rmsnorm (rmsnorm/reference.py:6-18)
    m = load_ref(ref_root, "rmsnorm")
    cases = []
    for i, (shape, dt) in enumerate([((2, 3, 256), torch.float32), ((1, 2, 4096), torch.float32),
                                     ((2, 3, 256), torch.bfloat16), ((2, 3, 256), torch.float16),
                                     ((3, 1, 100), torch.float32)]):
        g = gen(100 + i)
        x = torch.randn(*shape, generator=g).to(dt)
        w = (1.0 + 0.1 * torch.randn(shape[-1], generator=g)).to(dt)
        cases.append({"x": x, "w": w, "eps": 1e-6, "y": m.rmsnorm(x, w, 1e-6)})
    x = torch.zeros(1, 1, 64)
    w = torch.ones(64)
    cases.append({"x": x, "w": w, "eps": 1e-6, "y": m.rmsnorm(x, w, 1e-6)})
    out["rmsnorm"] = cases

    # ---- rope (rope/reference.py:6-25)
    m = load_ref(ref_root, "rope")
    cases = []
    for i, (shape, dt) in enumerate([((1, 2, 3, 64), torch.float32), ((2, 2, 4, 128), torch.float32),
                                     ((2, 2, 4, 128), torch.bfloat16)]):
        g = gen(200 + i)
        x = torch.randn(*shape, generator=g).to(dt)
        cos = torch.randn(shape[2], shape[3], generator=g).to(dt)
        sin = torch.randn(shape[2], shape[3], generator=g).to(dt)
        cases.append({"x": x, "cos": cos, "sin": sin, "y": m.rope(x, cos, sin)})
    out["rope"] = cases

    # ---- kv_append (kv_append/reference.py:10-40), including duplicate and
    # out-of-range slots
    m = load_ref(ref_root, "kv_append")
    cases = []
    for i, (B, H, L, T_new, D, dt) in enumerate([(1, 1, 32, 1, 64, torch.float32),
                                                 (2, 2, 16, 8, 16, torch.float32),
                                                 (2, 3, 16, 4, 32, torch.bfloat16)]):
        g = gen(300 + i)
        kc = torch.randn(B, H, L, D, generator=g).to(dt)
        vc = torch.randn(B, H, L, D, generator=g).to(dt)
        kn = torch.randn(B, H, T_new, D, generator=g).to(dt)
        vn = torch.randn(B, H, T_new, D, generator=g).to(dt)
        sm = torch.randint(-2, L + 2, (B, T_new), generator=g)
        if T_new > 1:
            sm[0, -1] = sm[0, 0]  # duplicate slot: the later token wins
        ko, vo = m.kv_append(kc, vc, kn, vn, sm)
        cases.append({"k_cache": kc, "v_cache": vc, "k_new": kn, "v_new": vn, "slot_mapping": sm,
                      "k_out": ko, "v_out": vo})
    out["kv_append"] = cases

    # ---- paged_kv (paged_kv/reference.py:6-27)
    m = load_ref(ref_root, "paged_kv")
    cases = []
    for i, (B, T_new, H, nb, bs, D, dt) in enumerate([(2, 3, 2, 8, 4, 16, torch.float32),
                                                      (3, 2, 4, 6, 16, 32, torch.bfloat16)]):
        g = gen(400 + i)
        kc = torch.randn(nb, bs, H, D, generator=g).to(dt)
        vc = torch.randn(nb, bs, H, D, generator=g).to(dt)
        kn = torch.randn(B, T_new, H, D, generator=g).to(dt)
        vn = torch.randn(B, T_new, H, D, generator=g).to(dt)
        sm = torch.randint(-3, nb * bs + 3, (B, T_new), generator=g)
        sm[1, 0] = sm[0, 0]  # duplicate global slot across sequences
        ko, vo = m.paged_kv(kc, vc, kn, vn, sm)
        cases.append({"k_cache": kc, "v_cache": vc, "k_new": kn, "v_new": vn, "slot_mapping": sm,
                      "k_out": ko, "v_out": vo})
    out["paged_kv"] = cases

    # ---- rope_kv_append (rope_kv_append/reference.py:10-47)
    m = load_ref(ref_root, "rope_kv_append")
    cases = []
    for i, (B, H, L, T_new, D, dt) in enumerate([(2, 2, 8, 3, 16, torch.float32),
                                                 (1, 4, 16, 2, 64, torch.float32)]):
        g = gen(500 + i)
        kn = torch.randn(B, H, T_new, D, generator=g).to(dt)
        cos = torch.randn(T_new, D, generator=g).to(dt)
        sin = torch.randn(T_new, D, generator=g).to(dt)
        kc = torch.randn(B, H, L, D, generator=g).to(dt)
        sm = torch.randint(-1, L + 1, (B, T_new), generator=g)
        ko = m.rope_kv_append(kn, cos, sin, kc, sm)
        cases.append({"k_new": kn, "cos": cos, "sin": sin, "k_cache": kc, "slot_mapping": sm,
                      "k_out": ko})
    out["rope_kv_append"] = cases

    # ---- paged_attention (paged_attention/reference.py:10-54) via _RowQuery
    m = load_ref(ref_root, "paged_attention")
    cases = []
    for i, (B, H, D, nb, bs, maxb, ctxs, bad) in enumerate([
        (2, 2, 32, 12, 4, 5, [7, 16], False),
        (3, 4, 32, 10, 16, 3, [1, 33, 48], False),
        (2, 2, 32, 10, 4, 6, [13, 20], True),  # invalid block ids in the table
    ]):
        g = gen(600 + i)
        q = torch.randn(B, H, D, generator=g)
        kc = torch.randn(nb, bs, H, D, generator=g)
        vc = torch.randn(nb, bs, H, D, generator=g)
        bt = torch.randint(0, nb, (B, maxb), generator=g)
        if bad:
            bt[0, 1] = -1
            bt[1, 0] = nb + 3
        cl = torch.tensor(ctxs, dtype=torch.long)
        o = m.paged_attention(q.as_subclass(_RowQuery), kc, vc, bt, cl).as_subclass(torch.Tensor)
        cases.append({"q": q, "k_cache": kc, "v_cache": vc, "block_table": bt, "context_len": cl,
                      "out": o.clone()})
    out["paged_attention"] = cases

    # ---- quant_matmul (quant_matmul/reference.py:6-28)
    m = load_ref(ref_root, "quant_matmul")
    cases = []
    for i, (B, M, K, N, dt) in enumerate([(2, 8, 64, 16, torch.float32), (1, 5, 128, 24, torch.float16),
                                          (1, 4, 32, 8, torch.float32)]):
        g = gen(700 + i)
        a = torch.randn(B, M, K, generator=g).to(dt)
        b = torch.randn(K, N, generator=g).to(dt)
        if i == 2:
            a[0, 1] = 0.0  # zero row -> scale replaced by 1e-6
            b[:, 3] = 0.0  # zero column
        cases.append({"a": a, "b": b, "c": m.quant_matmul(a, b)})
    out["quant_matmul"] = cases

    # ---- flash_attn_like (flash_attn_like/reference.py:7-31)
    m = load_ref(ref_root, "flash_attn_like")
    cases = []
    for i, (B, H, T, S, D, causal) in enumerate([(1, 1, 1, 1, 64, False), (1, 2, 16, 16, 32, False),
                                                 (2, 2, 24, 24, 32, True), (1, 1, 8, 12, 16, False)]):
        g = gen(800 + i)
        q = torch.randn(B, H, T, D, generator=g)
        k = torch.randn(B, H, S, D, generator=g)
        v = torch.randn(B, H, S, D, generator=g)
        cases.append({"q": q, "k": k, "v": v, "causal": causal, "out": m.flash_attn_like(q, k, v, causal)})
    out["flash_attn_like"] = cases

    for op, cs in out.items():
        torch.save(cs, HERE / f"{op}.pt")
        print(f"{op}: {len(cs)} cases")


def main() -> None:
    ap = argparse.ArgumentParser()
    env = os.environ.get("TRITON_AGENT_REF")
    ap.add_argument("--ref", default=env, required=env is None,
                    help="root of a Triton-Agent checkout (default: $TRITON_AGENT_REF)")
    args = ap.parse_args()
    make(Path(args.ref))


if __name__ == "__main__":
    main()
