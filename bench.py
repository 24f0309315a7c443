"""Benchmark of the paged-decode hot path on B200 (one JSON line on rank 0).

A step is one decode step of 64 sequences per GPU (a global batch of 64 x N
sequences sharded by KV bytes, each rank owning its share's pages):
  1. fused RoPE(q, k) + paged K/V append of the step's 64 new tokens
     (32 q / 8 kv heads, head dim 128, bf16, 65536 x 16-token cache blocks),
  2. paged-attention decode over context lengths ~ U[512, 8192]
     (GQA 4:1, random block tables, fp32 softmax).
`value` is decoded tokens per second summed over all ranks (weak scaling:
each rank owns its own 64 sequences and its own KV pages, no collective on
the data path).  The KV cache (4 GiB) is far larger than L2, so no flush is
needed between steps.

Usage:
  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
  (N > 1: launch with torchrun, one rank per GPU)
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "triton-agent_b200"))

import torch  # noqa: E402

METRIC = "paged-decode tokens/s"
# DRAM bytes (read + write) per algorithmic byte of the paged-decode kernel,
# from one ncu capture of `bench.py --case decode` (16384-block cache, 64
# sequences, ctx U[512,4096]):
# 609.92 MB of DRAM traffic for the launch's algorithmic bytes.  The full
# launch (ctx U[512,8192], 65536 blocks) is too large for a full-set capture;
# its traffic is this ratio times its algorithmic bytes (both grow with the
# pages read).
DECODE_DRAM_BYTES_SMALL = 604_623_872 + 5_299_712
DECODE_ALGO_BYTES_SMALL = 601_964_708  # printed by the same `bench.py --case decode` run
UNIT = "tokens/s"
# the decode follows the append on one stream and neither writes the other's
# context lengths / block tables: programmatic dependent launch lets the
# decode's prologue overlap the append's tail (b200_paged_attention cfg flags bit 3)
DECODE_CFG = {"flags": 8}
N_SEQ, HQ, HKV, D, BS, NBLK = 64, 32, 8, 128, 16, 65536
WORKLOAD = {
    "workload": "decode step: fused RoPE+paged KV append (64 tok) then paged-attention decode",
    "seqs_per_gpu": N_SEQ, "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "block_size": BS,
    "num_blocks": NBLK, "context_len": "U[512,8192]", "dtype": "bf16", "rope_theta": 1e4,
    "l2": "inputs larger than L2 (4 GiB KV cache per GPU), no flush",
}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, local):
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        return dist
    return None


def max_over_ranks(dist, v: float, device) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_per_rank(dist, device, ws, **vals) -> dict:
    """Each named figure from every rank (rank order), with its max/min
    spread: which rank limits a weak-scaled step and whether its clock did."""
    if dist is None or ws == 1:
        return {k: [v] for k, v in vals.items()}
    t = torch.tensor([float(v) for v in vals.values()], dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(ws)]
    dist.all_gather(out, t)
    cols = torch.stack(out).cpu()
    res = {}
    for i, k in enumerate(vals):
        col = [float(x) for x in cols[:, i]]
        res[k] = col
        if min(col) > 0:
            res[f"{k}_spread"] = max(col) / min(col)
    return res


def barrier(dist):
    if dist is not None:
        dist.barrier()


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"b200_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        try:
            self.path.unlink()
        except Exception:
            pass
        loaded = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def _median_us(fn, warmup=3, repeat=20, flush_l2=False):
    from b200ops.core.profiler import time_device

    lat = sorted(time_device(fn, warmup, repeat, flush_l2=flush_l2))
    return lat[len(lat) // 2]


def secondary_ops(dev) -> dict:
    """The other operators of the hot path, each timed alone with CUDA events
    on the current stream (medians of 20; L2 written over and read back
    before each timed call): INT8 GEMM (the metric's second
    part), causal flash prefill, rmsnorm.  INT8 peak: no measured INT8 figure
    exists for this pool, so the fraction is against 2x the measured dense
    bf16 GEMM (the tensor core's int8:bf16 rate is 2:1) and cuBLAS int8 is
    timed beside it on the same shapes."""
    from b200ops import workloads as WL
    from b200ops.runtime import ops as K

    peaks = measured_peaks()
    int8_peak = 2 * peaks["bf16_tflops"]
    res = {}
    for M, N in ((4096, 14336), (4096, 4096), (16, 14336)):
        A, W, sA, sW = WL.int8_gemm_inputs(M, N, 4096, device=dev)
        C = torch.empty(M, N, dtype=torch.float16, device=dev)
        us = _median_us(lambda: K.int8_gemm(A, W, sA, sW, out=C), flush_l2=True)
        ops = 2 * M * N * 4096
        entry = {"us": us, "TOPS": ops / us / 1e6, "peak_TOPS": int8_peak, "frac": ops / us / 1e6 / int8_peak,
                 "peak_src": f"2x {peaks['src']} bf16"}
        if M == 16:
            nbytes = N * 4096 + M * 4096 + 4 * (M + N) + 2 * M * N
            entry.update({"bound": "hbm", "GBps": nbytes / us / 1e3, "hbm_frac": nbytes / us / 1e3 / peaks["hbm_gbs"]})
        else:
            try:
                cu = _median_us(lambda: torch._int_mm(A, W.t()), flush_l2=True)
                entry["cublas_int_mm_TOPS"] = ops / cu / 1e6
            except Exception as e:  # cuBLAS int8 needs M > 16
                entry["cublas_int_mm_TOPS"] = None
        res[f"int8_gemm_M{M}_N{N}_K4096"] = entry
    q, k, v = WL.flash_inputs(device=dev)
    us = _median_us(lambda: K.flash_attn(q, k, v, causal=True), 2, 10)
    fl = WL.causal_flops(4, 32, 4096, 128)
    res["flash_prefill_causal_B4_H32_T4096_D128"] = {"us": us, "TFLOPs": fl / us / 1e6,
                                                     "frac": fl / us / 1e6 / peaks["bf16_tflops"]}
    try:  # the library comparator: PyTorch's fused attention (its best available backend)
        us_sdpa = _median_us(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True), 2, 10)
        res["flash_prefill_causal_B4_H32_T4096_D128"]["torch_sdpa_TFLOPs"] = fl / us_sdpa / 1e6
    except Exception:
        pass
    x, w = WL.rmsnorm_inputs(device=dev)
    y = torch.empty_like(x)
    us = _median_us(lambda: K.rmsnorm(x, w, out=y), flush_l2=True)
    nb = 2 * x.numel() * 4 + 4096 * 4
    res["rmsnorm_fp32_8x2048x4096"] = {"us": us, "GBps": nb / us / 1e3, "frac": nb / us / 1e3 / peaks["hbm_gbs"]}
    # matmul_epilogue: fp16 [8*256, 4096] x [4096, 4096] + bias, GELU
    g = torch.Generator(device=dev).manual_seed(11)
    a_e = (torch.randn(8 * 256, 4096, generator=g, device=dev) / 8).half()
    b_e = torch.randn(4096, 4096, generator=g, device=dev).half()
    bias_e = torch.randn(4096, generator=g, device=dev).half()
    us = _median_us(lambda: K.gemm_bias_gelu(a_e, b_e, bias_e), flush_l2=True)
    fl = 2 * 2048 * 4096 * 4096
    res["matmul_epilogue_fp16_2048x4096x4096"] = {"us": us, "TFLOPs": fl / us / 1e6,
                                                  "frac": fl / us / 1e6 / peaks["bf16_tflops"]}
    try:
        us_cb = _median_us(lambda: torch.nn.functional.gelu(torch.addmm(bias_e, a_e, b_e), approximate="tanh"),
                           flush_l2=True)
        res["matmul_epilogue_fp16_2048x4096x4096"]["torch_cublas_addmm_gelu_TFLOPs"] = fl / us_cb / 1e6
    except Exception:
        pass
    # rmsnorm fused with the INT8 activation quantiser (bf16 in, int8 codes + f32 row scales out)
    xb, wb = x.bfloat16().reshape(-1, 4096), w.bfloat16()
    us = _median_us(lambda: K.rmsnorm_quant_int8(xb, wb), flush_l2=True)
    nb = xb.numel() * 2 + xb.numel() + xb.shape[0] * 4 + 4096 * 2
    res["rmsnorm_quant_int8_bf16_16384x4096"] = {"us": us, "GBps": nb / us / 1e3,
                                                 "frac": nb / us / 1e3 / peaks["hbm_gbs"]}
    # prefill-size fused RoPE + paged append: 16384 new tokens into the decode cache layout
    cache = WL.paged_cache(num_blocks=16384, block_size=BS, Hkv=HKV, D=D, device=dev, seed=9)
    app = WL.decode_append_inputs(cache, n_tok=16384, Hq=HQ, device=dev, seed=9)
    q_out = torch.empty_like(app["q"])
    us = _median_us(lambda: K.rope_kv_append_paged(app["q"], app["k"], app["v"], app["positions"], app["cos"],
                                                   app["sin"], app["slot_mapping"], cache.k_cache, cache.v_cache,
                                                   q_out=q_out), flush_l2=True)
    nb = WL.append_bytes(16384, HQ, HKV, D)
    res["rope_kv_append_paged_prefill_16384tok"] = {"us": us, "GBps": nb / us / 1e3,
                                                    "frac": nb / us / 1e3 / peaks["hbm_gbs"]}
    # quant_matmul through the reference interface (ops/quant_matmul cuda_v1: per-row quantiser of a,
    # per-column quantiser of b with the transposed K-major output, INT8 GEMM, fp32 out), and its two
    # quantisers alone
    from b200ops.ops.quant_matmul.templates import cuda_v1 as qm
    g = torch.Generator(device=dev).manual_seed(13)
    a_q = torch.randn(1, 4096, 4096, generator=g, device=dev).bfloat16()
    b_q = torch.randn(4096, 14336, generator=g, device=dev).bfloat16()
    us = _median_us(lambda: K.quantize_int8(a_q.reshape(4096, 4096)), flush_l2=True)
    nb = 4096 * 4096 * 3 + 4096 * 4
    res["quantize_int8_rows_bf16_4096x4096"] = {"us": us, "GBps": nb / us / 1e3, "frac": nb / us / 1e3 / peaks["hbm_gbs"]}
    us = _median_us(lambda: K.quantize_int8(b_q, by_column=True), flush_l2=True)
    nb = 4096 * 14336 * 3 + 14336 * 4
    res["quantize_int8_cols_bf16_4096x14336"] = {"us": us, "GBps": nb / us / 1e3,
                                                  "frac": nb / us / 1e3 / peaks["hbm_gbs"]}
    fn = qm.sm100()
    us = _median_us(lambda: fn(a_q, b_q), flush_l2=True)
    res["quant_matmul_op_bf16_1x4096x4096_x_4096x14336"] = {
        "us": us, "includes": "both quantisers + INT8 GEMM with fp32 output, as the reference op"}
    return res


def sharded_gemm(dev, dist, ws) -> dict:
    """quant_matmul split by output columns over the ranks, timed on the device
    as the max over ranks, two ways: (1) the tcgen05 GEMM on each rank's W
    rows, then an NCCL all-gather over NVLink and one placement copy; (2) the
    all-gather fused into the GEMM -- each epilogue stores its tiles into every
    rank's C over NVLink, then a one-warp flag exchange.  Roofline of (2): the
    slower of the GEMM at the INT8 peak and the bytes each rank sends over
    NVLink at the measured 770 GB/s per direction."""
    from b200ops import workloads as WL
    from b200ops.dist.collectives import FusedAllGatherGemm, sharded_int8_gemm
    from b200ops.dist.sharding import column_shard
    from b200ops.runtime import ops as K

    M, N, Kd = 4096, 14336, 4096
    A, W, sA, sW = WL.int8_gemm_inputs(M, N, Kd, device=dev)
    rank = dist.get_rank()
    n0, n1 = column_shard(N, ws, rank)
    Wl, sWl = W[n0:n1].contiguous(), sW[n0:n1].contiguous()

    def gemm(A_, W_, sA_, sW_, out):
        K.int8_gemm(A_, W_, sA_, sW_, out=out)

    def timed(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(dist, e0.elapsed_time(e1) * 1e3 / reps, dev)

    ops = 2 * M * N * Kd
    # both multi-GPU results equal the one-GPU GEMM bit for bit before either is timed
    full = K.int8_gemm(A, W, sA, sW)
    exact_nccl = bool(torch.equal(sharded_int8_gemm(A, Wl, sA, sWl, N, gemm), full))
    fused = FusedAllGatherGemm(M, N, device=dev)
    exact_fused = bool(torch.equal(fused(A, Wl, sA, sWl).clone(), full))
    torch.cuda.synchronize()
    exact = max_over_ranks(dist, 0.0 if (exact_nccl and exact_fused and K.read_device_error(dev) == 0) else 1.0,
                           dev) == 0.0
    if not exact:
        raise RuntimeError("sharded INT8 GEMM differs from the one-GPU GEMM on some rank")
    del full
    us_nccl = timed(lambda: sharded_int8_gemm(A, Wl, sA, sWl, N, gemm))
    us_fused = timed(lambda: fused(A, Wl, sA, sWl))
    fused.close()
    peaks = measured_peaks()
    link_gbs = 770.0
    sent = (ws - 1) * M * (n1 - n0) * 2
    target_us = max(ops / ws / (2 * peaks["bf16_tflops"]) / 1e6, sent / link_gbs / 1e3)
    return {
        f"int8_gemm_colsharded_M{M}_N{N}_K{Kd}_x{ws}": {
            "us": us_nccl, "TOPS_total": ops / us_nccl / 1e6, "bit_exact_vs_1gpu": exact_nccl,
            "includes": "local GEMM + NCCL all-gather + placement"},
        f"int8_gemm_allgather_fused_M{M}_N{N}_K{Kd}_x{ws}": {
            "us": us_fused, "TOPS_total": ops / us_fused / 1e6, "nvlink_bytes_sent_per_rank": sent,
            "roofline_us": target_us, "frac": target_us / us_fused, "bit_exact_vs_1gpu": exact_fused,
            "includes": "ready-flag exchange + GEMM with peer-store epilogue + done-flag exchange"},
    }


# --------------------------------------------------------------------------- B200
def run_b200(args, ws, rank, local, dist):
    from b200ops import workloads as WL
    from b200ops.runtime import lib as L
    from b200ops.runtime import ops as K

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L.load()
    from b200ops.dist.sharding import imbalance, shard_sequences

    seed = 1000 * rank
    # a global batch of 64 sequences per GPU, sharded by KV bytes (longest
    # first onto the least-loaded rank): each rank owns its share's KV pages
    ctx_all = WL.context_lengths(N_SEQ * ws)
    parts = shard_sequences(ctx_all.tolist(), ws)
    mine = ctx_all[parts[rank]]
    cache = WL.paged_cache(num_blocks=NBLK, block_size=BS, Hkv=HKV, D=D, device=dev, seed=seed)
    app = WL.decode_append_inputs(cache, n_tok=len(mine), Hq=HQ, device=dev, seed=seed)
    att = WL.decode_attention_inputs(cache, Hq=HQ, device=dev, seed=seed, context_len=mine)
    q_out = torch.empty_like(app["q"])
    out = torch.empty_like(att["q"])
    stream = torch.cuda.current_stream(dev)

    def step():
        K.rope_kv_append_paged(app["q"], app["k"], app["v"], app["positions"], app["cos"], app["sin"],
                               app["slot_mapping"], cache.k_cache, cache.v_cache, q_out=q_out)
        K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"], att["context_len"], out=out,
                          cfg=DECODE_CFG)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timing.  The n steps are captured in one CUDA graph
    # (one graph launch; no host gaps between the 2n kernels, as a serving
    # loop would run them) and the graph's replay is timed; per-kernel times
    # come from two more graphs of n appends and n decodes timed the same
    # way.  If capture is refused, the same loop runs eagerly.
    n = args.steps
    peaks = measured_peaks()

    def append_only():
        K.rope_kv_append_paged(app["q"], app["k"], app["v"], app["positions"], app["cos"], app["sin"],
                               app["slot_mapping"], cache.k_cache, cache.v_cache, q_out=q_out)

    def decode_only():
        K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"], att["context_len"], out=out,
                          cfg=DECODE_CFG)

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(n):
                fn()
        return g

    try:
        graphs = [capture(step), capture(append_only), capture(decode_only)]
        timing = "cuda graph of the timed steps"
    except Exception as e:  # capture refused: time the eager loop instead
        graphs = None
        timing = f"eager ({type(e).__name__})"
    torch.cuda.synchronize()

    def run(which):
        if graphs is not None:
            graphs[which].replay()
        else:
            for _ in range(n):
                (step, append_only, decode_only)[which]()

    def timed(which):
        barrier(dist)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run(which)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(dist)
        return e0.elapsed_time(e1)

    with ClockSampler(local) as clk:
        ms_local = timed(0)
    ms = max_over_ranks(dist, ms_local, dev)
    append_local = timed(1) / n
    decode_local = timed(2) / n
    append_ms = max_over_ranks(dist, append_local, dev)
    decode_ms = max_over_ranks(dist, decode_local, dev)
    clocks = clk.summary()
    per_rank = gather_per_rank(dist, dev, ws, step_ms=ms_local / n, decode_ms=decode_local,
                               append_ms=append_local, sm_mhz=clocks.get("sm_mhz") or 0.0,
                               decode_gbps=WL.decode_bytes(att["context_len"], HQ, HKV, D, BS) / decode_local / 1e6)
    assert K.read_device_error(dev) == 0, "device error word set during the timed region"
    graphs = None  # release the graphs before the process group goes

    # ---- end to end through the public API with host buffers
    # Per-step inputs come from pinned host memory; the KV cache and the
    # cos/sin tables are resident state (like weights) and stay on the device.
    # A serving loop's pipeline: the step's eight inputs are packed into one
    # pinned staging buffer (one host->device copy per step, on a copy
    # stream), double-buffered so step i+1's copy overlaps step i's kernels;
    # each step's output is read back to pinned host memory on a third stream.
    # Every step's copies are inside the timed region.
    step_inputs = {"app_q": app["q"], "app_k": app["k"], "app_v": app["v"], "app_pos": app["positions"],
                   "app_slots": app["slot_mapping"], "att_q": att["q"], "att_table": att["block_table"],
                   "att_ctx": att["context_len"]}
    layout, off = {}, 0
    for k_, v_ in step_inputs.items():
        nb = v_.numel() * v_.element_size()
        layout[k_] = (off, nb, v_.dtype, tuple(v_.shape))
        off += (nb + 255) // 256 * 256
    staged = off
    pin = torch.empty(staged, dtype=torch.uint8).pin_memory()
    for k_, v_ in step_inputs.items():
        o_, nb, _, _ = layout[k_]
        pin[o_:o_ + nb].copy_(v_.contiguous().view(torch.uint8).reshape(-1).cpu())
    dev_raw = [torch.empty(staged, dtype=torch.uint8, device=dev) for _ in range(2)]

    def views(raw):
        return {k_: raw[o_:o_ + nb].view(dt).view(shp) for k_, (o_, nb, dt, shp) in layout.items()}

    dev_in = [views(r) for r in dev_raw]
    out_buf = [torch.empty_like(out) for _ in range(2)]
    out_host = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    h2d = staged
    d2h = out_host[0].numel() * out_host[0].element_size()
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("in_ready", "in_free", "out_ready", "out_free")}

    def e2e_step(i):
        k_ = i & 1
        x = dev_in[k_]
        with torch.cuda.stream(h2d_s):
            if i >= 2:
                h2d_s.wait_event(ev["in_free"][k_])
            dev_raw[k_].copy_(pin, non_blocking=True)
            ev["in_ready"][k_].record(h2d_s)
        stream.wait_event(ev["in_ready"][k_])
        if i >= 2:
            stream.wait_event(ev["out_free"][k_])
        K.rope_kv_append_paged(x["app_q"], x["app_k"], x["app_v"], x["app_pos"], app["cos"], app["sin"],
                               x["app_slots"], cache.k_cache, cache.v_cache, q_out=q_out)
        K.paged_attention(x["att_q"], cache.k_cache, cache.v_cache, x["att_table"], x["att_ctx"], out=out_buf[k_],
                          cfg=DECODE_CFG)
        ev["in_free"][k_].record(stream)
        ev["out_ready"][k_].record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(ev["out_ready"][k_])
            out_host[k_].copy_(out_buf[k_], non_blocking=True)
            ev["out_free"][k_].record(d2h_s)

    def e2e_run(steps):
        for i in range(steps):
            e2e_step(i)
        stream.wait_stream(d2h_s)  # the last read-back is part of the run

    e2e_run(max(2, args.warmup))
    torch.cuda.synchronize()
    barrier(dist)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h2d_s.wait_stream(stream)
    d2h_s.wait_stream(stream)
    e2e_run(n)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1), dev)
    assert torch.equal(out_host[(n - 1) & 1], out_buf[(n - 1) & 1].cpu()), "end-to-end read-back mismatch"

    tokens = N_SEQ * ws * n
    value = tokens / (ms / 1e3)
    dec_bytes = WL.decode_bytes(att["context_len"], HQ, HKV, D, BS, index_bytes=4)
    achieved = dec_bytes / (decode_ms / 1e3) / 1e9
    traffic = DECODE_DRAM_BYTES_SMALL / DECODE_ALGO_BYTES_SMALL * dec_bytes if DECODE_ALGO_BYTES_SMALL else None
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": n, "warmup": args.warmup,
        "ms_per_step": ms / n, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded, on device)", "config": dict(WORKLOAD),
        "parallelism": f"dp{ws} (sequences; each rank owns its sequences' KV pages, no collective)",
        "e2e": {"value": N_SEQ * ws * n / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / n,
                "pipeline": "inputs packed into one pinned buffer, host->device copy of step i+1 on a copy "
                            "stream overlapping step i's kernels (double-buffered), output read back on a "
                            "third stream; the device-timed loop above also records 3 events per step"},
        "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel", "achieved": achieved,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_src": peaks["src"], "traffic": traffic, "traffic_src": "ncu DRAM bytes of the small decode case, scaled by algorithmic bytes",
                     "algorithmic_bytes_per_launch": dec_bytes,
                     "kernel_ms": decode_ms},
        "per_op_ms": {"rope_kv_append_paged": append_ms, "paged_attention": decode_ms}, "timing": timing,
        "decode_step_append": {
            "what": "the step's fused RoPE + paged append of 64 new tokens alone (n appends in one graph)",
            "us": append_ms * 1e3, "tokens_per_s": N_SEQ * ws / (append_ms / 1e3),
            "GBps": WL.append_bytes(len(mine), HQ, HKV, D) / append_ms / 1e6,
            "frac": WL.append_bytes(len(mine), HQ, HKV, D) / append_ms / 1e6 / peaks["hbm_gbs"],
            "algorithmic_bytes": WL.append_bytes(len(mine), HQ, HKV, D),
            "bound": "launch/latency (1.6 MB per call)"},
        "sharding": {"global_sequences": N_SEQ * ws, "sequences_per_rank": [len(p) for p in parts],
                     "kv_tokens_per_rank": [int(ctx_all[p].sum()) for p in parts],
                     "imbalance": imbalance(ctx_all.tolist(), parts),
                     "rule": "longest first onto the least-loaded rank (b200ops.dist.sharding.shard_sequences)"},
        **({"per_rank": per_rank} if ws > 1 else {}),
        "gpu_launches": 2 * n,
        "clocks": clocks,
    }


# ------------------------------------------------------------------- CPU baseline
def cpu_decode_inputs(n_seq_sample: int, seed: int = 0) -> dict:
    """Host inputs of the decode step for `n_seq_sample` sequences of the
    workload (ctx U[512,8192], random block tables, 64 new tokens' rows)."""
    import oracle.ops as O

    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(512, 8193, (n_seq_sample,), generator=g)
    nb = int(((ctx + BS - 1) // BS).sum())
    kc = torch.randn(nb, BS, HKV, D, generator=g).bfloat16()
    vc = torch.randn(nb, BS, HKV, D, generator=g).bfloat16()
    table = torch.randperm(nb, generator=g)
    maxb = 8192 // BS
    bt = torch.full((n_seq_sample, maxb), -1, dtype=torch.long)
    off = 0
    for b in range(n_seq_sample):
        k = int((ctx[b] + BS - 1) // BS)
        bt[b, :k] = table[off:off + k]
        off += k
    cos, sin = O.rope_cos_sin(4096, D)
    return dict(n=n_seq_sample, nb=nb, ctx=ctx, kc=kc, vc=vc, bt=bt, cos=cos, sin=sin,
                q=torch.randn(n_seq_sample, HQ, D, generator=g).bfloat16(),
                kn=torch.randn(n_seq_sample, HKV, D, generator=g).bfloat16(),
                vn=torch.randn(n_seq_sample, HKV, D, generator=g).bfloat16(),
                pos=torch.randint(0, 4096, (n_seq_sample,), generator=g),
                slots=torch.randperm(nb * BS, generator=g)[:n_seq_sample])


def cpu_decode_time(x: dict) -> float:
    """Seconds of the oracle's decode step (append rows + paged attention) on
    the host cores for the inputs of cpu_decode_inputs."""
    import oracle.ops as O

    t0 = time.perf_counter()
    O.rope_kv_append_paged(x["q"], x["kn"], x["vn"], x["pos"], x["cos"], x["sin"], x["slots"], x["nb"] * BS)
    O.paged_attention(x["q"], x["kc"], x["vc"], x["bt"], x["ctx"])
    return time.perf_counter() - t0


CPU_SAMPLE_DESC = "decode step of {n} sequences (ctx U[512,8192]), oracle port"


def cpu_clone_seconds(reps: int = 2) -> float:
    """Seconds per step of the reference's functional append semantics: its
    paged append returns modified copies of both caches
    (paged_kv/reference.py:15-16, kv_append/reference.py:30-31), i.e. one
    clone of each [65536, 16, 8, 128] bf16 cache (2 GiB each) per step."""
    kc = torch.empty(NBLK, BS, HKV, D, dtype=torch.bfloat16).fill_(1.0)
    vc = torch.empty_like(kc).fill_(1.0)
    kc.clone(), vc.clone()
    t0 = time.perf_counter()
    for _ in range(reps):
        k2, v2 = kc.clone(), vc.clone()
        del k2, v2
    return (time.perf_counter() - t0) / reps


def run_reference(args, ws, rank):
    """Reference arm: the reference's CPU path (oracle port) on the host cores."""
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    sample = N_SEQ  # a step is the whole decode step of the GPU arm's workload
    x = cpu_decode_inputs(sample, seed=1)
    for _ in range(args.warmup):
        cpu_decode_time(x)
    t_total = sum(cpu_decode_time(x) for _ in range(args.steps))
    desc = CPU_SAMPLE_DESC.format(n=sample)
    value = sample * args.steps / t_total
    try:
        clone_s = cpu_clone_seconds()
        with_clone = {"value": sample / (t_total / args.steps + clone_s), "unit": UNIT, "clone_s_per_step": clone_s,
                      "what": "the same step plus one clone of each 2 GiB cache (paged_kv/reference.py:15-16)"}
    except RuntimeError as e:
        with_clone = {"unavailable": str(e)[:120]}
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)", "config": dict(WORKLOAD),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": desc + " (clone-free; the reference's per-append cache clones are timed in "
                                          "with_reference_clone)", "with_reference_clone": with_clone},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


PROFILE_CASES = ("decode", "decode-split", "append", "gemm", "gemm-cublas", "gemm-skinny", "flash", "flash-full",
                 "rmsnorm", "rmsnorm-quant", "gemm-gelu", "append-prefill", "sdpa-full")


def profile_case(name: str, reps: int = 3) -> None:
    """Runs one operator on a profiling-sized case `reps` times (for an ncu
    capture of a single kernel: inputs larger than L2, a few GB at most)."""
    from b200ops import workloads as WL
    from b200ops.runtime import ops as K

    dev = torch.device("cuda", 0)
    if name in ("decode", "decode-split", "append"):
        cache = WL.paged_cache(num_blocks=16384, block_size=BS, Hkv=HKV, D=D, device=dev)
        if name == "append":
            app = WL.decode_append_inputs(cache, n_tok=N_SEQ, Hq=HQ, device=dev)
            fn = lambda: K.rope_kv_append_paged(app["q"], app["k"], app["v"], app["positions"], app["cos"],  # noqa: E731
                                                app["sin"], app["slot_mapping"], cache.k_cache, cache.v_cache)
        else:
            att = WL.decode_attention_inputs(cache, B=N_SEQ, Hq=HQ, ctx_lo=512, ctx_hi=4096, device=dev)
            cfg = {"flags": 2} if name == "decode-split" else None
            fn = lambda: K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"],  # noqa: E731
                                           att["context_len"], cfg=cfg)
    elif name in ("gemm", "gemm-skinny", "gemm-cublas"):
        M = 16 if name == "gemm-skinny" else 4096
        A, W, sA, sW = WL.int8_gemm_inputs(M, 14336, 4096, device=dev)
        if name == "gemm-cublas":  # the library comparator on the same operands (int32 out, no dequant)
            fn = lambda: torch._int_mm(A, W.t())  # noqa: E731
        else:
            fn = lambda: K.int8_gemm(A, W, sA, sW)  # noqa: E731
    elif name == "flash":
        q, k, v = WL.flash_inputs(B=1, H=8, T=4096, device=dev)
        fn = lambda: K.flash_attn(q, k, v, causal=True)  # noqa: E731
    elif name in ("flash-full", "sdpa-full"):  # the prefill bench shape, 4 x 32 x 4096 x 128
        q, k, v = WL.flash_inputs(device=dev)
        if name == "flash-full":
            fn = lambda: K.flash_attn(q, k, v, causal=True)  # noqa: E731
        else:
            fn = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)  # noqa: E731
    elif name == "rmsnorm-quant":
        x, w = WL.rmsnorm_inputs(device=dev)
        xb, wb = x.bfloat16().reshape(-1, 4096), w.bfloat16()
        fn = lambda: K.rmsnorm_quant_int8(xb, wb)  # noqa: E731
    elif name == "gemm-gelu":
        g = torch.Generator(device=dev).manual_seed(11)
        a_e = (torch.randn(2048, 4096, generator=g, device=dev) / 8).half()
        b_e = torch.randn(4096, 4096, generator=g, device=dev).half()
        bias_e = torch.randn(4096, generator=g, device=dev).half()
        fn = lambda: K.gemm_bias_gelu(a_e, b_e, bias_e)  # noqa: E731
    elif name == "append-prefill":
        cache = WL.paged_cache(num_blocks=16384, block_size=BS, Hkv=HKV, D=D, device=dev, seed=9)
        app = WL.decode_append_inputs(cache, n_tok=16384, Hq=HQ, device=dev, seed=9)
        fn = lambda: K.rope_kv_append_paged(app["q"], app["k"], app["v"], app["positions"], app["cos"],  # noqa: E731
                                            app["sin"], app["slot_mapping"], cache.k_cache, cache.v_cache)
    else:
        x, w = WL.rmsnorm_inputs(device=dev)
        fn = lambda: K.rmsnorm(x, w)  # noqa: E731
    for _ in range(reps):
        fn()
    torch.cuda.synchronize()
    assert K.read_device_error(dev) == 0
    info = {"case": name, "reps": reps, "ok": True}
    if name in ("decode", "decode-split"):
        info["algorithmic_bytes"] = WL.decode_bytes(att["context_len"], HQ, HKV, D, BS)
    print(json.dumps(info))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the per-op lines (GEMM, prefill, rmsnorm)")
    ap.add_argument("--case", choices=PROFILE_CASES, default=None,
                    help="run one operator on a small case for a profiler capture, then exit")
    args = ap.parse_args()
    if args.case:
        profile_case(args.case)
        return
    ws, rank, local = dist_env()
    if args.impl == "reference":
        res = run_reference(args, ws, rank)
        if res is not None:
            print(json.dumps(res))
        return
    dist = init_dist(ws, local)
    try:
        res = run_b200(args, ws, rank, local, dist)
        if not args.no_secondary:
            sec = secondary_ops(torch.device("cuda", local))
            if ws > 1:
                sec.update(sharded_gemm(torch.device("cuda", local), dist, ws))
            if rank == 0:
                res["secondary"] = sec
        if rank == 0:
            if ws == 1 and not args.no_cpu_baseline:
                # whole decode steps (64 sequences) repeated for about 10 s of host work
                torch.set_num_threads(os.cpu_count() or 1)
                x = cpu_decode_inputs(N_SEQ, seed=7)
                cpu_decode_time(x)
                secs, i = 0.0, 0
                while secs < 10.0 and i < 50:
                    secs, i = secs + cpu_decode_time(x), i + 1
                res["cpu_baseline"] = {"value": N_SEQ * i / secs, "unit": UNIT, "cores": torch.get_num_threads(),
                                       "kind": "port", "sample": f"{i} x " + CPU_SAMPLE_DESC.format(n=N_SEQ),
                                       "seconds": secs}
                try:
                    clone_s = cpu_clone_seconds()
                    step_s = secs / i
                    res["cpu_baseline"]["with_reference_clone"] = {
                        "value": N_SEQ / (step_s + clone_s), "unit": UNIT, "clone_s_per_step": clone_s,
                        "what": "the same step plus the reference's functional append: one clone of each 2 GiB "
                                "cache per step (paged_kv/reference.py:15-16)"}
                except RuntimeError as e:  # host memory: two 2 GiB caches and their clones
                    res["cpu_baseline"]["with_reference_clone"] = {"unavailable": str(e)[:120]}
            print(json.dumps(res))
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
