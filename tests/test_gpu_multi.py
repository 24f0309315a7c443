"""Multi-GPU paths (one process per GPU, NCCL over NVLink): the
column-sharded INT8 GEMM with its all-gather equals the single-GPU GEMM bit
for bit, and batch-sharded decode (each rank owns its sequences' KV pages)
equals the single-GPU decode of the same sequences.  Skipped on a box with
one GPU."""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    sys.path[:0] = [str(REPO), str(REPO / "triton-agent_b200")]
    import datetime

    import torch.distributed as dist

    from b200ops import workloads as WL
    from b200ops.dist.collectives import sharded_int8_gemm
    from b200ops.dist.sharding import column_shard, shard_sequences
    from b200ops.runtime import ops as K

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        # column-sharded GEMM
        M, N, Kd = 512, 3000, 1024
        A, W, sA, sW = WL.int8_gemm_inputs(M, N, Kd, device=dev, seed=5)
        full = K.int8_gemm(A, W, sA, sW)
        n0, n1 = column_shard(N, world, rank)
        C = sharded_int8_gemm(A, W[n0:n1].contiguous(), sA, sW[n0:n1].contiguous(), N,
                              lambda a, w, s1, s2, out: K.int8_gemm(a, w, s1, s2, out=out))
        gemm_ok = bool(torch.equal(C, full))
        # the same GEMM with the all-gather fused into the epilogue (peer
        # stores over NVLink): bit-identical, twice (the flags' epochs advance),
        # and for a small M (persistent one-SM kernel) on a fresh object
        from b200ops.dist.collectives import FusedAllGatherGemm
        fused = FusedAllGatherGemm(M, N, device=dev)
        for _ in range(2):
            Cf = fused(A, W[n0:n1].contiguous(), sA, sW[n0:n1].contiguous())
            torch.cuda.synchronize()
            gemm_ok = gemm_ok and bool(torch.equal(Cf, full))
        # a rank still reading the previous result is not overwritten: rank 0
        # holds its stream for a while before the next call and then snapshots
        # C; the peers' next call (different scales) must not have landed yet
        sA_b = (sA * 2).contiguous()
        full_b = K.int8_gemm(A, W, sA_b, sW)
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            torch.cuda._sleep(200_000_000)  # ~0.1 s of device time
            snap = fused.C.clone()
        Cb = fused(A, W[n0:n1].contiguous(), sA_b, sW[n0:n1].contiguous())
        torch.cuda.synchronize()
        gemm_ok = gemm_ok and bool(torch.equal(Cb, full_b)) and K.read_device_error(dev) == 0
        if rank == 0:
            gemm_ok = gemm_ok and bool(torch.equal(snap, full))
        fused.close()
        A2, W2, sA2, sW2 = WL.int8_gemm_inputs(40, 1000, 256, device=dev, seed=7)
        full2 = K.int8_gemm(A2, W2, sA2, sW2)
        m0, m1 = column_shard(1000, world, rank)
        fused2 = FusedAllGatherGemm(40, 1000, device=dev)
        C2 = fused2(A2, W2[m0:m1].contiguous(), sA2, sW2[m0:m1].contiguous())
        torch.cuda.synchronize()
        gemm_ok = gemm_ok and bool(torch.equal(C2, full2)) and K.read_device_error(dev) == 0
        fused2.close()
        # fp32 output through the fused all-gather (the staged epilogue's 64-column groups)
        full32 = K.int8_gemm(A, W, sA, sW, out_dtype=torch.float32)
        fused32 = FusedAllGatherGemm(M, N, out_dtype=torch.float32, device=dev)
        C32 = fused32(A, W[n0:n1].contiguous(), sA, sW[n0:n1].contiguous())
        torch.cuda.synchronize()
        gemm_ok = gemm_ok and bool(torch.equal(C32, full32)) and K.read_device_error(dev) == 0
        fused32.close()
        # batch-sharded decode: same inputs on every rank, each computes its share
        cache = WL.paged_cache(num_blocks=2048, block_size=16, Hkv=8, D=128, device=dev, seed=6)
        att = WL.decode_attention_inputs(cache, B=16, Hq=32, ctx_lo=100, ctx_hi=1500, device=dev, seed=6)
        ref = K.paged_attention(att["q"], cache.k_cache, cache.v_cache, att["block_table"], att["context_len"])
        parts = shard_sequences(att["context_len"].cpu().tolist(), world)
        mine = torch.tensor(parts[rank], dtype=torch.long, device=dev)
        out = K.paged_attention(att["q"][mine].contiguous(), cache.k_cache, cache.v_cache,
                                att["block_table"][mine].contiguous(), att["context_len"][mine].contiguous())
        dec_ok = bool(torch.allclose(out.float(), ref[mine].float(), atol=2e-2, rtol=0))
        torch.cuda.synchronize()
        q.put((rank, gemm_ok, dec_ok))
    finally:
        dist.destroy_process_group()


def test_sharded_gemm_and_decode_match_single_gpu():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2+ GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    assert all(g for _, g, _ in res), res
    assert all(d for _, _, d in res), res
