"""Multi-rank host logic on CPU (gloo, world size 2): sequence/row/column
sharding, the column all-gather layout of the sharded INT8 GEMM, and
failure detection when a rank dies before a collective."""

import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent
from b200ops.dist.sharding import column_shard, imbalance, shard_rows, shard_sequences  # noqa: E402


def test_shard_rows_cover_exactly():
    for n, w in [(16384, 8), (10, 3), (3, 4)]:
        idx = []
        for r in range(w):
            s = shard_rows(n, w, r)
            idx.extend(range(s.start, s.stop))
        assert idx == list(range(n))


def test_sequences_balanced_by_kv_bytes():
    g = torch.Generator().manual_seed(0)
    ctx = torch.randint(512, 8193, (64 * 8,), generator=g).tolist()
    for w in (2, 4, 8):
        parts = shard_sequences(ctx, w)
        assert sorted(i for p in parts for i in p) == list(range(len(ctx)))
        assert imbalance(ctx, parts) < 1.01
    assert shard_sequences([5, 0, 7], 2) == shard_sequences([5, 0, 7], 2)  # deterministic


def test_column_shards_tile_aligned():
    for N, w in [(14336, 8), (4096, 2), (4096, 8), (100, 3)]:
        cols = []
        for r in range(w):
            n0, n1 = column_shard(N, w, r)
            assert n0 % 128 == 0 or n0 == N
            cols.extend(range(n0, n1))
        assert cols == list(range(N))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker_gather(rank, world, port, q):
    sys.path[:0] = [str(REPO), str(REPO / "triton-agent_b200")]
    import datetime

    import torch.distributed as dist

    from b200ops.dist.collectives import sharded_int8_gemm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(3)
        M, N, K = 5, 300, 32
        A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        W = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        sA = torch.rand(M, generator=g) * 0.02
        sW = torch.rand(N, generator=g) * 0.02
        n0, n1 = column_shard(N, world, rank)

        def cpu_gemm(A_, W_, sA_, sW_, out):  # stand-in for the CUDA GEMM of this rank's block
            acc = A_.to(torch.int64) @ W_.to(torch.int64).T
            out.copy_((acc.float() * sA_[:, None] * sW_[None, :]).to(out.dtype))

        C = sharded_int8_gemm(A, W[n0:n1], sA, sW[n0:n1], N, cpu_gemm, out_dtype=torch.float32)
        full = (A.to(torch.int64) @ W.to(torch.int64).T).float() * sA[:, None] * sW[None, :]
        q.put((rank, bool(torch.equal(C, full))))
    finally:
        dist.destroy_process_group()


def test_column_allgather_reassembles_full_output():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _worker_fail(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # the rank fails between steps, before its next collective
        os._exit(3)
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except Exception as e:  # the surviving rank learns of it with an error, not a hang
        q.put((rank, type(e).__name__))


def test_dead_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and outcome != "completed"
    assert time.time() - t0 < 110
    assert procs[1].exitcode == 3
