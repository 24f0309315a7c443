"""Column-sharded INT8 GEMM with an all-gather of the output blocks.

Rank r holds W rows [n0_r, n1_r) (equal blocks, column_shard) and the whole
A; it computes C_r = A W_r^T, [M, n_r], then every rank receives every block.
NCCL all-gather needs equal contiguous chunks, so blocks are gathered as
[world, M, n_blk] and placed into the row-major [M, N] output with one
device copy; both steps are inside the timed region of the benchmark.
"""

from __future__ import annotations

import torch

from .sharding import column_shard


def allgather_columns(local: torch.Tensor, N: int, group=None) -> torch.Tensor:
    """local [M, n_blk] (n_blk the padded block width) -> full C [M, N]."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M, n_blk = local.shape
    buf = torch.empty(world * M, n_blk, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
    return buf.view(world, M, n_blk).permute(1, 0, 2).reshape(M, world * n_blk)[:, :N]


def sharded_int8_gemm(A, W_local, sA, sW_local, N: int, gemm, out_dtype=torch.float16, group=None):
    """C = gather_r(gemm(A, W_r)) for the column block of this rank.

    `gemm(A, W, sA, sW, out)` writes [M, n_r] into `out`; blocks narrower than
    the common width (last rank) are zero-padded before the gather.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n0, n1 = column_shard(N, world, rank)
    n_blk = column_shard(N, world, 0)[1]
    M = A.shape[0]
    local = torch.zeros(M, n_blk, dtype=out_dtype, device=A.device)
    if n1 > n0:
        gemm(A, W_local, sA, sW_local, local[:, : n1 - n0])
    return allgather_columns(local, N, group)


class FusedAllGatherGemm:
    """Column-sharded INT8 GEMM with the all-gather fused into the GEMM
    (b200_int8_gemm_allgather): each rank's epilogue stores its output tiles
    into every rank's C over NVLink, then a one-warp kernel exchanges
    per-call flags with the peers -- no collective call, no placement copy.

    Construction (collective over `group`): every rank allocates its full C
    [M, N] and a 2*world-entry uint32 flag array ("done" and "ready" flags),
    shares CUDA IPC handles of both through one all_gather_object and maps its
    peers'.  Each call returns this object's C, which the next call
    overwrites.  A call first exchanges "ready" flags with every peer, so no
    rank writes into a peer's C before that peer's stream has reached the
    call (and so finished its reads of the previous result); then the GEMM;
    then "done" flags, so the returned C is complete.  W_local/sW_local are
    this rank's rows [n0, n1) of W (column_shard(N, world, rank)).
    """

    def __init__(self, M: int, N: int, out_dtype=torch.float16, device=None, group=None):
        import ctypes

        import torch.distributed as dist

        from b200ops.runtime import lib as L

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("fused all-gather GEMM supports up to 8 ranks (one node)")
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.M, self.N, self.out_dtype = M, N, out_dtype
        self.col0, n1 = column_shard(N, self.world, self.rank)
        self.n_local = n1 - self.col0
        self.C = torch.empty(M, N, dtype=out_dtype, device=dev)
        self.sig = torch.zeros(2 * self.world, dtype=torch.int32, device=dev)
        lib = L.load()
        mine = []
        for t in (self.C, self.sig):
            h = (ctypes.c_char * 64)()
            off = ctypes.c_int64()
            L.check(lib.b200_ipc_handle(t.data_ptr(), h, ctypes.byref(off)), "ipc_handle")
            mine.append((bytes(h), off.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened: list[tuple[int, int]] = []
        c_ptrs, s_ptrs = [], []
        for r in range(self.world):
            if r == self.rank:
                c_ptrs.append(self.C.data_ptr())
                s_ptrs.append(self.sig.data_ptr())
                continue
            for (h, off), ptrs in zip(everyone[r], (c_ptrs, s_ptrs)):
                p = ctypes.c_void_p()
                L.check(lib.b200_ipc_open(h, off, ctypes.byref(p)), "ipc_open")
                self._opened.append((p.value, off))
                ptrs.append(p.value)
        self._c_arr = (ctypes.c_void_p * self.world)(*c_ptrs)
        self._s_arr = (ctypes.c_void_p * self.world)(*s_ptrs)
        self.epoch = 0
        self._lib = lib

    def __call__(self, A: torch.Tensor, W_local: torch.Tensor, sA: torch.Tensor, sW_local: torch.Tensor,
                 cfg=None) -> torch.Tensor:
        from b200ops.runtime import lib as L
        from b200ops.runtime import ops as K

        M, Kd = A.shape
        if M != self.M or W_local.shape[0] != self.n_local:
            raise L.B200OpsError(L.ERR_BAD_ARG, "int8_gemm_allgather", "shape differs from construction")
        self.epoch += 1
        dev = A.device
        c = dict(cfg or {})
        c["flags"] = int(c.get("flags", 0)) | 1  # the tile kernels carry the multi-destination epilogue
        ws_bytes = int(self._lib.b200_int8_gemm_workspace_size(M, max(self.n_local, 1), Kd, K._cfg(c)))
        ws = K.WORKSPACES.get(dev, ws_bytes, "int8_gemm") if ws_bytes else None
        st = self._lib.b200_int8_gemm_allgather(
            K._ptr(A), K._ptr(W_local), K._ptr(sA), K._ptr(sW_local), self._c_arr, self._s_arr, self.world,
            self.rank, M, self.n_local, self.col0, Kd, self.N, K.dtype_code(self.out_dtype), self.epoch,
            K._ptr(ws), ws.numel() if ws is not None else 0, K._cfg(c), K._stream(dev))
        L.check(st, "int8_gemm_allgather")
        return self.C

    def close(self) -> None:
        for p, off in self._opened:
            self._lib.b200_ipc_close(p, off)
        self._opened = []
