"""Failure detection on one GPU without a fault: a bounded cross-GPU flag
wait that nobody answers gives up, records its code in the device error word
and returns, and the next call runs clean.

The fused all-gather GEMM (b200_int8_gemm_allgather) is called as rank 0 of
a world of 2 whose "peer" buffers are this GPU's own: the GEMM and its
epilogue run normally (both destinations are local memory), but no second
rank ever stores the flags rank 0 waits for.  With a 20 ms wait limit, both
flag exchanges (ready before the GEMM, done after it) run out; the host
reads code 6 (a cross-GPU wait gave up).  Then the test stores the peer's
flags itself and the next call completes with no error and the exact GEMM
result."""

import ctypes

import pytest
import torch

from b200ops import workloads as WL
from b200ops.runtime import lib as L
from b200ops.runtime import ops as K

pytestmark = pytest.mark.gpu


def _call(lib, A, W, sA, sW, Cs, sigs, epoch):
    M, Kd = A.shape
    N = W.shape[0]
    c_arr = (ctypes.c_void_p * 2)(*[c.data_ptr() for c in Cs])
    s_arr = (ctypes.c_void_p * 2)(*[s.data_ptr() for s in sigs])
    cfg = L.LaunchCfg(flags=1)
    ws_bytes = int(lib.b200_int8_gemm_workspace_size(M, N, Kd, ctypes.byref(cfg)))
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device=A.device)
    return lib.b200_int8_gemm_allgather(
        A.data_ptr(), W.data_ptr(), sA.data_ptr(), sW.data_ptr(), c_arr, s_arr, 2, 0, M, N, 0, Kd, N,
        L.F16, epoch, ws.data_ptr(), ws_bytes, ctypes.byref(cfg),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_unanswered_peer_flag_wait_times_out_then_recovers(cuda_device):
    lib = L.load()
    A, W, sA, sW = WL.int8_gemm_inputs(256, 512, 256, device=cuda_device, seed=3)
    full = K.int8_gemm(A, W, sA, sW)
    Cs = [torch.zeros(256, 512, dtype=torch.float16, device=cuda_device) for _ in range(2)]
    sigs = [torch.zeros(4, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    torch.cuda.synchronize()
    assert K.read_device_error() == 0
    K.set_peer_wait_timeout_us(20_000)
    try:
        st = _call(lib, A, W, sA, sW, Cs, sigs, 1)
        assert st == L.OK, L.status_string(st)
        torch.cuda.synchronize()
        assert K.read_device_error() == K.DEV_ERR_TIMEOUT_PEER
        # the GEMM itself ran: both "ranks'" C hold the full result
        assert torch.equal(Cs[0], full) and torch.equal(Cs[1], full)
        # rank 0 announced itself to its peer (ready at world + 0, done at 0)
        assert sigs[1].tolist() == [1, 0, 1, 0]
        # the next call, with the peer's flags in place, runs clean
        for c in Cs:
            c.zero_()
        sigs[0].copy_(torch.tensor([0, 2, 0, 2], dtype=torch.int32))
        st = _call(lib, A, W, sA, sW, Cs, sigs, 2)
        assert st == L.OK, L.status_string(st)
        torch.cuda.synchronize()
        assert K.read_device_error() == 0
        assert torch.equal(Cs[0], full)
    finally:
        K.set_peer_wait_timeout_us(0)


def test_timeout_setter_rejects_negative():
    lib = L.load()
    assert lib.b200_set_peer_wait_timeout_us(-1) == L.ERR_BAD_ARG
    assert lib.b200_set_peer_wait_timeout_us(0) == L.OK
