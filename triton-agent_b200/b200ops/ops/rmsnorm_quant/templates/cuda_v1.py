"""sm_100a CUDA variant of rmsnorm_quant (libb200ops.so through ctypes):
b200_rmsnorm_quant_int8, rmsnorm and the row INT8 quantiser in one pass.
Returns (codes [B, T, D] int8, scale [B, T, 1] f32).  No fallback."""

import torch as _torch  # noqa: F401

from b200ops.ops._variant import make_factory as _make_factory
from b200ops.runtime import ops as _K


def _run(x, weight, cfg=None):
    q, scale = _K.rmsnorm_quant_int8(x, weight, 1e-6, cfg=cfg)
    return q, scale.view(*x.shape[:-1], 1)


sm100 = _make_factory(_run, uses_threads=True)
