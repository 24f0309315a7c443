"""sm_100a CUDA variant of matmul_epilogue (libb200ops.so through ctypes):
b200_gemm_bias_gelu, tcgen05 kind::f16 on CTA pairs with the bias + GELU
epilogue.  No fallback."""

import torch as _torch  # noqa: F401

from b200ops.ops._variant import make_factory as _make_factory
from b200ops.runtime import ops as _K


def _run(a, b, bias, cfg=None):
    return _K.gemm_bias_gelu(a, b, bias, cfg=cfg)


sm100 = _make_factory(_run, uses_threads=False)
