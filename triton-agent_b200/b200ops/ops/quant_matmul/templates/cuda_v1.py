"""sm_100a CUDA variant of quant_matmul (libb200ops.so through ctypes).

`sm100(**compile_args)` returns kernel_fn(*inputs) for the inputs produced by
reference.generate_test_inputs, the calling convention of the reference's
Triton templates; compile_args may carry b200_launch_cfg fields chosen by the
tuner.  There is no fallback: without the library or a GPU the call raises.
"""

import torch as _torch  # noqa: F401

from b200ops.ops._variant import make_factory as _make_factory
from b200ops.runtime import ops as _K


def _run(a, b, cfg=None):
    lead, (M, K) = a.shape[:-2], a.shape[-2:]
    qa, sa = _K.quantize_int8(a.reshape(-1, K).contiguous())
    qb, sb = _K.quantize_int8(b.contiguous(), by_column=True)
    return _K.int8_gemm(qa, qb, sa, sb, out_dtype=_torch.float32, cfg=cfg).reshape(*lead, M, b.shape[1])


sm100 = _make_factory(_run, uses_threads=False)
