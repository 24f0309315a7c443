"""sm_100a CUDA variant of rope (libb200ops.so through ctypes).

`sm100(**compile_args)` returns kernel_fn(*inputs) for the inputs produced by
reference.generate_test_inputs, the calling convention of the reference's
Triton templates; compile_args may carry b200_launch_cfg fields chosen by the
tuner.  There is no fallback: without the library or a GPU the call raises.
"""

import torch as _torch  # noqa: F401

from b200ops.ops._variant import make_factory as _make_factory
from b200ops.runtime import ops as _K


def _run(x, cos, sin, cfg=None):
    return _K.rope(x, cos, sin, cfg=cfg)


sm100 = _make_factory(_run, uses_threads=True)
