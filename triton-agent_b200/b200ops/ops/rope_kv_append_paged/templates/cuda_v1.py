"""sm_100a CUDA variant of rope_kv_append_paged (libb200ops.so through ctypes).

`sm100(**compile_args)` returns kernel_fn(*inputs) for the inputs produced by
reference.generate_test_inputs, the calling convention of the reference's
Triton templates; compile_args may carry b200_launch_cfg fields chosen by the
tuner.  There is no fallback: without the library or a GPU the call raises.
"""

import torch as _torch  # noqa: F401

from b200ops.ops._variant import make_factory as _make_factory
from b200ops.runtime import ops as _K


def _run(q, k, v, positions, cos, sin, slot_mapping, k_cache, v_cache, cfg=None):
    q_out = _K.rope_kv_append_paged(q, k, v, positions, cos, sin, slot_mapping, k_cache, v_cache, cfg=cfg)
    return q_out, k_cache, v_cache


sm100 = _make_factory(_run, uses_threads=True)
