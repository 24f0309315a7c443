"""Correctness check of the kv_append CUDA variant against reference.py
(role of triton_agent/ops/kv_append/verify.py)."""

from pathlib import Path

from b200ops.core.contract import OpContract
from b200ops.core.verifier import check_numerical

_HERE = Path(__file__).resolve().parent


def verify_kv_append(kernel_fn, inputs, reference_fn=None):
    from importlib import import_module

    contract = OpContract.from_yaml(_HERE / "contract.yaml")
    ref = reference_fn or getattr(import_module("b200ops.ops.kv_append.reference"), "kv_append")
    expected = ref(*inputs)
    got = kernel_fn(*inputs)
    return check_numerical(got, expected, contract)
