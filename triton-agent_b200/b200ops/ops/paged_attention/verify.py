"""Correctness check of the paged_attention CUDA variant against reference.py
(role of triton_agent/ops/paged_attention/verify.py)."""

from pathlib import Path

from b200ops.core.contract import OpContract
from b200ops.core.verifier import check_numerical

_HERE = Path(__file__).resolve().parent


def verify_paged_attention(kernel_fn, inputs, reference_fn=None):
    from importlib import import_module

    contract = OpContract.from_yaml(_HERE / "contract.yaml")
    ref = reference_fn or getattr(import_module("b200ops.ops.paged_attention.reference"), "paged_attention")
    expected = ref(*inputs)
    got = kernel_fn(*inputs)
    return check_numerical(got, expected, contract)
