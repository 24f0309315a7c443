"""Correctness check of the matmul_epilogue CUDA variant against reference.py."""

from pathlib import Path

from b200ops.core.contract import OpContract
from b200ops.core.verifier import check_numerical

_HERE = Path(__file__).resolve().parent


def verify_matmul_epilogue(kernel_fn, inputs, reference_fn=None):
    from importlib import import_module

    contract = OpContract.from_yaml(_HERE / "contract.yaml")
    ref = reference_fn or getattr(import_module("b200ops.ops.matmul_epilogue.reference"), "matmul_epilogue")
    expected = ref(*inputs)
    got = kernel_fn(*inputs)
    return check_numerical(got, expected, contract)
