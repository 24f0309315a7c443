"""Variant "compilation": bind a CUDA variant factory to its launch config.

Same contract as triton_agent/core/compiler.py:19-52 -- compile_kernel(
template, compile_args) calls template(**compile_args) and captures any
exception into CompileResult.error_log.  The kernels are compiled ahead of
time into libb200ops.so, so this step only validates the parameters and
returns a callable; it is a table lookup, not a JIT.
"""

from __future__ import annotations

import time
import traceback
from dataclasses import dataclass
from typing import Any, Callable


@dataclass
class CompileResult:
    success: bool = False
    kernel_fn: Callable | None = None
    compile_time_s: float = 0.0
    error_log: str = ""


class VariantCompiler:
    def compile(self, kernel_template: Callable, compile_args: dict[str, Any]) -> CompileResult:
        res = CompileResult()
        t0 = time.perf_counter()
        try:
            res.kernel_fn = kernel_template(**compile_args)
            res.success = True
        except Exception:
            res.error_log = traceback.format_exc()
        res.compile_time_s = time.perf_counter() - t0
        return res


def compile_kernel(kernel_template: Callable, compile_args: dict[str, Any]) -> CompileResult:
    return VariantCompiler().compile(kernel_template, compile_args)
