"""Correctness gate (triton_agent/core/verifier.py:10-79).

check_numerical(output, reference, contract) -> CandidateResult with the
same verify_log JSON keys (max_abs_error, mean_abs_error, tolerance_*,
has_nan, has_inf, passed).  Shapes and dtypes must match exactly, as in the
reference.  Outputs may be a tuple (kv_append returns two caches); every
element is checked.  With tolerance.exact the comparison is bitwise; with
tolerance.max_rel_error an element passes when
|out - ref| <= max_abs_error + max_rel_error * |ref|.
"""

from __future__ import annotations

import json
from typing import Any

from .contract import OpContract
from .spec import CandidateResult


def _pairs(output: Any, reference: Any):
    if isinstance(reference, (tuple, list)):
        if not isinstance(output, (tuple, list)) or len(output) != len(reference):
            raise TypeError("output arity does not match the reference")
        return list(zip(output, reference))
    return [(output, reference)]


def check_numerical(output: Any, reference: Any, contract: OpContract) -> CandidateResult:
    import torch

    res = CandidateResult(compile_pass=True)
    tol = contract.tolerance
    try:
        max_ae = 0.0
        sum_ae = 0.0
        count = 0
        rel_ok = True
        exact_ok = True
        has_nan = has_inf = False
        for out, ref in _pairs(output, reference):
            if not isinstance(out, torch.Tensor):
                res.verify_log = "output is not a torch.Tensor"
                return res
            if out.shape != ref.shape:
                res.verify_log = f"shape mismatch: output={list(out.shape)} reference={list(ref.shape)}"
                return res
            if str(out.dtype) != str(ref.dtype):
                res.verify_log = f"dtype mismatch: output={out.dtype} reference={ref.dtype}"
                return res
            o = out.detach().cpu()
            r = ref.detach().cpu()
            if tol.exact:
                exact_ok = exact_ok and torch.equal(o, r)
            of, rf = o.double(), r.double()
            diff = (of - rf).abs()
            if diff.numel():
                max_ae = max(max_ae, float(diff.max()))
                sum_ae += float(diff.sum())
                count += diff.numel()
            if tol.max_rel_error is not None and diff.numel():
                rel_ok = rel_ok and bool((diff <= tol.max_abs_error + tol.max_rel_error * rf.abs()).all())
            if o.is_floating_point():
                has_nan = has_nan or bool(torch.isnan(o).any())
                has_inf = has_inf or bool(torch.isinf(o).any())
        mean_ae = sum_ae / count if count else 0.0
        if tol.exact:
            passed = exact_ok
        elif tol.max_rel_error is not None:
            passed = rel_ok and mean_ae <= tol.mean_abs_error
        else:
            passed = max_ae <= tol.max_abs_error and mean_ae <= tol.mean_abs_error
        passed = passed and not has_nan and not has_inf
        res.verify_pass = bool(passed)
        log = {"max_abs_error": max_ae, "mean_abs_error": mean_ae, "tolerance_max_abs": tol.max_abs_error,
               "tolerance_mean_abs": tol.mean_abs_error, "has_nan": has_nan, "has_inf": has_inf,
               "passed": bool(passed)}
        if tol.max_rel_error is not None:
            log["tolerance_max_rel"] = tol.max_rel_error
        if tol.exact:
            log["exact"] = True
        res.verify_log = json.dumps(log)
    except Exception as e:  # malformed outputs end up in the log, like the reference
        res.verify_pass = False
        res.verify_log = str(e)
    return res
