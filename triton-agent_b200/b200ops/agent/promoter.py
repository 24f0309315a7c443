"""Promotion gate (triton_agent/agent/promoter.py:7-26): compiled, verified,
fast enough (speedup >= min_speedup) and stable (CV <= max_variance)."""

from __future__ import annotations

from ..core.contract import OpContract
from ..core.spec import CandidateResult


def should_promote(result: CandidateResult, contract: OpContract) -> bool:
    return (result.compile_pass and result.verify_pass and result.speedup >= contract.promotion.min_speedup
            and result.variance <= contract.promotion.max_variance)
