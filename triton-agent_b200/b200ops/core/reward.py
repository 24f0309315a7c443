"""Scalar reward of a candidate (rules of triton_agent/core/reward.py:6-58).

+0.2 compile_pass; +0.6 verify_pass, else -1.0; +min(0.5, speedup - 1) when
speedup >= 1.05; -0.2 when the latency CV exceeds 0.10; -0.2 when peak memory
exceeds 110% of the baseline; -1.0 when the verify log reports NaN or Inf.
The tuner compares configurations with this same score, so the rules are kept.
"""

from __future__ import annotations

import json

from .spec import CandidateResult


def compute_score(result: CandidateResult, baseline_memory_mb: float = 0.0) -> float:
    score = 0.2 if result.compile_pass else 0.0
    score += 0.6 if result.verify_pass else -1.0
    if result.speedup >= 1.05:
        score += min(0.5, result.speedup - 1.0)
    if result.variance > 0.10:
        score -= 0.2
    if baseline_memory_mb > 0 and result.memory_peak_mb > 1.10 * baseline_memory_mb:
        score -= 0.2
    try:
        log = json.loads(result.verify_log)
        if isinstance(log, dict) and (log.get("has_nan") or log.get("has_inf")):
            score -= 1.0
    except (TypeError, ValueError):
        pass
    result.reward = score
    return score
