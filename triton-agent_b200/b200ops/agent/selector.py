"""Best candidate by reward, ties broken by lower p50 latency
(triton_agent/agent/selector.py:9-31)."""

from __future__ import annotations

from typing import Any

from ..core.spec import CandidateResult


def select_best(candidates: list[Any], results: list[CandidateResult]) -> tuple[int, CandidateResult]:
    best = 0
    for i in range(1, len(results)):
        r, b = results[i], results[best]
        if r.reward > b.reward or (r.reward == b.reward and r.latency_us_p50 < b.latency_us_p50):
            best = i
    return best, results[best]
