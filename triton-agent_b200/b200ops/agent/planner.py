"""Search-strategy choice (triton_agent/agent/planner.py:7-25): full grid up to
64 combinations, best-of-64 sampling above that."""

from __future__ import annotations

from ..core.contract import OpContract
from ..core.spec import OpState
from .generator import _axes


def plan(contract: OpContract, state: OpState, history: list | None = None) -> dict:
    total = 1
    for _, values in _axes(contract):
        total *= len(values)
    if total <= 64:
        return {"strategy": "grid", "candidates": total}
    return {"strategy": "best_of_n", "n": 64}
