"""Repair of failed candidates from their logs (role of
triton_agent/agent/repairer.py:16-137), for CUDA launch parameters.

A failed launch reports a b200_status in its compile_log ("workspace",
"shared memory"/"unsupported", "timed out", ...).  The repair shrinks what
the status points at: pipeline depth and tile width for resource failures,
CTA size for launch failures, the KV split for workspace failures; a
numerical failure disables vectorisation and halves block_d as the
reference does.  should_retry refuses an unchanged or degenerate action.
"""

from __future__ import annotations

import json
from copy import deepcopy

from ..core.spec import CandidateResult, OpAction


def repair_action(action: OpAction, result: CandidateResult, max_block_size: int = 1024,
                  min_block_size: int = 32) -> OpAction | None:
    if result.compile_pass and result.verify_pass:
        return None
    a = deepcopy(action)
    if not result.compile_pass or "status" in result.compile_log:
        log = result.compile_log.lower()
        if "shared memory" in log or "too large" in log or "out of memory" in log or "unsupported" in log:
            a.num_stages = max(2, a.num_stages - 1)
            if a.tile_n:
                a.tile_n = 128
            a.block_d = max(min_block_size, a.block_d // 2)
        elif "register" in log or "spill" in log:
            a.block_d = max(min_block_size, a.block_d // 2)
            a.threads = max(0, a.threads // 2) if a.threads > 64 else a.threads
        elif "workspace" in log:
            a.split = 0
        elif "launch" in log or "warp" in log or "bad argument" in log:
            a.threads = 0
            a.num_warps = max(1, min(8, a.num_warps))
        else:
            a.block_d = max(min_block_size, a.block_d // 2)
        return a
    try:
        log = json.loads(result.verify_log)
    except (TypeError, ValueError):
        return a
    if log.get("has_nan") or log.get("has_inf"):
        a.vectorize = False
        a.block_d = max(min_block_size, a.block_d // 2)
        a.num_stages = max(1, a.num_stages - 1)
    elif log.get("max_abs_error", 0) > 1e-2:
        a.vectorize = False
        a.block_d = max(64, a.block_d // 2)
    elif a.vectorize:
        a.vectorize = False
    return a


def should_retry(action: OpAction | None, original: OpAction, result: CandidateResult) -> bool:
    if action is None:
        return False
    if action.arm_key() == original.arm_key():
        return False
    return action.block_d >= 32 and action.num_warps >= 1
