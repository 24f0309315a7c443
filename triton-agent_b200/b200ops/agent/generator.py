"""Candidate (template_id, OpAction) generation over a contract's search space.

Same entry points as triton_agent/agent/generator.py:10-83 (generate_grid,
generate_best_of_n).  The grid spans the reference's four legacy axes and
every CUDA axis the contract declares (threads, split, stages, tile_n, ...),
so the tuner explores the kernel's real launch/tile parameters.
"""

from __future__ import annotations

import itertools
import random
from typing import Any

from ..core.contract import OpContract
from ..core.spec import CUDA_FIELDS, OpAction, OpState

# contract search_space key -> OpAction field
_AXES = {"BLOCK_D": "block_d", "BLOCK_SIZE": "block_d", "num_warps": "num_warps", "num_stages": "num_stages",
         "stages": "num_stages", "vectorize": "vectorize", **{k: k for k in CUDA_FIELDS}}


def _axes(contract: OpContract) -> list[tuple[str, list]]:
    ss = contract.search_space
    axes: dict[str, list] = {}
    for key, values in ss.to_dict().items():
        field = _AXES.get(key)
        if field is None or not values:
            continue
        axes[field] = list(values)
    # Legacy axes that no CUDA variant reads collapse to one value so the
    # grid does not multiply identical launches.
    if any(k in axes for k in CUDA_FIELDS):
        for legacy in ("block_d", "vectorize", "num_warps"):
            if legacy in axes:
                axes[legacy] = axes[legacy][:1]
    return list(axes.items())


def generate_grid(contract: OpContract, state: OpState, templates: dict[str, Any]) -> list[tuple[str, OpAction]]:
    axes = _axes(contract)
    names = [a for a, _ in axes]
    out: list[tuple[str, OpAction]] = []
    for tid in templates:
        for combo in itertools.product(*[v for _, v in axes]):
            out.append((tid, OpAction(template_id=tid, **dict(zip(names, combo)))))
    return out


def generate_best_of_n(contract: OpContract, state: OpState, templates: dict[str, Any], n: int = 32,
                       seed: int | None = None) -> list[tuple[str, OpAction]]:
    rng = random.Random(seed)
    axes = _axes(contract)
    tids = list(templates)
    out = []
    for _ in range(n):
        tid = rng.choice(tids)
        out.append((tid, OpAction(template_id=tid, **{a: rng.choice(v) for a, v in axes})))
    return out
