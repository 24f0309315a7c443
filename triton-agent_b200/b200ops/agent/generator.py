"""Candidate (template_id, OpAction) generation over a contract's search space.

Same entry points as triton_agent/agent/generator.py:10-83 (generate_grid,
generate_best_of_n).  The grid spans the reference's four legacy axes and
every CUDA axis the contract declares (threads, split, stages, tile_n, ...),
pruned by b200_query_config_space to the parameters the kernel selected for
the shape actually reads, so the tuner explores the kernel's real launch/tile
parameters and never times two identical launches.
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


def _axes(contract: OpContract, space: dict | None = None) -> list[tuple[str, list]]:
    """Search axes (OpAction field -> values) of the contract's search space.

    With `space` (b200_query_config_space of the op at this shape) the axes
    are pruned to what the selected kernel reads: a CUDA axis the kernel
    ignores collapses to its default (0), values the kernel does not accept
    are dropped, the legacy Triton axes collapse to their first value, and
    num_warps/num_stages stand for the kernel's defaults (0) unless the
    kernel reads threads/stages -- so no two arms launch the same kernel
    with the same parameters."""
    ss = contract.search_space
    axes: dict[str, list] = {}
    for key, values in ss.to_dict().items():
        field = _AXES.get(key)
        if field is None or not values:
            continue
        axes[field] = list(values)
    # Legacy axes that no CUDA variant reads collapse to one value so the
    # grid does not multiply identical launches.
    if any(k in axes for k in CUDA_FIELDS) or space is not None:
        for legacy in ("block_d", "vectorize", "num_warps"):
            if legacy in axes:
                axes[legacy] = axes[legacy][:1]
    if space is None:
        return list(axes.items())
    reads = space.get("fields", {})
    # the library's field names are b200_launch_cfg's; OpAction keeps stages in num_stages
    lib_axis = {"stages": "num_stages", **{k: k for k in CUDA_FIELDS}}
    for cfg_name, field in lib_axis.items():
        if cfg_name not in reads:
            if field in axes:
                axes[field] = [0]
            continue
        legal = list(reads[cfg_name].get("values", []))
        chosen = [v for v in axes.get(field, [0]) if v in legal] or [0]
        axes[field] = list(dict.fromkeys(chosen))
    if "threads" not in reads:
        axes["num_warps"] = [0]
    return list(axes.items())


def library_axes(space: dict) -> list[tuple[str, list]]:
    """Every value b200_query_config_space lists, on every field the kernel
    reads (the `--space library` search)."""
    lib_axis = {"stages": "num_stages", **{k: k for k in CUDA_FIELDS}}
    axes = [(lib_axis[k], list(v["values"])) for k, v in space.get("fields", {}).items() if k in lib_axis]
    names = {a for a, _ in axes}
    if "num_stages" not in names:
        axes.append(("num_stages", [0]))
    if "threads" not in names:
        axes.append(("num_warps", [0]))
    return axes


def default_action(template_id: str, axes: list[tuple[str, list]]) -> OpAction:
    """The grid arm whose launch parameters are all the kernel's defaults (0
    on every axis that offers it; first value of the legacy Triton axes): the
    configuration every tuned one is compared with."""
    legacy = ("block_d", "vectorize")
    return OpAction(template_id=template_id,
                    **{a: (v[0] if a in legacy or 0 not in v else 0) for a, v in axes})


def generate_grid(contract: OpContract, state: OpState, templates: dict[str, Any],
                  space: dict | None = None, axes: list | None = None) -> list[tuple[str, OpAction]]:
    axes = axes if axes is not None else _axes(contract, space)
    names = [a for a, _ in axes]
    out: list[tuple[str, OpAction]] = []
    for tid in templates:
        for combo in itertools.product(*[v for _, v in axes]):
            out.append((tid, OpAction(template_id=tid, **dict(zip(names, combo)))))
    return out


def generate_best_of_n(contract: OpContract, state: OpState, templates: dict[str, Any], n: int = 32,
                       seed: int | None = None, space: dict | None = None,
                       axes: list | None = None) -> list[tuple[str, OpAction]]:
    rng = random.Random(seed)
    axes = axes if axes is not None else _axes(contract, space)
    tids = list(templates)
    out = []
    for _ in range(n):
        tid = rng.choice(tids)
        out.append((tid, OpAction(template_id=tid, **{a: rng.choice(v) for a, v in axes})))
    return out
