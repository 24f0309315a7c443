"""Factory protocol of a CUDA variant.

The reference's pipeline calls `template(**compile_args)` and then
`kernel_fn(*inputs)` (triton_agent/core/compiler.py:37, cli.py:252,911).
compile_args carries shape keys (B, T, D, H) and the Triton-era keys
(BLOCK_SIZE, NUM_WARPS, NUM_STAGES); the tuner adds the CUDA launch keys of
b200_launch_cfg.  make_factory maps them onto a b200_launch_cfg dict and
returns a callable that runs the op on its inputs with that config.
"""

from __future__ import annotations

from typing import Callable

_CFG_KEYS = ("threads", "rows_per_cta", "stages", "split", "tile_m", "tile_n", "tile_k", "flags")


def launch_cfg_from_args(compile_args: dict) -> dict[str, int]:
    cfg = {k: int(compile_args[k]) for k in _CFG_KEYS if compile_args.get(k)}
    if "stages" not in cfg and compile_args.get("NUM_STAGES"):
        cfg["stages"] = int(compile_args["NUM_STAGES"])
    if "threads" not in cfg and compile_args.get("NUM_WARPS"):
        cfg["threads"] = 32 * int(compile_args["NUM_WARPS"])
    return cfg


def make_factory(run: Callable, uses_threads: bool = True) -> Callable:
    def factory(**compile_args):
        cfg = launch_cfg_from_args(compile_args)
        if not uses_threads:
            cfg.pop("threads", None)
        for k, v in cfg.items():
            if v < 0:
                raise ValueError(f"launch parameter {k} must be >= 0")

        def kernel_fn(*inputs):
            return run(*inputs, cfg=cfg or None)

        kernel_fn.launch_cfg = cfg
        return kernel_fn

    return factory
