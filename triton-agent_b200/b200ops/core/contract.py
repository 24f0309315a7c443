"""contract.yaml schema -> dataclasses.

Same schema and field names as the reference (triton_agent/core/contract.py:
13-175) so existing contract files load unchanged.  Two additions, both
optional: `tolerance` accepts `max_rel_error` (element passes when
|out - ref| <= max_abs_error + max_rel_error * |ref|) and `exact` (bit
equality), and `search_space` keeps every key it is given -- the CUDA launch
and tile parameters (threads, split, stages, tile_n, ...) as well as the
reference's BLOCK_D / num_warps / num_stages / vectorize -- instead of
silently dropping unknown keys (the reference's SearchSpace.from_raw reads
only four of them, core/contract.py:62-69).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import yaml


class ContractError(Exception):
    """Contract file missing, malformed, or without a required section."""


@dataclass
class ShapeSpec:
    dims: list[str]

    @classmethod
    def from_raw(cls, raw: list[str]) -> "ShapeSpec":
        return cls(dims=list(raw))


@dataclass
class InputSpec:
    name: str
    shape: ShapeSpec

    @classmethod
    def from_raw(cls, name: str, raw: list[str]) -> "InputSpec":
        return cls(name, ShapeSpec.from_raw(raw))


@dataclass
class OutputSpec:
    name: str
    shape: ShapeSpec

    @classmethod
    def from_raw(cls, name: str, raw: list[str]) -> "OutputSpec":
        return cls(name, ShapeSpec.from_raw(raw))


@dataclass
class ToleranceSpec:
    max_abs_error: float
    mean_abs_error: float
    max_rel_error: float | None = None
    exact: bool = False

    @classmethod
    def from_raw(cls, raw: dict) -> "ToleranceSpec":
        rel = raw.get("max_rel_error")
        return cls(
            max_abs_error=float(raw["max_abs_error"]),
            mean_abs_error=float(raw["mean_abs_error"]),
            max_rel_error=None if rel is None else float(rel),
            exact=bool(raw.get("exact", False)),
        )

    def to_dict(self) -> dict[str, Any]:
        d: dict[str, Any] = {"max_abs_error": self.max_abs_error, "mean_abs_error": self.mean_abs_error}
        if self.max_rel_error is not None:
            d["max_rel_error"] = self.max_rel_error
        if self.exact:
            d["exact"] = True
        return d


_LEGACY_DEFAULTS: dict[str, list] = {
    "BLOCK_D": [64, 128, 256, 512],
    "num_warps": [1, 2, 4, 8],
    "num_stages": [3, 4],
    "vectorize": [True, False],
}


@dataclass
class SearchSpace:
    """Tunable parameters.  The four legacy fields keep the reference's
    defaults; `cuda` holds every other key of the YAML section (the CUDA
    launch/tile parameters of b200_launch_cfg)."""

    BLOCK_D: list[int] = field(default_factory=lambda: list(_LEGACY_DEFAULTS["BLOCK_D"]))
    num_warps: list[int] = field(default_factory=lambda: list(_LEGACY_DEFAULTS["num_warps"]))
    num_stages: list[int] = field(default_factory=lambda: list(_LEGACY_DEFAULTS["num_stages"]))
    vectorize: list[bool] = field(default_factory=lambda: list(_LEGACY_DEFAULTS["vectorize"]))
    cuda: dict[str, list] = field(default_factory=dict)

    @classmethod
    def from_raw(cls, raw: dict) -> "SearchSpace":
        raw = dict(raw or {})
        legacy = {k: list(raw.pop(k, v)) for k, v in _LEGACY_DEFAULTS.items()}
        cuda = {k: list(v) if isinstance(v, (list, tuple)) else [v] for k, v in raw.items()}
        return cls(**legacy, cuda=cuda)

    def to_dict(self) -> dict[str, Any]:
        d = {"BLOCK_D": self.BLOCK_D, "num_warps": self.num_warps, "num_stages": self.num_stages,
             "vectorize": self.vectorize}
        d.update(self.cuda)
        return d


@dataclass
class BenchmarkSpec:
    warmup: int = 20
    repeat: int = 100
    metric: str = "latency_us_p50"

    @classmethod
    def from_raw(cls, raw: dict) -> "BenchmarkSpec":
        raw = raw or {}
        return cls(int(raw.get("warmup", 20)), int(raw.get("repeat", 100)), str(raw.get("metric", "latency_us_p50")))


@dataclass
class PromotionSpec:
    min_speedup: float = 1.05
    max_variance: float = 0.10
    regression_required: bool = True

    @classmethod
    def from_raw(cls, raw: dict) -> "PromotionSpec":
        raw = raw or {}
        return cls(float(raw.get("min_speedup", 1.05)), float(raw.get("max_variance", 0.10)),
                   bool(raw.get("regression_required", True)))


@dataclass
class OpContract:
    op: str
    inputs: list[InputSpec]
    outputs: list[OutputSpec]
    dtype: list[str]
    device: list[str]
    tolerance: ToleranceSpec
    search_space: SearchSpace
    benchmark: BenchmarkSpec
    promotion: PromotionSpec

    @classmethod
    def from_dict(cls, data: dict) -> "OpContract":
        try:
            return cls(
                op=data["op"],
                inputs=[InputSpec.from_raw(n, s) for n, s in data["inputs"].items()],
                outputs=[OutputSpec.from_raw(n, s) for n, s in data["outputs"].items()],
                dtype=list(data.get("dtype", [])),
                device=list(data.get("device", [])),
                tolerance=ToleranceSpec.from_raw(data["tolerance"]),
                search_space=SearchSpace.from_raw(data.get("search_space", {})),
                benchmark=BenchmarkSpec.from_raw(data.get("benchmark", {})),
                promotion=PromotionSpec.from_raw(data.get("promotion", {})),
            )
        except KeyError as e:
            raise ContractError(f"Missing required field: {e}") from e

    @classmethod
    def from_yaml(cls, path: str | Path) -> "OpContract":
        path = Path(path)
        if not path.exists():
            raise ContractError(f"Contract file not found: {path}")
        data = yaml.safe_load(path.read_text(encoding="utf-8"))
        if not isinstance(data, dict):
            raise ContractError(f"Invalid contract YAML: expected dict, got {type(data)}")
        return cls.from_dict(data)

    def to_dict(self) -> dict[str, Any]:
        return {
            "op": self.op,
            "inputs": {i.name: i.shape.dims for i in self.inputs},
            "outputs": {o.name: o.shape.dims for o in self.outputs},
            "dtype": self.dtype,
            "device": self.device,
            "tolerance": self.tolerance.to_dict(),
            "search_space": self.search_space.to_dict(),
            "benchmark": {"warmup": self.benchmark.warmup, "repeat": self.benchmark.repeat,
                          "metric": self.benchmark.metric},
            "promotion": {"min_speedup": self.promotion.min_speedup, "max_variance": self.promotion.max_variance,
                          "regression_required": self.promotion.regression_required},
        }
