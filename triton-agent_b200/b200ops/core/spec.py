"""OpState / OpAction / CandidateResult (triton_agent/core/spec.py:7-124).

Field names and to_dict/from_dict round trips are those of the reference.
OpAction gains the CUDA launch/tile parameters of b200_launch_cfg (threads,
rows_per_cta, split, tile_m, tile_n, tile_k, flags) with 0 = kernel default, and
CandidateResult gains roofline fields; both default so old records load.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, fields
from typing import Any


@dataclass
class OpState:
    op_name: str
    B: int
    T: int
    D: int
    dtype: str
    device: str
    gpu_name: str = ""
    baseline_latency_us: float = 0.0
    historical_best_config: dict | None = None
    # the generator's full shape ("K=V,..." in key order) for operators whose
    # shape is not B/T/D (GEMM M,N,K; paged caches; heads); empty = B/T/D only
    shape: str = ""

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "OpState":
        req = {k: data[k] for k in ("op_name", "B", "T", "D", "dtype", "device")}
        return cls(**req, gpu_name=data.get("gpu_name", ""),
                   baseline_latency_us=data.get("baseline_latency_us", 0.0),
                   historical_best_config=data.get("historical_best_config"), shape=data.get("shape", ""))


CUDA_FIELDS = ("threads", "rows_per_cta", "split", "tile_m", "tile_n", "tile_k", "flags")


@dataclass
class OpAction:
    template_id: str
    block_d: int = 128
    num_warps: int = 4
    num_stages: int = 3
    vectorize: bool = False
    fusion: bool = False
    threads: int = 0
    rows_per_cta: int = 0
    split: int = 0
    tile_m: int = 0
    tile_n: int = 0
    tile_k: int = 0
    flags: int = 0  # kernel-variant bits of the op (b200_launch_cfg.flags)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "OpAction":
        known = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in known})

    def launch_cfg(self) -> dict[str, int]:
        """b200_launch_cfg fields: explicit CUDA parameters win; otherwise
        num_stages is the pipeline depth and block_d/num_warps give the CTA
        size where the op takes one."""
        cfg = {k: getattr(self, k) for k in CUDA_FIELDS}
        cfg["stages"] = self.num_stages
        if not cfg["threads"] and self.num_warps:
            cfg["threads"] = 32 * self.num_warps
        return cfg

    def arm_key(self) -> str:
        """Stable identity of this configuration for the tuner."""
        return "|".join(str(getattr(self, f.name)) for f in fields(self) if f.name != "fusion")


@dataclass
class CandidateResult:
    compile_pass: bool = False
    verify_pass: bool = False
    latency_us_p50: float = 0.0
    latency_us_p90: float = 0.0
    latency_us_p99: float = 0.0
    speedup: float = 1.0
    variance: float = 0.0
    memory_peak_mb: float = 0.0
    reward: float = 0.0
    promoted: bool = False
    compile_log: str = ""
    verify_log: str = ""
    achieved_GBps: float = 0.0
    achieved_TOPS: float = 0.0
    roofline_fraction: float = 0.0
    num_gpus: int = 1
    cpu_baseline_us: float = 0.0
    cpu_cores: int = 0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "CandidateResult":
        known = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in known})
