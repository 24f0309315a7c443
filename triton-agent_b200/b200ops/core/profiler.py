"""Latency profiler (fields of triton_agent/core/profiler.py:9-71).

The reference times each call with host perf_counter around a device
synchronize, which folds launch overhead and host jitter into every sample.
Here each iteration is timed on the device with CUDA events recorded on the
launching stream; with `flush_l2` a buffer larger than L2 is overwritten
and then read back between iterations, so memory-bound kernels are not served
from cache and the timed call does not pay for writing back the flush's
dirty lines (the read evicts them before the start event).
Reported fields are unchanged: p50/p90/p99 in microseconds, variance as the
coefficient of variation, speedup against baseline_latency_us, and the peak
allocated memory.
"""

from __future__ import annotations

from typing import Any, Callable

from .spec import CandidateResult

L2_FLUSH_BYTES = 256 * 1024 * 1024  # > 126 MB L2 of a B200


def _quantile(sorted_vals: list[float], q: float) -> float:
    if not sorted_vals:
        return 0.0
    pos = q * (len(sorted_vals) - 1)
    lo = int(pos)
    hi = min(lo + 1, len(sorted_vals) - 1)
    return sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (pos - lo)


def time_device(fn: Callable[[], Any], warmup: int = 20, repeat: int = 100, flush_l2: bool = False,
                device=None) -> list[float]:
    """Per-iteration device times in microseconds (CUDA events, current stream)."""
    import torch

    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev) if flush_l2 else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(repeat)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(repeat)]
    for i in range(repeat):
        if flush is not None:
            flush.fill_(float(i))
            flush.sum()  # leaves L2 holding clean lines of the flush buffer
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    return [s.elapsed_time(e) * 1e3 for s, e in zip(starts, ends)]


def profile_kernel(kernel_fn: Callable, input_args: tuple, kwargs: dict[str, Any] | None = None, warmup: int = 20,
                   repeat: int = 100, baseline_latency_us: float = 0.0, flush_l2: bool = False) -> CandidateResult:
    import torch

    res = CandidateResult(compile_pass=True, verify_pass=True)
    kwargs = kwargs or {}
    try:
        lat = time_device(lambda: kernel_fn(*input_args, **kwargs), warmup, repeat, flush_l2)
    except Exception as e:
        res.compile_pass = False
        res.compile_log = str(e)
        return res
    lat.sort()
    res.latency_us_p50 = _quantile(lat, 0.5)
    res.latency_us_p90 = _quantile(lat, 0.9)
    res.latency_us_p99 = _quantile(lat, 0.99)
    mean = sum(lat) / len(lat)
    sd = (sum((x - mean) ** 2 for x in lat) / max(1, len(lat) - 1)) ** 0.5
    res.variance = sd / (mean + 1e-12)
    res.speedup = baseline_latency_us / (res.latency_us_p50 + 1e-12) if baseline_latency_us > 0 else 1.0
    try:
        res.memory_peak_mb = torch.cuda.max_memory_allocated() / (1024 * 1024)
    except Exception:
        res.memory_peak_mb = 0.0
    return res
