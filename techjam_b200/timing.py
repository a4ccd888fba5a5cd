"""Paired A/B timing with drift cancellation, restating the reference's
``src/infra/timing.py:23-230`` so that speedups measured here use the same
statistics as the reference's published ones.

A GPU's clock drifts while a benchmark runs: boost budget is spent in wall
time, and a 1 kW part settles under its power cap.  Timing one implementation
before the other therefore favours whichever runs first.  The schedule here
interleaves the two sides as ``AB BA AB BA ...``; both sides then have the same
mean position in the run, and monotonic drift cancels in the medians.  The
noise floor is computed from the per-pair ratios (each pair is measured
microseconds apart under the same clock), not from the raw spread, which
includes the drift the schedule already removed.

Device samples are CUDA event pairs that stay pending until every sample is
recorded; one synchronise resolves them.  A synchronise per sample would idle
the GPU between samples and let its clocks climb back, which is exactly the
drift this module exists to control.
"""

from __future__ import annotations

import math
import statistics
import time
from typing import Any, Callable, Dict, List, Mapping, Sequence

BASELINE = "baseline"
CANDIDATE = "candidate"

Runner = Callable[[], Any]


def paired_schedule(repeats: int) -> List[str]:
    """``repeats`` samples per side, pairs alternating AB / BA
    (reference ``timing.py:23-37``)."""
    if repeats <= 0:
        raise ValueError(f"repeats must be positive, got {repeats}")
    order = (BASELINE, CANDIDATE)
    out: List[str] = []
    for i in range(repeats):
        out += order if i % 2 == 0 else order[::-1]
    return out


def resolve_sample(sample: Any) -> float:
    """A sample is a float (host timer) or an object whose ``milliseconds()``
    reads a recorded device timer."""
    read = getattr(sample, "milliseconds", None)
    return float(read()) if callable(read) else float(sample)


def _is_cuda(device: Any) -> bool:
    return device is not None and getattr(device, "type", None) == "cuda"


def measure_pair(runners: Mapping[str, Runner], repeats: int, device: Any = None) -> Dict[str, List[float]]:
    """Run the paired schedule; return per-side milliseconds in schedule order
    (reference ``timing.py:46-69``).  Every sample is issued before any is
    resolved, with one device synchronise in between."""
    absent = sorted({BASELINE, CANDIDATE} - set(runners))
    if absent:
        raise KeyError(f"runners must provide {absent}")
    issued: Dict[str, List[Any]] = {BASELINE: [], CANDIDATE: []}
    for side in paired_schedule(repeats):
        issued[side].append(runners[side]())
    if _is_cuda(device):
        import torch

        torch.cuda.synchronize(device)
    return {side: [resolve_sample(s) for s in samples] for side, samples in issued.items()}


def paired_summary(samples: Mapping[str, Sequence[float]]) -> Dict[str, float]:
    """Medians, minima and the median speedup baseline/candidate
    (reference ``timing.py:72-82``)."""
    b_med = statistics.median(samples[BASELINE])
    c_med = statistics.median(samples[CANDIDATE])
    return {
        "baseline_median_ms": b_med,
        "candidate_median_ms": c_med,
        "baseline_min_ms": min(samples[BASELINE]),
        "candidate_min_ms": min(samples[CANDIDATE]),
        "speedup": b_med / c_med,
    }


def paired_ratios(samples: Mapping[str, Sequence[float]]) -> List[float]:
    """baseline/candidate within each schedule pair (reference ``timing.py:85-94``)."""
    b, c = samples[BASELINE], samples[CANDIDATE]
    return [b[i] / c[i] for i in range(min(len(b), len(c)))]


# The standard error of a sample median is sqrt(pi/2) ~= 1.2533 times that of
# the mean for normally distributed data; 1.96 is the two-sided 95% z value.
_MEDIAN_SE_FACTOR = math.sqrt(math.pi / 2.0)
_Z95 = 1.96


def noise_floor_ratio(samples: Mapping[str, Sequence[float]]) -> float:
    """Half-width of the 95% interval of the speedup, from the spread of the
    per-pair ratios (reference ``timing.py:97-113``); ``inf`` with < 2 pairs."""
    r = paired_ratios(samples)
    if len(r) < 2:
        return float("inf")
    return _Z95 * _MEDIAN_SE_FACTOR * statistics.stdev(r) / math.sqrt(len(r))


def is_significant(speedup: float, noise_floor: float) -> bool:
    """A speedup counts only outside the run's own noise band (reference ``timing.py:116-118``)."""
    return abs(speedup - 1.0) > noise_floor


def choose_block_size(per_iteration_ms: float, target_ms: float = 50.0, maximum: int = 200) -> int:
    """Forward passes per timed sample so one sample covers ~``target_ms``
    (launch-bound shapes average away per-call host jitter; reference
    ``timing.py:120-134``)."""
    if per_iteration_ms <= 0:
        raise ValueError(f"per_iteration_ms must be positive, got {per_iteration_ms}")
    return min(max(1, round(target_ms / per_iteration_ms)), maximum)


class PendingCudaSample:
    """A recorded event pair over ``block`` forwards; read after the final synchronise."""

    __slots__ = ("start", "end", "block")

    def __init__(self, start: Any, end: Any, block: int) -> None:
        self.start, self.end, self.block = start, end, block

    def milliseconds(self) -> float:
        return self.start.elapsed_time(self.end) / self.block


def make_block_runner(model: Any, x: Any, valid_mask: Any, device: Any, block_size: int = 1) -> Runner:
    """A runner timing ``block_size`` forwards per sample, reported per forward
    (reference ``timing.py:162-197``).  On CUDA it records events on the current
    stream and returns a pending sample; on the host it returns milliseconds."""
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")
    if _is_cuda(device):
        import torch

        def cuda_runner() -> PendingCudaSample:
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            with torch.inference_mode():
                start.record()
                for _ in range(block_size):
                    model(x, valid_mask)
                end.record()
            return PendingCudaSample(start, end, block_size)

        return cuda_runner

    def host_runner() -> float:
        t0 = time.perf_counter_ns()
        for _ in range(block_size):
            model(x, valid_mask)
        return (time.perf_counter_ns() - t0) / 1e6 / block_size

    return host_runner


def settle(model: Any, x: Any, valid_mask: Any, device: Any, seconds: float, chunk: int = 4) -> int:
    """Keep the device under load for ``seconds`` of wall time, so timing starts
    at steady-state clocks rather than inside the boost window (reference
    ``timing.py:200-230``).  Runs at least one chunk; returns the forwards run."""
    if seconds < 0:
        raise ValueError(f"seconds must be non-negative, got {seconds}")
    calls = 0
    deadline = time.perf_counter() + seconds
    while True:
        for _ in range(chunk):
            model(x, valid_mask)
        calls += chunk
        if _is_cuda(device):
            import torch

            torch.cuda.synchronize(device)
        if time.perf_counter() >= deadline:
            return calls


def percentile(values: Sequence[float], q: float) -> float:
    """Linear-interpolated percentile, q in [0, 1] (the reference's ``TimingResult.p90_ms``)."""
    if not values:
        raise ValueError("percentile of an empty sequence")
    s = sorted(values)
    pos = (len(s) - 1) * q
    lo = int(math.floor(pos))
    hi = min(lo + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (pos - lo)


def timing_summary(samples: Sequence[float]) -> Dict[str, Any]:
    """Median / mean / p90 / min of per-forward samples (``TimingResult``,
    torch_transformer_benchmark.py:440-460)."""
    return {
        "samples_ms": list(samples),
        "median_ms": statistics.median(samples),
        "mean_ms": statistics.fmean(samples),
        "p90_ms": percentile(samples, 0.90),
        "min_ms": min(samples),
    }
