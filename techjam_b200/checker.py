"""The reference's accuracy criterion, evaluated in bounded memory.

Restates ``compare_outputs`` (torch_transformer_benchmark.py:289-356): an
element passes iff both values are finite and ``|err| <= atol`` OR
``|err| <= rtol * |ref|`` (the exact OR, not ``torch.isclose``'s sum); a run
passes iff no element fails.  The evaluation is streamed over token chunks
and may be fed sample by sample (``AccuracyAccumulator``), as the reference's
streamed checker does for its over-size case
(src/implementations/fp32_reference.py:145-204,
src/case14_fp32_reference.py:180-230), so checking a 4 GB output needs no
full-size temporaries.  The result carries every field of the reference's
``AccuracyResult`` (:276-287).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch

DEFAULT_RTOL = 0.02   # src/benchmark.py --rtol default
DEFAULT_ATOL = 0.002  # src/benchmark.py --atol default


@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    failed_feature_dims: List[int] = field(default_factory=list)
    worst_index: Tuple[int, ...] = ()
    reference_at_worst: float = 0.0
    optimized_at_worst: float = 0.0


class AccuracyAccumulator:
    """Accumulates the criterion over pieces of one logical ``[B, N, D]`` output.

    ``add(ref, got, batch_offset)`` takes any ``[b, n, D]`` slice (a sample, a
    token chunk of it); indices in the result are in the full output's
    coordinates.  Non-finite values fail; a NaN error makes ``max_abs_error``
    NaN, as ``abs_error.max()`` does in the reference.
    """

    def __init__(self, rtol: float = DEFAULT_RTOL, atol: float = DEFAULT_ATOL, token_chunk: int = 4096) -> None:
        if rtol < 0 or atol < 0:
            raise ValueError("rtol and atol must be non-negative")
        if token_chunk <= 0:
            raise ValueError("token_chunk must be positive")
        self.rtol, self.atol, self.token_chunk = rtol, atol, token_chunk
        self.total = 0
        self.failed = 0
        self.abs_sum = 0.0
        self.max_abs = -1.0
        self.max_rel = 0.0
        self.worst: Tuple[int, ...] = ()
        self.ref_at_worst = 0.0
        self.got_at_worst = 0.0
        self.failed_dims: Optional[torch.Tensor] = None

    def add(self, reference: torch.Tensor, candidate: torch.Tensor, batch_offset: int = 0,
            token_offset: int = 0) -> None:
        if reference.shape != candidate.shape:
            raise AssertionError(f"shape mismatch: baseline={tuple(reference.shape)}, "
                                 f"optimized={tuple(candidate.shape)}")
        if reference.ndim != 3:
            raise ValueError("reference and candidate must be [B, N, D]")
        b, n, d = reference.shape
        if self.failed_dims is None:
            self.failed_dims = torch.zeros(d, dtype=torch.bool)
        if reference.numel() == 0:
            return
        for s in range(0, n, self.token_chunk):
            e = min(s + self.token_chunk, n)
            ref = reference[:, s:e].detach().float()
            got = candidate[:, s:e].detach().float()
            err = (got - ref).abs()
            finite = torch.isfinite(ref) & torch.isfinite(got)
            ok = finite & ((err <= self.atol) | (err <= self.rtol * ref.abs()))
            bad = ~ok
            self.failed += int(bad.sum().item())
            self.failed_dims |= bad.reshape(-1, d).any(dim=0).cpu()
            self.abs_sum += float(err.sum(dtype=torch.float64).item())
            # torch's max/argmax propagate NaN (a NaN error is the worst one); the
            # first NaN seen stays the worst element
            flat = int(err.reshape(-1).argmax().item())
            m = float(err.reshape(-1)[flat].item())
            if not math.isnan(self.max_abs) and (math.isnan(m) or m > self.max_abs):
                self.max_abs = m
                bi, rem = divmod(flat, (e - s) * d)
                ti, di = divmod(rem, d)
                self.worst = (batch_offset + bi, token_offset + s + ti, di)
                self.ref_at_worst = float(ref.reshape(-1)[flat].item())
                self.got_at_worst = float(got.reshape(-1)[flat].item())
            rel = err / ref.abs().clamp_min(1e-12)
            r = float(rel.max().item())
            if not math.isnan(self.max_rel) and (math.isnan(r) or r > self.max_rel):
                self.max_rel = r
        self.total += reference.numel()

    def result(self) -> AccuracyResult:
        dims = [] if self.failed_dims is None else torch.nonzero(self.failed_dims).flatten().tolist()
        return AccuracyResult(
            passed=self.failed == 0,
            total_elements=self.total,
            failed_elements=self.failed,
            max_abs_error=max(self.max_abs, 0.0) if not math.isnan(self.max_abs) else self.max_abs,
            max_relative_error=self.max_rel,
            mean_abs_error=self.abs_sum / max(self.total, 1),
            failed_feature_dims=dims,
            worst_index=self.worst,
            reference_at_worst=self.ref_at_worst,
            optimized_at_worst=self.got_at_worst,
        )


def compare_outputs(reference: torch.Tensor, candidate: torch.Tensor, rtol: float = DEFAULT_RTOL,
                    atol: float = DEFAULT_ATOL, token_chunk: int = 4096) -> AccuracyResult:
    """One-shot form: the reference's ``compare_outputs`` on ``[B, N, D]`` tensors."""
    acc = AccuracyAccumulator(rtol, atol, token_chunk)
    acc.add(reference, candidate)
    return acc.result()
