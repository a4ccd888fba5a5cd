"""The product-side checker and paired-timing statistics against the
reference's own outputs (``tests/golden/checker.*``, written by
``make_golden.py`` from ``torch_transformer_benchmark.compare_outputs`` /
``percentile`` and ``src/infra/timing.py``).  CPU only."""

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from techjam_b200 import timing
from techjam_b200.checker import compare_outputs

GOLDEN = Path(__file__).resolve().parent / "golden"
DATA = np.load(GOLDEN / "checker.npz")
META = json.loads((GOLDEN / "checker.json").read_text())


def _same(a, b):
    return (math.isnan(a) and math.isnan(b)) or a == b


@pytest.mark.parametrize("name", sorted(META["verdicts"]))
@pytest.mark.parametrize("chunk", [1, 2, 4096])
def test_checker_matches_reference_verdict(name, chunk):
    want = META["verdicts"][name]
    ref = torch.from_numpy(DATA[f"{name}_ref"])
    cand = torch.from_numpy(DATA[f"{name}_cand"])
    got = compare_outputs(ref, cand, rtol=0.02, atol=0.002, token_chunk=chunk)
    assert got.passed == want["passed"]
    assert got.total_elements == want["total_elements"]
    assert got.failed_elements == want["failed_elements"]
    assert got.failed_feature_dims == want["failed_feature_dims"]
    assert list(got.worst_index) == want["worst_index"]
    assert _same(got.max_abs_error, want["max_abs_error"])
    assert _same(got.max_relative_error, want["max_relative_error"])
    assert _same(got.reference_at_worst, want["reference_at_worst"])
    assert _same(got.optimized_at_worst, want["optimized_at_worst"])
    if math.isfinite(want["mean_abs_error"]):
        assert got.mean_abs_error == pytest.approx(want["mean_abs_error"], rel=1e-5)
    else:
        assert not math.isfinite(got.mean_abs_error)


def test_timing_statistics_match_reference():
    t = META["timing"]
    for q, v in t["percentile"].items():
        assert timing.percentile([3.0, 1.0, 4.0, 1.5, 9.0, 2.6], float(q)) == pytest.approx(v, abs=1e-12)
    assert timing.paired_schedule(5) == t["paired_schedule_5"]
    s = t["samples"]
    assert timing.paired_summary(s) == pytest.approx(t["paired_summary"], rel=1e-12)
    assert timing.paired_ratios(s) == pytest.approx(t["paired_ratios"], rel=1e-12)
    assert timing.noise_floor_ratio(s) == pytest.approx(t["noise_floor_ratio"], rel=1e-4)
    for ms, blocks in t["choose_block_size"].items():
        assert timing.choose_block_size(float(ms)) == blocks
