"""Paired-timing statistics (``techjam_b200.timing``) against the behaviour the
reference pins in ``src/tests/test_timing.py``: balanced AB/BA schedule, drift
cancellation, deferred resolution of device samples, a noise floor taken from
per-pair disagreement, block sizing and settling.  Host-only."""

import statistics

import pytest

from techjam_b200 import timing
from techjam_b200.timing import BASELINE, CANDIDATE


def drifting(baseline_ms, candidate_ms, final_multiplier, total):
    """Fake runners whose latency grows linearly over the run (boost decay)."""
    state = {"n": 0}

    def mult():
        m = 1.0 + (final_multiplier - 1.0) * state["n"] / max(1, total - 1)
        state["n"] += 1
        return m

    return {BASELINE: lambda: baseline_ms * mult(), CANDIDATE: lambda: candidate_ms * mult()}


def test_schedule_counts_and_balanced_positions():
    s = timing.paired_schedule(64)
    assert s.count(BASELINE) == s.count(CANDIDATE) == 64
    pos_b = [i for i, v in enumerate(s) if v == BASELINE]
    pos_c = [i for i, v in enumerate(s) if v == CANDIDATE]
    assert statistics.mean(pos_b) == pytest.approx(statistics.mean(pos_c), abs=1e-12)
    assert s[:4] == [BASELINE, CANDIDATE, CANDIDATE, BASELINE]
    with pytest.raises(ValueError, match="repeats"):
        timing.paired_schedule(0)


@pytest.mark.parametrize("cand,expected", [(80.0, 1.25), (100.0, 1.0)])
def test_two_fold_drift_cancels(cand, expected):
    r = 200
    summary = timing.paired_summary(timing.measure_pair(drifting(100.0, cand, 2.0, 2 * r), r))
    assert summary["speedup"] == pytest.approx(expected, abs=0.02 if expected != 1.0 else 0.01)


def test_unpaired_schedule_would_be_fooled():
    """Sanity check of the fake: all baselines first, then all candidates,
    reports a large fabricated slowdown of the candidate."""
    r = 200
    run = drifting(100.0, 100.0, 2.0, 2 * r)
    b = [run[BASELINE]() for _ in range(r)]
    c = [run[CANDIDATE]() for _ in range(r)]
    assert statistics.median(b) / statistics.median(c) < 0.8


class Pending:
    def __init__(self, value, log):
        self.value, self.log = value, log

    def milliseconds(self):
        self.log.append("resolve")
        return self.value


def test_samples_resolve_only_after_all_are_recorded():
    log = []

    def runner():
        log.append("record")
        return Pending(1.0, log)

    out = timing.measure_pair({BASELINE: runner, CANDIDATE: runner}, repeats=3)
    assert log == ["record"] * 6 + ["resolve"] * 6
    assert out[BASELINE] == [1.0] * 3 and out[CANDIDATE] == [1.0] * 3


def test_missing_runner_is_an_error():
    with pytest.raises(KeyError):
        timing.measure_pair({BASELINE: lambda: 1.0}, 2)


def test_noise_floor_zero_for_noiseless_ratio_despite_drift():
    r = 100
    samples = timing.measure_pair(drifting(100.0, 50.0, 2.0, 2 * r), r)
    # the within-pair ratio moves only by the drift between two adjacent samples
    assert timing.noise_floor_ratio(samples) < 0.002
    raw_cv = statistics.stdev(samples[BASELINE]) / statistics.mean(samples[BASELINE])
    assert raw_cv > 0.15  # raw spread would have charged the drift to the floor


def test_noise_floor_from_ratio_spread():
    samples = {BASELINE: [10.0, 12.0, 10.0, 12.0], CANDIDATE: [10.0, 10.0, 10.0, 10.0]}
    ratios = [1.0, 1.2, 1.0, 1.2]
    expected = 1.96 * 1.2533141373155 * statistics.stdev(ratios) / 2.0
    assert timing.noise_floor_ratio(samples) == pytest.approx(expected, rel=1e-9)
    assert timing.noise_floor_ratio({BASELINE: [1.0], CANDIDATE: [1.0]}) == float("inf")
    assert timing.is_significant(1.10, 0.05) and not timing.is_significant(1.03, 0.05)
    assert timing.is_significant(0.90, 0.05)


def test_block_size():
    assert timing.choose_block_size(100.0) == 1
    assert timing.choose_block_size(5.0) == 10
    assert timing.choose_block_size(0.01) == 200
    assert timing.choose_block_size(0.01, maximum=50) == 50
    with pytest.raises(ValueError):
        timing.choose_block_size(0.0)


def test_host_block_runner_and_settle():
    calls = []
    model = lambda x, m: calls.append(1)
    run = timing.make_block_runner(model, None, None, None, block_size=5)
    ms = run()
    assert len(calls) == 5 and ms >= 0.0
    with pytest.raises(ValueError):
        timing.make_block_runner(model, None, None, None, block_size=0)
    calls.clear()
    n = timing.settle(model, None, None, None, seconds=0.0, chunk=3)
    assert n == 3 and len(calls) == 3
    with pytest.raises(ValueError):
        timing.settle(model, None, None, None, seconds=-1.0)


def test_percentile_and_summary():
    assert timing.percentile([3.0], 0.9) == 3.0
    assert timing.percentile([1.0, 2.0, 3.0, 4.0, 5.0], 0.9) == pytest.approx(4.6)
    s = timing.timing_summary([4.0, 1.0, 3.0, 2.0])
    assert s["median_ms"] == 2.5 and s["min_ms"] == 1.0 and s["mean_ms"] == 2.5
    with pytest.raises(ValueError):
        timing.percentile([], 0.5)
