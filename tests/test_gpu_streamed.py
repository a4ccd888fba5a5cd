"""Every sample of the five seeded C4 trials (B=64, N=8192; seeds 1234..1238
as src/benchmark.py:184-190 draws them) against the bounded-memory FP32
oracle, streamed one sample at a time; the five-trial C5 run uses the same
code through ``tests/streamed_validation.py``."""

import pytest

import streamed_validation

pytestmark = pytest.mark.gpu


def test_c4_five_trials_every_sample():
    report = streamed_validation.run(streamed_validation.parse_args(
        ["--config", "C4", "--trials", "5", "--validate-dense-n", "1024"]))
    assert report["dense_validation"]["status"] == "pass"
    assert [t["samples"] for t in report["trials"]] == [64] * 5
    assert report["passed"], report["trials"]
