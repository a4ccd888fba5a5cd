"""The streamed accuracy checker (``techjam_b200.checker``) agrees with the
oracle's restatement of the reference criterion on CPU tensors, including
chunk boundaries, per-sample accumulation and non-finite values."""

import math

import pytest
import torch

from oracle.reference_model import check_outputs
from techjam_b200.checker import AccuracyAccumulator, compare_outputs


def _pair(seed, b=3, n=37, d=16, noise=1e-3):
    g = torch.Generator().manual_seed(seed)
    ref = torch.randn(b, n, d, generator=g)
    got = ref + noise * torch.randn(b, n, d, generator=g)
    return ref, got


@pytest.mark.parametrize("chunk", [1, 5, 37, 4096])
def test_matches_oracle_checker(chunk):
    ref, got = _pair(0, noise=3e-3)
    got[1, 7, 3] += 0.5  # one clear failure
    mine = compare_outputs(ref, got, token_chunk=chunk)
    theirs = check_outputs(ref, got)
    assert mine.passed == theirs.passed is False
    assert mine.failed_elements == theirs.failed_elements
    assert mine.total_elements == theirs.total_elements == ref.numel()
    assert mine.max_abs_error == pytest.approx(theirs.max_abs_error, rel=1e-6)
    assert mine.max_relative_error == pytest.approx(theirs.max_relative_error, rel=1e-6)
    assert mine.mean_abs_error == pytest.approx(theirs.mean_abs_error, rel=1e-6)
    assert mine.worst_index == (1, 7, 3)
    assert 3 in mine.failed_feature_dims
    assert mine.optimized_at_worst - mine.reference_at_worst == pytest.approx(got[1, 7, 3] - ref[1, 7, 3])


def test_or_criterion_exactly():
    ref = torch.tensor([[[1.0, 1.0, 0.01, 100.0]]])
    # |err| = 0.002 passes by atol; 0.0021 on |ref|=0.01 fails both; 2.0 on 100 passes by rtol
    got = torch.tensor([[[1.002, 1.0, 0.0121, 102.0]]])
    r = compare_outputs(ref, got)
    assert r.failed_elements == 1 and r.failed_feature_dims == [2]


def test_accumulated_samples_equal_one_shot():
    ref, got = _pair(1, b=4, n=50, d=8, noise=2e-3)
    acc = AccuracyAccumulator(token_chunk=16)
    for i in range(4):
        acc.add(ref[i:i + 1], got[i:i + 1], batch_offset=i)
    a, b = acc.result(), compare_outputs(ref, got)
    assert (a.failed_elements, a.total_elements, a.worst_index) == (b.failed_elements, b.total_elements,
                                                                     b.worst_index)
    assert a.max_abs_error == b.max_abs_error
    assert a.mean_abs_error == pytest.approx(b.mean_abs_error, rel=1e-12)


def test_non_finite_values_fail():
    ref, got = _pair(2, noise=1e-4)
    got[0, 0, 0] = float("nan")
    got[2, 5, 1] = float("inf")
    r = compare_outputs(ref, got, token_chunk=8)
    assert not r.passed and r.failed_elements == 2
    assert math.isnan(r.max_abs_error) and r.worst_index == (0, 0, 0)


def test_shape_errors_and_empty():
    with pytest.raises(AssertionError):
        compare_outputs(torch.zeros(1, 2, 3), torch.zeros(1, 3, 3))
    with pytest.raises(ValueError):
        compare_outputs(torch.zeros(2, 3), torch.zeros(2, 3))
    with pytest.raises(ValueError):
        AccuracyAccumulator(rtol=-1.0)
    r = compare_outputs(torch.zeros(0, 4, 3), torch.zeros(0, 4, 3))
    assert r.passed and r.total_elements == 0
