"""The benchmark CLI with the B200 candidate on the GPU: accuracy trials pass
against the oracle as the dense baseline, and the paired schedule reports a
speedup with its noise floor."""

import json

import pytest

from techjam_b200 import benchmark

pytestmark = pytest.mark.gpu


def test_paired_cli_against_dense_baseline(tmp_path):
    out = tmp_path / "c1.json"
    rc = benchmark.main(["--workload", "C1", "--baseline-module", "oracle.reference_model:OracleEncoder",
                         "--accuracy-trials", "2", "--accuracy-precision", "fp32", "--repeats", "10",
                         "--settle-seconds", "0.5", "--output", str(out)])
    assert rc == 0
    res = json.loads(out.read_text())
    assert res["accuracy"]["passed"] and res["accuracy"]["failed_elements"] == 0
    perf = res["performance"]
    assert perf["timing_mode"] == "paired" and perf["block_size"] >= 1
    assert perf["timing_method"] == "torch.cuda.Event"
    assert perf["speedup"] > 1.0  # the dense FP32 baseline materialises [B, H, N, N] scores
    assert perf["memory"]["candidate"]["peak_allocated_bytes"] > 0
