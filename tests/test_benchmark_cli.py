"""The benchmark CLI (``techjam_b200.benchmark``) on the CPU.

A stand-in candidate whose factory builds the oracle encoder makes the
accuracy trials exact, so these tests check the harness itself: shape
resolution, weight copy, the accuracy loop and its exit code, both timing
schedules, the per-sample baseline and the result file.  The GPU run against
the B200 candidate is in ``test_gpu_benchmark_cli.py``.
"""

import json
import sys
import types

import pytest
import torch

from oracle.reference_model import OracleEncoder
from techjam_b200 import benchmark
from techjam_b200.candidate import CandidateSpec

SMALL = ["--device", "cpu", "--batch-size", "2", "--seq-len", "16", "--d-model", "32", "--heads", "4",
         "--ffn-dim", "64", "--layers", "1", "--causal", "--padding-ratio", "0.5", "--accuracy-trials", "2",
         "--repeats", "4", "--settle-seconds", "0", "--block-size", "1"]
BASE = ["--baseline-module", "oracle.reference_model:OracleEncoder"]


class _Perturbed(OracleEncoder):
    def forward(self, x, valid_token_mask=None):
        return super().forward(x, valid_token_mask) * 1.01 + 0.01


@pytest.fixture(autouse=True, scope="module")
def _stand_in_candidates():
    pkg = types.ModuleType("tjclitest")
    pkg.__path__ = []
    mod = types.ModuleType("tjclitest.cands")
    mod.CANDIDATE = CandidateSpec(name="oracle-copy", model_factory=OracleEncoder, owner="tests",
                                  description="oracle encoder as a CPU stand-in candidate")
    mod.BROKEN = CandidateSpec(name="perturbed", model_factory=_Perturbed, owner="tests", description="fails")
    mod.NOT_A_SPEC = 42
    sys.modules["tjclitest"], sys.modules["tjclitest.cands"] = pkg, mod
    yield
    sys.modules.pop("tjclitest.cands", None)
    sys.modules.pop("tjclitest", None)


def test_paired_run_writes_result(tmp_path, capsys):
    out = tmp_path / "r.json"
    rc = benchmark.main(["--candidate", "tjclitest.cands", *BASE, *SMALL, "--output", str(out)])
    assert rc == 0
    res = json.loads(out.read_text())
    acc, perf = res["accuracy"], res["performance"]
    assert acc["passed"] and acc["failed_elements"] == 0 and len(acc["trials"]) == 2
    assert acc["max_abs_error"] == 0.0  # same weights, same arithmetic
    assert acc["trials"][1]["seed"] == 1235
    assert perf["timing_mode"] == "paired" and perf["block_size"] == 1
    assert len(perf["baseline"]["samples_ms"]) == len(perf["candidate"]["samples_ms"]) == 4
    assert perf["speedup"] > 0 and perf["noise_floor_ratio"] >= 0
    assert res["config"]["causal"] is True and res["baseline"]["mode"] == "batch"
    assert "accuracy 02/2: PASS" in capsys.readouterr().out
    with pytest.raises(FileExistsError):  # never overwrites
        benchmark.main(["--candidate", "tjclitest.cands", *BASE, *SMALL, "--output", str(out)])


def test_failing_candidate_skips_timing(capsys):
    rc = benchmark.main(["--candidate", "tjclitest.cands:BROKEN", *BASE, *SMALL])
    assert rc == 2
    assert "benchmark skipped because correctness failed" in capsys.readouterr().out


def test_legacy_schedule_and_per_sample_baseline(tmp_path):
    out = tmp_path / "legacy.json"
    rc = benchmark.main(["--candidate", "tjclitest.cands", *BASE, *SMALL, "--timing", "legacy", "--warmup", "1",
                         "--benchmark-rounds", "2", "--baseline-per-sample", "on", "--output", str(out)])
    assert rc == 0
    res = json.loads(out.read_text())
    assert res["baseline"]["mode"] == "per-sample"
    assert res["accuracy"]["max_abs_error"] == 0.0
    perf = res["performance"]
    assert perf["timing_mode"] == "legacy" and len(perf["candidate"]["samples_ms"]) == 2 * 4


def test_shape_resolution():
    args = benchmark.parse_args(["--workload", "C2"])
    cfg, scale = benchmark.resolve_shape(args)
    assert (cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers) == \
        (16, 2048, 1024, 16, 4096, 4)
    assert args.padding_ratio == 0.5 and scale == 1.0
    cfg, scale = benchmark.resolve_shape(benchmark.parse_args(["--workload", "C5"]))
    assert scale == 0.5 and cfg.seq_len == 262144
    cfg, _ = benchmark.resolve_shape(benchmark.parse_args(["--case", "13"]))
    assert (cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads) == (64, 1024, 128, 4) and cfg.causal
    cfg, _ = benchmark.resolve_shape(benchmark.parse_args([]))
    assert (cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_layers, cfg.causal) == (8, 128, 512, 6, False)
    with pytest.raises(ValueError, match="fixes --seq-len"):
        benchmark.resolve_shape(benchmark.parse_args(["--workload", "C1", "--seq-len", "64"]))
    with pytest.raises(ValueError, match="mutually exclusive"):
        benchmark.resolve_shape(benchmark.parse_args(["--workload", "C1", "--case", "2"]))
    with pytest.raises(ValueError, match="padding_ratio"):
        benchmark.resolve_shape(benchmark.parse_args(["--padding-ratio", "1.0"]))


def test_loaders_and_baseline_modes(tmp_path):
    assert benchmark.load_candidate("dispatcher").name == "b200"  # short name under techjam_b200
    with pytest.raises(AttributeError):
        benchmark.load_candidate("tjclitest.cands:NOPE")
    with pytest.raises(TypeError):
        benchmark.load_candidate("tjclitest.cands:NOT_A_SPEC")
    src = tmp_path / "my_baseline.py"
    src.write_text("import torch.nn as nn\nclass BaselineTransformer(nn.Module):\n    pass\n")
    assert benchmark.load_baseline_class(str(src)).__name__ == "BaselineTransformer"
    assert benchmark.load_baseline_class("oracle.reference_model:OracleEncoder") is OracleEncoder
    # dense scores of the 262k-token workload cannot exist; a C4 sample can
    c5, _ = benchmark.resolve_shape(benchmark.parse_args(["--workload", "C5"]))
    c4, _ = benchmark.resolve_shape(benchmark.parse_args(["--workload", "C4"]))
    assert benchmark.dense_score_bytes(c5, 1) > 8e12
    assert benchmark.dense_score_bytes(c4, 1) < 10e9 < benchmark.dense_score_bytes(c4, 64)
    args = benchmark.parse_args([])
    assert benchmark.baseline_mode(args, c4, torch.device("cpu")) == "per-sample"


def test_candidate_contract_checked_before_allocation():
    from techjam_b200.candidate import validate_candidate_execution

    spec = CandidateSpec(name="c", model_factory=OracleEncoder, owner="t", description="d",
                         unsupported_official_cases=(6,), official_case_dtypes=((8, ("float16",)),),
                         candidate_only_official_cases=(14,), default_input_scale_only_cases=(13,),
                         cuda_only_official_cases=(12,), official_case_min_cuda_capability=((11, (10, 0)),),
                         official_case_torch_versions=((10, ("2.13.0",)),), self_compiling=True)
    spec.validate()
    validate_candidate_execution(spec, None)
    validate_candidate_execution(spec, 8, dtype_name="float16")
    for case, kwargs, what in [(6, {}, "does not support"), (8, {"dtype_name": "float32"}, "only with float16"),
                               (14, {}, "no runnable dense baseline"), (13, {"input_scale": 2.0}, "input scale"),
                               (12, {"device_type": "cpu"}, "requires CUDA"),
                               (11, {"cuda_capability": (9, 0)}, "capability"),
                               (10, {"torch_version": "2.11.0"}, "requires PyTorch"),
                               (1, {"compile_user": True}, "compiles itself")]:
        with pytest.raises(ValueError, match=what):
            validate_candidate_execution(spec, case, **kwargs)
    validate_candidate_execution(spec, 11, cuda_capability=(10, 0))


def test_cli_refuses_a_declared_unsupported_case(capsys):
    sys.modules["tjclitest.cands"].NO_CASE_2 = CandidateSpec(
        name="no-case-2", model_factory=OracleEncoder, owner="tests", description="d",
        unsupported_official_cases=(2,))
    with pytest.raises(ValueError, match="does not support official case 2"):
        benchmark.main(["--candidate", "tjclitest.cands:NO_CASE_2", *BASE, "--case", "2", "--device", "cpu"])
    # --nvtx is accepted and is a no-op off the GPU
    rc = benchmark.main(["--candidate", "tjclitest.cands", *BASE, *SMALL, "--nvtx"])
    assert rc == 0
