"""The drop-in boundary exercised with the reference's own classes (CPU; runs
when ``TJ_REFERENCE_ROOT`` names a checkout of the reference repository,
skipped otherwise, e.g. on the GPU box).

The two-line shim -- re-wrapping ``CANDIDATE`` in the
reference's ``CandidateSpec`` -- must pass the reference's ``load_candidate``
and ``validate_candidate_execution``; the factory must accept the reference's
``TransformerConfig``; and the reference's strict ``copy_model_weights`` must
load its seeded ``BaselineTransformer`` into the B200 module and back.
Nothing here runs a forward (the B200 module has no CPU path).
"""

import os
import sys
import types
from dataclasses import asdict
from pathlib import Path

import pytest
import torch

REF = Path(os.environ["TJ_REFERENCE_ROOT"]) if os.environ.get("TJ_REFERENCE_ROOT") else None
pytestmark = pytest.mark.skipif(REF is None or not (REF / "torch_transformer_benchmark.py").exists(),
                                reason="TJ_REFERENCE_ROOT does not name a reference checkout")


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, str(REF))
    try:
        import torch_transformer_benchmark as ttb
        from src import infra
        yield ttb, infra
    finally:
        sys.path.remove(str(REF))


def test_shim_passes_the_reference_loader(ref):
    ttb, infra = ref
    from techjam_b200.dispatcher import CANDIDATE

    shim = types.ModuleType("tjshim.b200")
    shim.CANDIDATE = infra.CandidateSpec(**asdict(CANDIDATE))  # the reference's own class
    pkg = types.ModuleType("tjshim")
    pkg.__path__ = []
    sys.modules["tjshim"], sys.modules["tjshim.b200"] = pkg, shim
    try:
        spec = infra.load_candidate("tjshim.b200")
    finally:
        sys.modules.pop("tjshim.b200", None)
        sys.modules.pop("tjshim", None)
    assert spec.name == "b200" and spec.self_compiling
    for case in range(1, 15):
        infra.validate_candidate_execution(spec, case, compile_user=False, dtype_name="float32",
                                           candidate_only=False, input_scale=1.0, device_type="cuda",
                                           cuda_capability=(10, 0), torch_version=torch.__version__)
    with pytest.raises(ValueError, match="compiles itself"):
        infra.validate_candidate_execution(spec, None, compile_user=True)


@pytest.mark.parametrize("causal", [True, False])
def test_reference_weight_copy_round_trips(ref, causal):
    ttb, _ = ref
    from techjam_b200.dispatcher import CANDIDATE

    cfg = ttb.TransformerConfig(batch_size=2, seq_len=32, d_model=64, num_heads=4, ffn_dim=128, num_layers=2,
                                causal=causal)
    torch.manual_seed(1234)
    baseline = ttb.BaselineTransformer(cfg)
    candidate = CANDIDATE.model_factory(cfg)  # the reference's TransformerConfig, unchanged
    ttb.copy_model_weights(baseline, candidate, strict=True)
    for (kb, vb), (kc, vc) in zip(baseline.state_dict().items(), candidate.state_dict().items()):
        assert kb == kc and torch.equal(vb, vc)
    torch.manual_seed(1234)
    fresh = CANDIDATE.model_factory(cfg)  # seeded construction draws the reference's weights
    for k, v in baseline.state_dict().items():
        assert torch.equal(v, fresh.state_dict()[k]), k
    ttb.copy_model_weights(candidate, ttb.BaselineTransformer(cfg), strict=True)
