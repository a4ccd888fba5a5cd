"""Host-side checks that need no GPU: the C ABI library, the candidate contract
and the reference-compatible module tree."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from oracle.reference_model import EncoderShape, seeded_encoder
from techjam_b200 import _lib, build
from techjam_b200.candidate import CandidateSpec, TransformerConfig
from techjam_b200.dispatcher import CANDIDATE, DispatchingTransformer, UnsupportedCaseError

ROOT = Path(__file__).resolve().parent.parent


def _header_symbols():
    text = (ROOT / "include" / "tj.h").read_text()
    return sorted(set(re.findall(r"^TJ_API\s+[\w\s\*]+?\b(tj_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    build.build()
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    syms = _header_symbols()
    assert len(syms) >= 13
    for name in syms:
        assert hasattr(lib, name), f"{name} declared in include/tj.h but not exported"
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with tj.h"
    assert _lib.load().tj_version() >= 1


def test_library_rejects_bad_arguments_without_gpu():
    lib = _lib.load()
    out = ctypes.c_void_p()
    assert lib.tj_model_create(None, ctypes.byref(out)) == 1  # TJ_ERR_INVALID
    assert b"null" in lib.tj_last_error()
    cfg = _lib.TjConfig(1000, 16, 4096, 1, 1, 1e-5)  # head_dim not supported
    assert lib.tj_model_create(ctypes.byref(cfg), ctypes.byref(out)) in (1, 2)
    size = ctypes.c_size_t()
    assert lib.tj_workspace_bytes(None, 1, 1, 0, ctypes.byref(size)) == 1


def test_candidate_contract_validates():
    CANDIDATE.validate()
    assert CANDIDATE.name == "b200" and CANDIDATE.self_compiling
    with pytest.raises(ValueError):
        CandidateSpec("Bad Name", DispatchingTransformer, "o", "d").validate()
    with pytest.raises(ValueError):
        CandidateSpec("x", DispatchingTransformer, "o", "d", unsupported_official_cases=(15,)).validate()


@pytest.mark.parametrize("cfg", [EncoderShape(4, 512, 256, 8, 1024, 2, True),
                                 EncoderShape(2, 64, 128, 4, 256, 3, False)])
def test_parameter_tree_and_seeded_init_match_reference(cfg):
    oracle = seeded_encoder(cfg, 1234)
    torch.manual_seed(1234)
    cand = CANDIDATE.model_factory(TransformerConfig(*(getattr(cfg, f) for f in (
        "batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers", "causal"))))
    so, sc = oracle.state_dict(), cand.state_dict()
    assert list(so) == list(sc)
    for k in so:
        assert torch.equal(so[k], sc[k]), k
    cand.load_state_dict(so, strict=True)
    oracle.load_state_dict(cand.state_dict(), strict=True)


def test_cpu_input_raises():
    cfg = TransformerConfig(2, 64, 128, 4, 256, 1, True)
    model = CANDIDATE.model_factory(cfg).eval()
    with pytest.raises(UnsupportedCaseError):
        model(torch.zeros(2, 64, 128))
