"""GPU test of ``tj_forward_noalloc``, the allocation-free forward entry point.

Some callers cannot allocate device memory on their call path -- a serving
runtime or host application that owns a fixed device budget and forbids
``cudaMalloc`` after start-up, or a latency-critical path that cannot afford
cudaMalloc's implicit device synchronisation.  ``tj_forward_noalloc`` serves
them: its scratch is a fixed array inside libtj (``TJ_NOALLOC_SCRATCH_BYTES``
per device), and it must give the same result as ``tj_forward``, which uses a
caller-provided workspace.

This file is named so pytest collects it last.  It builds its own model and
inputs, so it passes both alone in a fresh process and after the other tests.
"""

import ctypes

import pytest
import torch

from oracle.reference_model import EncoderShape, check_outputs, generate_random_case, seeded_encoder
from techjam_b200 import _lib
from techjam_b200.dispatcher import CANDIDATE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _noalloc(model, x, mask):
    """Call tj_forward_noalloc through the C ABI; returns (status, out)."""
    handle = model._ensure_packed(x.device)  # the model's packed weights (made by tj_model_create earlier)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream(x.device)
    status = _lib.load().tj_forward_noalloc(handle.ptr, x.data_ptr(), None if mask is None else mask.data_ptr(),
                                            out.data_ptr(), x.shape[0], x.shape[1], _lib.ROUTE_EXACT,
                                            ctypes.c_void_p(stream.cuda_stream))
    return status, out


def test_noalloc_forward_matches_workspace_forward_twice():
    cfg = EncoderShape(4, 512, 256, 8, 1024, 2, True)  # C1 shape: ~9 MiB of scratch
    oracle = seeded_encoder(cfg, 1234)
    model = CANDIDATE.model_factory(cfg)
    model.load_state_dict(oracle.state_dict(), strict=True)
    model = model.to(DEV).eval()
    model.attention_route = "exact"
    with torch.inference_mode():
        # two calls in a row, with different inputs and shapes, each against tj_forward
        x1, m1 = generate_random_case(cfg, DEV, torch.float32, 1234, 0.5)
        cfg2 = EncoderShape(3, 384, 256, 8, 1024, 2, True)
        x2, m2 = generate_random_case(cfg2, DEV, torch.float32, 1235, 0.3)
        for x, m in ((x1, m1), (x2, m2)):
            expected = model(x, m)  # tj_forward with a caller workspace
            status, got = _noalloc(model, x, m)
            torch.cuda.synchronize()
            assert status == _lib.TJ_OK, _lib.load().tj_last_error()
            assert model.device_error() == 0
            verdict = check_outputs(expected, got)  # the reference's OR criterion
            assert verdict.passed, verdict
            assert (got - expected).abs().max().item() <= 1e-6
            assert torch.all(got[~m] == 0)


def test_noalloc_forward_rejects_oversize_shape():
    cfg = EncoderShape(16, 2048, 256, 8, 1024, 1, True)  # needs far more than 32 MiB of scratch
    model = CANDIDATE.model_factory(cfg).to(DEV).eval()
    x = torch.zeros(16, 2048, 256, device=DEV)
    status, _ = _noalloc(model, x, None)
    assert status == 2  # TJ_ERR_UNSUPPORTED
    assert b"scratch" in _lib.load().tj_last_error()


def test_noalloc_forward_captures_without_allocating():
    """The entry point's promise, checked directly: once the first call has
    resolved the scratch array's address, a call captured into a CUDA graph
    with capture_error_mode="global" (where any cudaMalloc, from any thread,
    invalidates the capture) succeeds, and replaying it gives the eager
    result bit for bit."""
    cfg = EncoderShape(2, 384, 256, 8, 1024, 2, True)
    model = CANDIDATE.model_factory(cfg)
    model.load_state_dict(seeded_encoder(cfg, 77).state_dict(), strict=True)
    model = model.to(DEV).eval()
    model.attention_route = "exact"
    x, m = generate_random_case(cfg, DEV, torch.float32, 77, 0.4)
    with torch.inference_mode():
        status, eager = _noalloc(model, x, m)
        torch.cuda.synchronize()
        assert status == _lib.TJ_OK, _lib.load().tj_last_error()
        handle = model._ensure_packed(x.device)
        out = torch.zeros_like(x)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="global"):
            stream = torch.cuda.current_stream(x.device)
            status = _lib.load().tj_forward_noalloc(handle.ptr, x.data_ptr(), m.data_ptr(), out.data_ptr(),
                                                    x.shape[0], x.shape[1], _lib.ROUTE_EXACT,
                                                    ctypes.c_void_p(stream.cuda_stream))
        assert status == _lib.TJ_OK, _lib.load().tj_last_error()
        graph.replay()
        torch.cuda.synchronize()
    assert model.device_error() == 0
    assert torch.equal(out, eager)
    del graph
