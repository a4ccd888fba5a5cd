"""Failure detection on the GPU without a fault.

Every spin-wait in libtj's kernels is bounded.  Here a wait that nothing
completes (``tj_wait_selftest``: one warp on a barrier no one arrives at, the
same bounded-wait code every kernel uses) runs out after a 1 ms limit set at
run time; the kernel records its site code and returns, the host reports
``TJ_ERR_DEVICE``, and the context stays usable -- a normal forward right
after it still passes the reference criterion.  Nothing faults, traps or
hangs.  The reference's counterpart is its dispatcher's error contract
(``src/dispatcher.py:684-706``: unsupported or failed routes raise before
returning wrong results).
"""

import time

import pytest
import torch

from oracle.reference_model import EncoderShape, check_outputs, generate_random_case, seeded_encoder
from techjam_b200 import _lib
from techjam_b200.dispatcher import CANDIDATE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
SELFTEST_SITE = 900


def _stream():
    return torch.cuda.current_stream(DEV).cuda_stream


def _timed_selftest(model_ptr, err_ptr, limit_ns):
    _lib.call("tj_set_wait_limit", limit_ns)
    try:
        torch.cuda.synchronize(DEV)
        t0 = time.perf_counter()
        _lib.call("tj_wait_selftest", model_ptr, err_ptr, _stream())
        torch.cuda.synchronize(DEV)
        return time.perf_counter() - t0
    finally:
        _lib.call("tj_set_wait_limit", 0)  # back to the 4 s default


def test_expired_wait_reports_site_and_context_survives():
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = EncoderShape(2, 384, 256, 8, 1024, 2, True)
    oracle = seeded_encoder(cfg, 1234)
    model = CANDIDATE.model_factory(cfg)
    model.load_state_dict(oracle.state_dict(), strict=True)
    oracle, model = oracle.to(DEV).eval(), model.to(DEV).eval()
    x, mask = generate_random_case(cfg, DEV, torch.float32, 1234, 0.5)
    with torch.inference_mode():
        model(x, mask)  # packs the weights and creates the library model
    torch.cuda.synchronize(DEV)
    model.check_device()

    elapsed = _timed_selftest(model._handle.ptr, None, 1_000_000)  # 1 ms
    assert elapsed < 2.0, f"the wait ran {elapsed:.2f} s: the 1 ms limit was not applied"
    with pytest.raises(_lib.TjError) as info:
        model.check_device()
    assert info.value.status == _lib.TJ_ERR_DEVICE
    assert f"site {SELFTEST_SITE}" in str(info.value)
    assert model.device_error() == 0  # the check cleared the word

    # the context is intact: the next forward is complete and correct
    with torch.inference_mode():
        got = model(x, mask)
        ref = oracle(x, mask)
    torch.cuda.synchronize(DEV)
    model.check_device()
    verdict = check_outputs(ref, got)
    assert verdict.passed, verdict
    assert torch.all(got[~mask] == 0)


def test_expired_wait_into_caller_error_word():
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _timed_selftest(None, err.data_ptr(), 200_000)  # 0.2 ms
    assert int(err.item()) == SELFTEST_SITE
    # a word that already holds an error is left as it is (first writer wins)
    err.fill_(123)
    _timed_selftest(None, err.data_ptr(), 200_000)
    assert int(err.item()) == 123
