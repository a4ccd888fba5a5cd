"""GPU parity of the guarded polynomial route against the poly oracle.

The oracle (``oracle.poly.poly_attention``, float64) restates the reference's
``poly_linear_attention`` (src/implementations/poly_reference.py:61-265) and is
pinned by ``tests/golden/poly_*.npz``; inputs follow the reference's own poly
tests (q, k, v with component rms 0.577 at head_dim 64, scale 1/8,
src/tests/test_poly_reference.py:26-33), which puts the score spread near the
measured sigma of 0.334.
"""

import pytest
import torch

from oracle import poly
from techjam_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCALE = 64 ** -0.5


def _qkv(b, h, n, seed, rms=0.577):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = (torch.randn(b, h, n, 64, generator=g, device=DEV) * rms).half()
    k = (torch.randn(b, h, n, 64, generator=g, device=DEV) * rms).half()
    v = (torch.randn(b, h, n, 64, generator=g, device=DEV) * 0.577).half()
    return q, k, v


def _strided_sigma(q, k):
    n = q.shape[2]
    rows = (torch.arange(512, device=q.device) * n) // 512
    s = (q[:, :, rows].float() @ k[:, :, rows].float().transpose(-1, -2)) * SCALE
    return s.std().item(), s.abs().max().item()


@pytest.mark.parametrize("b,h,n,prefix", [(1, 2, 8192, 1024), (2, 3, 6144, 4096)])
def test_poly_route_matches_oracle(b, h, n, prefix):
    q, k, v = _qkv(b, h, n, seed=n + b)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ctx, st = ops.poly_attention(q, k, v, exact_prefix=prefix, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    sig, mx = _strided_sigma(q, k)
    assert st.admit, st
    assert abs(st.sigma - sig) < 2e-4 and abs(st.max_abs - mx) < 1e-3
    c0, c1, c2 = poly.hermite_coefficients(st.sigma)
    assert (st.c0, st.c1, st.c2) == pytest.approx((c0, c1, c2), rel=1e-5)
    ref = poly.poly_attention(q, k, v, SCALE, chunk=512, exact_prefix=prefix, sigma=st.sigma, dtype=torch.float64)
    got = ctx.view(b, n, h, 64).transpose(1, 2).float()
    torch.testing.assert_close(got, ref.float(), atol=3e-3, rtol=1e-2)


def test_poly_guard_rejects_wide_scores_and_falls_back_to_exact():
    q, k, v = _qkv(1, 2, 8192, seed=5, rms=1.5)  # sigma ~ 2.25 > 0.40
    ctx, st = ops.poly_attention(q, k, v, exact_prefix=1024)
    assert not st.admit and st.sigma > 0.4
    info = ops.prepare_mask(None, 1, 8192, DEV)
    exact = ops.attention(q, k, v, info, causal=True)
    assert torch.equal(ctx, exact)
