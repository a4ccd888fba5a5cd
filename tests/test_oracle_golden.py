"""Pin the oracle restatement to fixtures produced by the reference's own code.

The fixtures in ``tests/golden`` were written by ``tests/golden/make_golden.py``
from the reference's ``BaselineTransformer``/``generate_random_case``
(torch_transformer_benchmark.py:148-172, 234-272) and
``poly_linear_attention``/``estimate_sigma``
(src/implementations/poly_reference.py:61-265, poly_guard.py:68-93).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import linear_memory, poly
from oracle.reference_model import (EncoderShape, check_outputs, generate_random_case,
                                    seeded_encoder)

GOLDEN = Path(__file__).resolve().parent / "golden"
MODEL_CASES = ["tiny_causal", "tiny_noncausal", "tiny_scaled", "c1", "c3_b4"]


def _load_model_case(name):
    z = np.load(GOLDEN / f"model_{name}.npz")
    b, n, d, h, f, layers, causal = (int(v) for v in z["config"])
    cfg = EncoderShape(b, n, d, h, f, layers, bool(causal))
    return z, cfg


@pytest.mark.parametrize("name", MODEL_CASES)
def test_oracle_matches_reference_outputs(name):
    z, cfg = _load_model_case(name)
    model = seeded_encoder(cfg, 1234, float(z["linear_scale"]))
    for seed in z["seeds"]:
        seed = int(seed)
        x, mask = generate_random_case(cfg, torch.device("cpu"), torch.float32, seed,
                                       float(z["padding_ratio"]))
        # the generator restatement is bit-identical to the reference's
        assert x.double().sum().item() == pytest.approx(z[f"xsum_{seed}"][0], abs=0, rel=0)
        assert np.array_equal(mask.sum(1).numpy(), z[f"lengths_{seed}"])
        with torch.inference_mode():
            y = model(x, mask).reshape(-1, cfg.d_model).numpy()
        rows = z[f"rows_{seed}"]
        np.testing.assert_allclose(y[rows], z[f"y_{seed}"], rtol=0, atol=2e-6)


def test_oracle_general_mask_matches_reference():
    z, cfg = _load_model_case("tiny_causal")
    model = seeded_encoder(cfg, 1234)
    x, _ = generate_random_case(cfg, torch.device("cpu"), torch.float32, 99, 0.0)
    mask = torch.from_numpy(z["general_mask"])
    x = x.masked_fill(~mask[..., None], 0)
    with torch.inference_mode():
        y = model(x, mask).reshape(-1, cfg.d_model).numpy()
    np.testing.assert_allclose(y, z["general_y"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("name", ["tiny_causal", "tiny_noncausal", "c1"])
def test_linear_memory_oracle_matches_dense(name):
    """The bounded-memory oracle equals the dense model (pins it the way
    src/tests/test_fp32_reference.py:24-69 pins the reference's SDPA oracle)."""
    z, cfg = _load_model_case(name)
    model = seeded_encoder(cfg, 1234)
    x, mask = generate_random_case(cfg, torch.device("cpu"), torch.float32, 1234,
                                   float(z["padding_ratio"]))
    with torch.inference_mode():
        dense = model(x, mask)
        lin = linear_memory.linear_memory_forward(model, x, mask, q_chunk=100)
    assert (dense - lin).abs().max().item() < 1e-4


@pytest.mark.parametrize("name", ["d32", "d64", "d64_taylor"])
def test_poly_oracle_matches_reference(name):
    z = np.load(GOLDEN / f"poly_{name}.npz")
    b, h, n, dh, chunk, prefix = (int(v) for v in z["spec"])
    sigma = None if float(z["sigma"]) < 0 else float(z["sigma"])
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(b, h, n, dh, generator=gen) * 0.577
    k = torch.randn(b, h, n, dh, generator=gen) * 0.577
    v = torch.randn(b, h, n, dh, generator=gen) * 0.577
    y = poly.poly_attention(q, k, v, dh ** -0.5, chunk=chunk, exact_prefix=prefix, sigma=sigma)
    np.testing.assert_allclose(y.numpy(), z["y"], rtol=0, atol=2e-5)
    assert poly.estimate_sigma(q, k, dh ** -0.5) == pytest.approx(float(z["sigma_est"]), rel=1e-6)
    assert poly.hermite_coefficients(sigma) == pytest.approx(tuple(z["coeffs"]), rel=1e-12)


def test_hermite_constants():
    # poly_reference.py:35-58 and src/tests/test_poly_reference.py:71-95
    assert poly.hermite_coefficients(None) == (1.0, 1.0, 0.5)
    for s in (0.1, 0.334, 0.4):
        c0, _, c2 = poly.hermite_coefficients(s)
        assert c0 + c2 * s * s == pytest.approx(np.exp(s * s / 2), rel=1e-12)


def test_poly_guard_admission():
    assert poly.poly_is_safe(0.334) and poly.poly_is_safe(0.40)
    assert not poly.poly_is_safe(0.41) and not poly.poly_is_safe(0.0)
    assert not poly.poly_is_safe(float("nan")) and not poly.poly_is_safe(None)


def test_checker_or_criterion():
    ref = torch.tensor([[[1.0, 0.0, 100.0, float("nan")]]])
    got = torch.tensor([[[1.019, 0.0019, 101.9, 0.0]]])
    v = check_outputs(ref, got)
    assert v.failed_elements == 1  # only the non-finite element fails
    got2 = torch.tensor([[[1.03, 0.0, 100.0, 0.0]]])
    assert check_outputs(ref[..., :3], got2[..., :3]).failed_elements == 1
