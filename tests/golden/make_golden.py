"""Generate the golden fixtures that pin ``oracle/`` to the reference itself.

Run with ``TJ_REFERENCE_ROOT`` naming a checkout of the reference repository::

    TJ_REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py

It imports the reference's own modules -- ``torch_transformer_benchmark``
(``BaselineTransformer``, ``generate_random_case``) and
``src.implementations.poly_reference`` / ``poly_guard`` -- runs them on the CPU
and writes small ``.npz`` files next to this script.  The reference is never
needed at test time: ``tests/test_oracle_golden.py`` only reads these files.

Fixtures
--------
``model_<name>.npz``  seeded model output for a configuration (full output for
                      tiny shapes, a fixed random subset of rows for larger
                      ones), the generated input's checksum and lengths.
``poly_<name>.npz``   ``poly_linear_attention`` output (compute/state float32)
                      for seeded q/k/v, plus the guard's sigma estimate.
``checker.npz`` +     the reference's ``compare_outputs`` verdicts (every field of
``checker.json``      its ``AccuracyResult``) on deterministic edge cases, its
                      ``percentile``, and the paired-timing statistics of
                      ``src/infra/timing.py`` on fixed samples -- they pin the
                      product-side checker and timing restatements.
"""

from __future__ import annotations

import importlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get("TJ_REFERENCE_ROOT"):
    raise SystemExit("set TJ_REFERENCE_ROOT to a checkout of the reference repository")
REF = Path(os.environ["TJ_REFERENCE_ROOT"])

# name: (B, N, d, H, F, L, causal, padding_ratio, linear_scale, rows_kept or None=all)
MODEL_CASES = {
    "tiny_causal": (2, 48, 64, 4, 96, 2, True, 0.5, 1.0, None),
    "tiny_noncausal": (3, 40, 32, 2, 64, 1, False, 0.3, 1.0, None),
    "tiny_scaled": (2, 64, 64, 2, 128, 1, True, 0.0, 0.5, None),
    "c1": (4, 512, 256, 8, 1024, 2, True, 0.5, 1.0, 96),
    "c3_b4": (4, 256, 512, 8, 2048, 4, True, 0.75, 1.0, 64),
}
MODEL_SEEDS = (1234, 1235)


def _import_reference():
    sys.path.insert(0, str(REF))
    ttb = importlib.import_module("torch_transformer_benchmark")
    poly_ref = importlib.import_module("src.implementations.poly_reference")
    guard = importlib.import_module("src.implementations.poly_guard")
    return ttb, poly_ref, guard


def _model_fixture(ttb, name, spec):
    b, n, d, h, f, layers, causal, pr, lscale, keep = spec
    cfg = ttb.TransformerConfig(b, n, d, h, f, layers, causal)
    torch.manual_seed(1234)
    model = ttb.BaselineTransformer(cfg).eval()
    if lscale != 1.0:
        with torch.no_grad():
            for mod in model.modules():
                if isinstance(mod, torch.nn.Linear):
                    mod.weight.mul_(lscale)
                    mod.bias.mul_(lscale)
    out = {"config": np.array([b, n, d, h, f, layers, int(causal)], dtype=np.int64),
           "padding_ratio": np.float64(pr), "linear_scale": np.float64(lscale),
           "seeds": np.array(MODEL_SEEDS, dtype=np.int64)}
    rng = np.random.default_rng(7)
    for seed in MODEL_SEEDS:
        x, mask = ttb.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed, pr, 1.0)
        with torch.inference_mode():
            y = model(x, mask)
        rows = np.arange(b * n) if keep is None else np.sort(rng.choice(b * n, size=keep, replace=False))
        out[f"rows_{seed}"] = rows.astype(np.int64)
        out[f"y_{seed}"] = y.reshape(b * n, d).numpy()[rows]
        out[f"lengths_{seed}"] = mask.sum(1).numpy().astype(np.int64)
        out[f"xsum_{seed}"] = np.array([x.double().sum().item(), x.double().abs().sum().item()])
        out[f"x0_{seed}"] = x.reshape(b * n, d).numpy()[rows[:4]]
    # A mask with interior holes (not right padding) exercises the general key mask.
    if name == "tiny_causal":
        x, _ = ttb.generate_random_case(cfg, torch.device("cpu"), torch.float32, 99, 0.0, 1.0)
        g = torch.Generator().manual_seed(5)
        mask = torch.rand(b, n, generator=g) > 0.3
        mask[:, 0] = True
        x = x.masked_fill(~mask[..., None], 0)
        with torch.inference_mode():
            y = model(x, mask)
        out["general_mask"] = mask.numpy()
        out["general_y"] = y.reshape(b * n, d).numpy()
    np.savez_compressed(HERE / f"model_{name}.npz", **out)


# name: (B, H, N, D, chunk, exact_prefix, sigma)
POLY_CASES = {
    "d32": (1, 2, 512, 32, 128, 128, 0.334),
    "d64": (1, 2, 384, 64, 128, 128, 0.334),
    "d64_taylor": (1, 1, 320, 64, 64, 0, None),
}


def _poly_fixture(poly_ref, guard, name, spec):
    b, h, n, dh, chunk, prefix, sigma = spec
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(b, h, n, dh, generator=gen) * 0.577
    k = torch.randn(b, h, n, dh, generator=gen) * 0.577
    v = torch.randn(b, h, n, dh, generator=gen) * 0.577
    scale = dh ** -0.5
    y = poly_ref.poly_linear_attention(q, k, v, scale, chunk=chunk, exact_prefix=prefix,
                                       sigma=sigma, state_dtype=torch.float32,
                                       compute_dtype=torch.float32)
    est = guard.estimate_sigma(q, k, scale)
    c = poly_ref.hermite_coefficients(sigma)
    np.savez_compressed(HERE / f"poly_{name}.npz", spec=np.array([b, h, n, dh, chunk, prefix]),
                        sigma=np.float64(-1.0 if sigma is None else sigma), y=y.numpy(),
                        sigma_est=np.float64(est), coeffs=np.array(c, dtype=np.float64))


def _checker_cases():
    """Deterministic (reference, candidate) pairs covering the criterion's edges."""
    g = torch.Generator().manual_seed(7)
    cases = {}
    ref = torch.randn(2, 5, 7, generator=g)
    cases["all_pass"] = (ref, ref + 1e-4 * torch.randn(2, 5, 7, generator=g))
    got = ref + 1e-4 * torch.randn(2, 5, 7, generator=g)
    got[1, 3, 4] += 0.25
    got[0, 0, 2] += 0.01
    cases["two_failures"] = (ref, got)
    r = torch.tensor([[[1.0, 1.0, 0.01, 100.0, -0.5, 0.0]]])
    c = torch.tensor([[[1.002, 1.0, 0.0121, 102.0, -0.5103, 0.0019]]])
    cases["thresholds"] = (r, c)
    got = ref.clone()
    got[1, 2, 3] = float("nan")
    cases["nan_candidate"] = (ref, got)
    r2 = ref.clone()
    r2[0, 4, 6] = float("inf")
    cases["inf_reference"] = (r2, ref.clone())
    return cases


def _checker_fixture(ttb):
    sys.path.insert(0, str(REF))
    timing = importlib.import_module("src.infra.timing")
    arrays, verdicts = {}, {}
    for name, (r, c) in _checker_cases().items():
        res = ttb.compare_outputs(r, c, rtol=0.02, atol=0.002)
        arrays[f"{name}_ref"] = r.numpy()
        arrays[f"{name}_cand"] = c.numpy()
        verdicts[name] = {k: (list(v) if isinstance(v, tuple) else v) for k, v in vars(res).items()}
    samples = {"baseline": [10.0, 12.0, 11.0, 13.0, 10.5, 12.5], "candidate": [5.0, 5.5, 5.2, 6.0, 5.1, 5.9]}
    stats = {
        "percentile": {str(q): ttb.percentile([3.0, 1.0, 4.0, 1.5, 9.0, 2.6], q) for q in (0.0, 0.5, 0.9, 1.0)},
        "paired_schedule_5": timing.paired_schedule(5),
        "samples": samples,
        "paired_summary": timing.paired_summary(samples),
        "paired_ratios": timing.paired_ratios(samples),
        "noise_floor_ratio": timing.noise_floor_ratio(samples),
        "choose_block_size": {str(ms): timing.choose_block_size(ms) for ms in (0.01, 0.3, 1.7, 5.0, 49.0, 80.0)},
    }
    np.savez_compressed(HERE / "checker.npz", **arrays)
    (HERE / "checker.json").write_text(json.dumps({"verdicts": verdicts, "timing": stats}, indent=1,
                                                  default=float) + "\n")


def main():
    ttb, poly_ref, guard = _import_reference()
    _checker_fixture(ttb)
    print("checker")
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name, spec in MODEL_CASES.items():
        _model_fixture(ttb, name, spec)
        print("model", name)
    for name, spec in POLY_CASES.items():
        _poly_fixture(poly_ref, guard, name, spec)
        print("poly", name)
    meta = {"reference_root": "$TJ_REFERENCE_ROOT (a checkout of IceyFoxes/techjam)", "torch": torch.__version__,
            "model_cases": {k: list(v) for k, v in MODEL_CASES.items()},
            "poly_cases": {k: list(v) for k, v in POLY_CASES.items()},
            "checker_cases": sorted(_checker_cases())}
    (HERE / "MANIFEST.json").write_text(json.dumps(meta, indent=1) + "\n")


if __name__ == "__main__":
    main()
