"""Chunked degree-2 polynomial (Hermite/Taylor-exp) causal linear attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates the algorithm
of the reference's ``src/implementations/poly_reference.py:30-265`` and the
score-spread guard of ``src/implementations/poly_guard.py:65-102``:

* ``a = q*sqrt(scale)``, ``b = k*sqrt(scale)`` so ``a.b`` is the scaled score;
* keys in EARLIER chunks are weighted by ``w(s) = c0 + c1 s + c2 s^2`` with the
  Gauss-Hermite coefficients of ``hermite_coefficients`` (poly_reference.py:35-58);
  their contribution is carried by running sums over all previous keys:
  ``S0 = sum v``, ``S1 = sum b v^T``, ``S2 = sum (b b^T) v^T`` (the d^2 x d
  quadratic state), ``Z1 = sum b``, ``G = sum b b^T`` and the key count
  (poly_reference.py:111-116, 184-204, 232-250);
* keys in the SAME chunk are weighted by the exact ``exp(s)`` with the causal
  triangle, without max subtraction (poly_reference.py:215-224);
* the first ``exact_prefix`` queries are recomputed by exact causal softmax
  (poly_reference.py:255-264).

Arithmetic runs in ``dtype`` throughout (float64 by default), so this is the
"infinitely precise" version of the route; the CUDA kernel's FP16-operand /
FP32-state rounding is judged against it.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

SIGMA_CEILING = 0.40  # poly_guard.py:65
CHUNK = 512           # poly_attention.py:17
EXACT_PREFIX = 4096   # poly_attention.py:18


def hermite_coefficients(sigma: Optional[float]) -> Tuple[float, float, float]:
    """(c0, c1, c2) of the L2-optimal quadratic fit to exp(s) for s ~ N(0, sigma^2):
    ``exp(sigma^2/2) * [(1 - sigma^2/2) + s + s^2/2]``; ``None`` is plain Taylor
    (poly_reference.py:35-58, including its 1e-3 floor on the constant term)."""
    if sigma is None:
        return 1.0, 1.0, 0.5
    g = math.exp(0.5 * sigma * sigma)
    return g * max(1.0 - 0.5 * sigma * sigma, 1e-3), g, 0.5 * g


def poly_is_safe(sigma: Optional[float]) -> bool:
    """Admission rule, poly_guard.py:96-102: finite and 0 < sigma <= 0.40."""
    if sigma is None or math.isnan(sigma) or math.isinf(sigma):
        return False
    return 0.0 < sigma <= SIGMA_CEILING


def estimate_sigma(q: torch.Tensor, k: torch.Tensor, scale: float, samples: int = 512,
                   seed: int = 0) -> float:
    """Std of scaled scores over all pairs of ``samples`` random rows per head
    (poly_guard.py:68-93): same generator, permutation and unbiased std."""
    n = q.shape[2]
    count = min(samples, n)
    gen = torch.Generator(device=q.device).manual_seed(seed)
    idx = torch.randperm(n, generator=gen, device=q.device)[:count]
    qs = q[:, :, idx].float()
    ks = k[:, :, idx].float()
    return float(((qs @ ks.transpose(-1, -2)) * scale).std().item())


def _exact_causal(q, k, v, scale, dtype):
    n = q.shape[2]
    s = (q.to(dtype) @ k.to(dtype).transpose(-1, -2)) * scale
    s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return torch.softmax(s, dim=-1) @ v.to(dtype)


@torch.no_grad()
def poly_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, *,
                   chunk: int = CHUNK, exact_prefix: int = EXACT_PREFIX,
                   sigma: Optional[float] = None, dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """Causal polynomial attention over ``[B, H, N, D]``; returns ``q.dtype``."""
    bsz, nh, n, dh = q.shape
    c0, c1, c2 = hermite_coefficients(sigma)
    r = math.sqrt(scale)
    dev = q.device
    out = torch.empty(bsz, nh, n, dh, dtype=dtype, device=dev)
    s0 = torch.zeros(bsz, nh, dh, dtype=dtype, device=dev)
    s1 = torch.zeros(bsz, nh, dh, dh, dtype=dtype, device=dev)
    s2 = torch.zeros(bsz, nh, dh, dh, dh, dtype=dtype, device=dev)
    z1 = torch.zeros(bsz, nh, dh, dtype=dtype, device=dev)
    g = torch.zeros(bsz, nh, dh, dh, dtype=dtype, device=dev)
    seen = 0
    for t0 in range(0, n, chunk):
        t1 = min(t0 + chunk, n)
        a = q[:, :, t0:t1].to(dtype) * r
        b = k[:, :, t0:t1].to(dtype) * r
        vv = v[:, :, t0:t1].to(dtype)
        c = t1 - t0
        w = torch.exp(a @ b.transpose(-1, -2))
        w = w.masked_fill(torch.ones(c, c, dtype=torch.bool, device=dev).triu(1), 0.0)
        num = w @ vv
        den = w.sum(-1)
        if seen:
            num = num + c0 * s0[:, :, None, :] + c1 * (a @ s1) \
                + c2 * torch.einsum("bhci,bhcj,bhijd->bhcd", a, a, s2)
            den = den + c0 * seen + c1 * (a @ z1[..., None])[..., 0] \
                + c2 * torch.einsum("bhci,bhij,bhcj->bhc", a, g, a)
        out[:, :, t0:t1] = num / den[..., None]
        s0 += vv.sum(2)
        s1 += b.transpose(-1, -2) @ vv
        s2 += torch.einsum("bhci,bhcj,bhcd->bhijd", b, b, vv)
        z1 += b.sum(2)
        g += b.transpose(-1, -2) @ b
        seen += c
    if exact_prefix > 0:
        w0 = min(exact_prefix, n)
        out[:, :, :w0] = _exact_causal(q[:, :, :w0], k[:, :, :w0], v[:, :, :w0], scale, dtype)
    return out.to(q.dtype)
