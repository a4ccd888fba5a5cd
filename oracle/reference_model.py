"""FP32 restatement of the reference pre-LN encoder, its input generator and checker.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function cites the
lines of the reference's immutable ``torch_transformer_benchmark.py`` whose
behaviour it restates.  The module tree (names and construction order) matches
the reference so that (a) ``torch.manual_seed(s)`` followed by construction draws
identical default-initialised weights and (b) state dicts load strictly in both
directions.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class EncoderShape:
    """Field-for-field restatement of ``TransformerConfig``
    (torch_transformer_benchmark.py:29-56)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.d_model % self.num_heads:
            raise ValueError("d_model must be divisible by num_heads")


class OracleAttention(nn.Module):
    """Multi-head self-attention, torch_transformer_benchmark.py:59-122.

    Parameter names ``q_proj/k_proj/v_proj/out_proj`` and their creation order
    (:72-75) are kept so seeded default init reproduces the reference weights.
    """

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)

    def heads(self, t: torch.Tensor) -> torch.Tensor:
        b, n, _ = t.shape
        return t.view(b, n, self.num_heads, self.head_dim).transpose(1, 2)

    def forward(self, h: torch.Tensor, mask: Optional[torch.Tensor], causal: bool) -> torch.Tensor:
        b, n, _ = h.shape
        q = self.heads(self.q_proj(h))
        k = self.heads(self.k_proj(h))
        v = self.heads(self.v_proj(h))
        # scores = q k^T * head_dim^-0.5 (:97); causal -inf above the diagonal
        # (:99-103); -inf on invalid keys (:105-108); softmax in fp32 (:111).
        scores = (q @ k.transpose(-1, -2)) * (self.head_dim ** -0.5)
        if causal:
            upper = torch.ones(n, n, dtype=torch.bool, device=h.device).triu(1)
            scores = scores.masked_fill(upper, float("-inf"))
        if mask is not None:
            scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(h.dtype)
        ctx = (probs @ v).transpose(1, 2).reshape(b, n, self.d_model)
        out = self.out_proj(ctx)
        if mask is not None:  # zero invalid query rows (:120-121)
            out = out.masked_fill(~mask[..., None], 0)
        return out


class OracleBlock(nn.Module):
    """Pre-LN block, torch_transformer_benchmark.py:125-145."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = OracleAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor], causal: bool) -> torch.Tensor:
        x = x + self.attention(self.norm1(x), mask, causal)
        # exact (erf) GELU, :141
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
        if mask is not None:  # :143-144
            x = x.masked_fill(~mask[..., None], 0)
        return x


class OracleEncoder(nn.Module):
    """``BaselineTransformer``, torch_transformer_benchmark.py:148-172."""

    def __init__(self, config) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            OracleBlock(config.d_model, config.num_heads, config.ffn_dim)
            for _ in range(config.num_layers)
        )
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        x = self.final_norm(x)
        if valid_token_mask is not None:  # :169-171
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def seeded_encoder(config, seed: int = 1234, linear_scale: float = 1.0) -> OracleEncoder:
    """CPU default init under ``torch.manual_seed(seed)`` (the reference harness
    seeds then constructs on CPU: torch_transformer_benchmark.py:672-680).

    ``linear_scale`` multiplies every ``nn.Linear`` weight AND bias (LayerNorm
    untouched); the long-sequence configuration uses 0.5.
    """
    torch.manual_seed(seed)
    model = OracleEncoder(config)
    if linear_scale != 1.0:
        with torch.no_grad():
            for module in model.modules():
                if isinstance(module, nn.Linear):
                    module.weight.mul_(linear_scale)
                    module.bias.mul_(linear_scale)
    return model.eval()


def generate_random_case(
    config,
    device: torch.device,
    dtype: torch.dtype,
    seed: int,
    padding_ratio: float,
    input_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded input + right-padding mask, torch_transformer_benchmark.py:234-272.

    The draws are made in the reference's order on a generator of the target
    device (x first, then the lengths), so the same seed gives the same tensors
    as the reference on the same device.
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    b, n, d = config.batch_size, config.seq_len, config.d_model
    x = torch.randn(b, n, d, generator=gen, device=device, dtype=dtype) * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(b, n, device=device, dtype=torch.bool)
    low = max(1, int(round(n * (1.0 - padding_ratio))))
    lengths = torch.randint(low=low, high=n + 1, size=(b,), generator=gen, device=device)
    mask = torch.arange(n, device=device)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


@dataclass
class Verdict:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float


def check_outputs(reference: torch.Tensor, candidate: torch.Tensor,
                  rtol: float = 0.02, atol: float = 0.002, token_chunk: int = 4096) -> Verdict:
    """Element-wise ``finite & (|err| <= atol OR |err| <= rtol*|ref|)``; pass iff no
    element fails (torch_transformer_benchmark.py:289-356; the chunked evaluation
    follows src/implementations/fp32_reference.py:157-204 so large outputs do not
    need full-size temporaries)."""
    if reference.shape != candidate.shape:
        raise AssertionError(f"shape mismatch {tuple(reference.shape)} vs {tuple(candidate.shape)}")
    ref3 = reference.reshape(reference.shape[0], -1, reference.shape[-1]) if reference.ndim >= 2 else reference.reshape(1, -1, 1)
    can3 = candidate.reshape(ref3.shape)
    failed = 0
    abs_sum = 0.0
    max_abs = 0.0
    max_rel = 0.0
    for s in range(0, ref3.shape[1], token_chunk):
        r = ref3[:, s:s + token_chunk].float()
        c = can3[:, s:s + token_chunk].float()
        err = (c - r).abs()
        ok = torch.isfinite(r) & torch.isfinite(c) & ((err <= atol) | (err <= rtol * r.abs()))
        failed += int((~ok).sum().item())
        finite_err = torch.where(torch.isfinite(err), err, torch.full_like(err, math.inf))
        abs_sum += float(err.double().sum().item())
        max_abs = max(max_abs, float(finite_err.max().item()) if finite_err.numel() else 0.0)
        rel = err / r.abs().clamp_min(1e-12)
        max_rel = max(max_rel, float(rel.max().item()) if rel.numel() else 0.0)
    total = reference.numel()
    return Verdict(failed == 0, total, failed, max_abs, max_rel, abs_sum / max(total, 1))


def mask_lengths(mask: Optional[torch.Tensor], batch: int, seq_len: int) -> torch.Tensor:
    """Valid-prefix length per sample (1 + last valid position; 0 if none)."""
    if mask is None:
        return torch.full((batch,), seq_len, dtype=torch.int64)
    pos = torch.arange(1, seq_len + 1, device=mask.device)[None, :]
    return (mask.to(torch.int64) * pos).amax(dim=1).cpu()


def algorithmic_flops(config, lengths) -> Tuple[float, float]:
    """(GEMM flops, exact causal attention flops) over valid tokens only.

    GEMM = L * 2 * T_v * (4 d^2 + 2 d F); attention = L * 2 * d * sum_b l_b (l_b + 1)
    (QK^T and PV over the causal valid pairs; non-causal uses 4 d l_b^2).
    """
    L, d, F_ = config.num_layers, config.d_model, config.ffn_dim
    lengths = [int(v) for v in lengths]
    tv = sum(lengths)
    gemm = L * 2.0 * tv * (4 * d * d + 2 * d * F_)
    if config.causal:
        attn = L * 2.0 * d * sum(l * (l + 1) for l in lengths)
    else:
        attn = L * 4.0 * d * sum(l * l for l in lengths)
    return gemm, attn
