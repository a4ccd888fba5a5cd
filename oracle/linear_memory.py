"""Bounded-memory FP32 oracle for configurations whose dense scores cannot exist.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates the idea of the
reference's ``LinearMemoryFP32Reference``
(src/implementations/fp32_reference.py:70-142): the immutable model with only
the ``[N, N]`` score/probability tensors replaced by an algebraically
equivalent evaluation.  Instead of a fused SDPA backend (whose FP32 kernels are
library code), attention here is an explicit two-pass FP32 softmax over query
chunks, so peak memory is ``O(chunk * N)`` per head and the arithmetic stays
inspectable.  It runs on whatever device its inputs live on.

It is itself pinned against the dense ``OracleEncoder`` at reduced sizes by
``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from .reference_model import OracleEncoder


def chunked_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                      causal: bool, key_mask: Optional[torch.Tensor] = None,
                      q_chunk: int = 1024) -> torch.Tensor:
    """Exact softmax attention, ``[B,H,N,D]`` in/out, FP32, query-chunked.

    For causal attention a query chunk only multiplies the keys at or before its
    last row, so work is also causal-trimmed.  Rows with every key masked give 0.
    """
    b, h, n, dh = q.shape
    out = torch.empty_like(q)
    for s in range(0, n, q_chunk):
        e = min(s + q_chunk, n)
        kend = e if causal else n
        sc = (q[:, :, s:e].float() @ k[:, :, :kend].float().transpose(-1, -2)) * scale
        if causal:
            qi = torch.arange(s, e, device=q.device)[:, None]
            kj = torch.arange(kend, device=q.device)[None, :]
            sc = sc.masked_fill(kj > qi, float("-inf"))
        if key_mask is not None:
            sc = sc.masked_fill(~key_mask[:, None, None, :kend], float("-inf"))
        mx = sc.amax(dim=-1, keepdim=True)
        mx = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
        p = torch.exp(sc - mx)
        den = p.sum(dim=-1, keepdim=True)
        o = (p @ v[:, :, :kend].float()) / den.clamp_min(1e-30)
        out[:, :, s:e] = torch.where(den > 0, o, torch.zeros_like(o)).to(q.dtype)
        del sc, p
    return out


@torch.no_grad()
def linear_memory_forward(model: OracleEncoder, x: torch.Tensor,
                          mask: Optional[torch.Tensor] = None, q_chunk: int = 1024,
                          attention_fn=None) -> torch.Tensor:
    """``OracleEncoder.forward`` with attention evaluated by ``chunked_attention``
    (or by ``attention_fn(q, k, v, scale, causal, key_mask)`` when given).

    Everything around attention -- LayerNorms, projections, GELU FFN, residuals
    and the padded-row zeroing -- is the reference arithmetic
    (torch_transformer_benchmark.py:93-95,118-121,134-145,162-172).
    """
    cfg = model.config
    attend = attention_fn or (lambda q, k, v, sc, c, km: chunked_attention(q, k, v, sc, c, km, q_chunk))
    for layer in model.layers:
        att = layer.attention
        hin = layer.norm1(x)
        q, k, v = att.heads(att.q_proj(hin)), att.heads(att.k_proj(hin)), att.heads(att.v_proj(hin))
        ctx = attend(q, k, v, att.head_dim ** -0.5, cfg.causal, mask)
        b, n, _ = x.shape
        o = att.out_proj(ctx.transpose(1, 2).reshape(b, n, cfg.d_model))
        if mask is not None:
            o = o.masked_fill(~mask[..., None], 0)
        x = x + o
        x = x + layer.ffn_out(F.gelu(layer.ffn_in(layer.norm2(x)), approximate="none"))
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
    x = model.final_norm(x)
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x
