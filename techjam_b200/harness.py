"""Benchmark-harness pieces of the reference, restated for the B200 build.

* ``CONFIGS``: the five workload presets (BASELINE configs C1-C5) as
  ``TransformerConfig`` + padding ratio + linear-weight scale.
* ``generate_random_case``: the reference's seeded input generator
  (torch_transformer_benchmark.py:234-272) -- same draws in the same order on
  the target device's generator, so inputs match the reference's bit for bit.
* ``seeded_model``: CPU default init under ``torch.manual_seed(seed)``
  (torch_transformer_benchmark.py:672-680) for any model class with the
  reference parameter tree; C5 scales every nn.Linear weight and bias by 0.5.
* ``valid_lengths`` / ``work``: the algorithmic work counts every reported
  rate divides by.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .candidate import TransformerConfig


@dataclass(frozen=True)
class Workload:
    name: str
    config: TransformerConfig
    padding_ratio: float
    linear_scale: float
    note: str


CONFIGS: Dict[str, Workload] = {
    "C1": Workload("C1", TransformerConfig(4, 512, 256, 8, 1024, 2, True), 0.5, 1.0,
                   "CPU-runnable small model"),
    "C2": Workload("C2", TransformerConfig(16, 2048, 1024, 16, 4096, 4, True), 0.5, 1.0,
                   "mid-size model, batch-sharded"),
    "C3": Workload("C3", TransformerConfig(256, 256, 512, 8, 2048, 4, True), 0.75, 1.0,
                   "many short sequences, batch-sharded"),
    "C4": Workload("C4", TransformerConfig(64, 8192, 768, 12, 3072, 1, True), 0.5, 1.0,
                   "memory-bound extreme batch, batch-sharded"),
    "C5": Workload("C5", TransformerConfig(4, 262144, 1024, 16, 4096, 1, True), 0.0, 0.5,
                   "long-sequence linear-memory, sequence-sharded"),
}


def generate_random_case(config, device, dtype: torch.dtype, seed: int, padding_ratio: float,
                         input_scale: float = 1.0) -> Tuple[torch.Tensor, torch.Tensor]:
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


def seeded_model(model_cls, config, seed: int = 1234, linear_scale: float = 1.0, **kwargs) -> nn.Module:
    torch.manual_seed(seed)
    model = model_cls(config, **kwargs)
    if linear_scale != 1.0:
        with torch.no_grad():
            for mod in model.modules():
                if isinstance(mod, nn.Linear):
                    mod.weight.mul_(linear_scale)
                    mod.bias.mul_(linear_scale)
    return model.eval()


def valid_lengths(mask: Optional[torch.Tensor], batch: int, seq_len: int) -> List[int]:
    if mask is None:
        return [seq_len] * batch
    pos = torch.arange(1, seq_len + 1, device=mask.device)[None, :]
    return [int(v) for v in (mask.to(torch.int64) * pos).amax(dim=1).cpu()]


def work(config, lengths: List[int]) -> Dict[str, float]:
    """Algorithmic work over valid tokens (no padded rows, no masked pairs).

    gemm_flops  = L * 2 * T_v * (4 d^2 + 2 d F)   (QKV 3d^2, out d^2, FFN 2dF per token)
    attn_flops  = L * 2 * d * sum_b l_b (l_b + 1)  (causal QK^T + PV; non-causal 4 d l^2)
    per-GEMM-class flops are returned too, for per-kernel rooflines.
    """
    L, d, F_ = config.num_layers, config.d_model, config.ffn_dim
    tv = float(sum(lengths))
    if config.causal:
        attn = L * 2.0 * d * sum(l * (l + 1) for l in lengths)
    else:
        attn = L * 4.0 * d * sum(l * l for l in lengths)
    return {
        "tokens_valid": tv,
        "gemm_flops": L * 2.0 * tv * (4 * d * d + 2 * d * F_),
        "attn_flops": attn,
        "gemm_qkv_flops": L * 2.0 * tv * 3 * d * d,
        "gemm_out_flops": L * 2.0 * tv * d * d,
        "gemm_ffn_in_flops": L * 2.0 * tv * d * F_,
        "gemm_ffn_out_flops": L * 2.0 * tv * d * F_,
        # LayerNorm bytes: read fp32 row, write fp16 row (2L of them) + final fp32->fp32
        "ln_bytes": L * 2 * tv * d * (4 + 2) + tv * d * 8,
    }
