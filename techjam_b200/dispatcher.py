"""Candidate entry point: ``CANDIDATE`` for the reference's ``--candidate`` loader.

Mirrors the role of the reference's ``src/dispatcher.py`` (``CANDIDATE``
:797-818, ``DispatchingTransformer`` :267-794): the benchmark harness builds
the model with ``CANDIDATE.model_factory(config)`` on the CPU, copies the
baseline's weights with a strict ``load_state_dict``, moves it with
``.to(device, dtype).eval()`` and calls ``model(x, valid_token_mask)``.

Unlike the reference, no configuration is routed to a PyTorch path: every
CUDA forward runs the sm_100a kernels of ``libtj.so`` and a non-CUDA input
raises (``UnsupportedCaseError``, as the reference does before unsafe work,
src/dispatcher.py:141-142).  The attention route -- exact flash or the guarded
polynomial route -- is chosen per call by the library (``attention_route``).
"""

from __future__ import annotations

from typing import Optional

import torch

from .candidate import CandidateSpec
from .model import B200Transformer


class UnsupportedCaseError(RuntimeError):
    """Raised before work the B200 path cannot do (non-CUDA input, bad dtype)."""


class DispatchingTransformer(B200Transformer):
    """``B200Transformer`` with the reference dispatcher's error contract."""

    def __init__(self, config, attention_route: str = "auto") -> None:
        super().__init__(config, attention_route=attention_route)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.device.type != "cuda":
            raise UnsupportedCaseError("the B200 candidate requires CUDA input on an sm_100 device")
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise UnsupportedCaseError(f"unsupported input dtype {x.dtype}")
        return super().forward(x, valid_token_mask)


CANDIDATE = CandidateSpec(
    name="b200",
    model_factory=DispatchingTransformer,
    owner="techjam-b200",
    description=("B200-native encoder forward: tcgen05/TMEM GEMMs with fused epilogues, flash causal "
                 "attention with tile skipping, fused LayerNorm, guarded polynomial long-sequence route."),
    self_compiling=True,
)
