"""Host-side mirror of the reference's candidate contract.

``CandidateSpec`` keeps the field names, defaults and validation rules of the
reference's ``src/infra/candidate.py:15-130``, and ``validate_candidate_execution``
its pre-allocation contract checks (:165-232), so that a module exposing
``CANDIDATE`` here can be consumed by the reference's loader
(``load_candidate``, :133-162) once re-wrapped in its own class (two lines:
build the reference's ``CandidateSpec`` from this one's fields);
``TransformerConfig`` mirrors
``torch_transformer_benchmark.py:29-56`` field for field so the model factory
accepts either class.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any, Callable, Optional, Tuple

ModelFactory = Callable[[Any], Any]
WeightLoader = Callable[[Any, Any, bool], None]


@dataclass(frozen=True)
class TransformerConfig:
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
        if self.d_model % self.num_heads != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by num_heads ({self.num_heads})")


@dataclass(frozen=True)
class CandidateSpec:
    """Description and construction hooks for one full-model candidate."""

    name: str
    model_factory: ModelFactory
    owner: str
    description: str
    weight_loader: Optional[WeightLoader] = None
    strict_weight_copy: bool = True
    self_compiling: bool = False
    unsupported_official_cases: Tuple[int, ...] = ()
    official_case_dtypes: Tuple[Tuple[int, Tuple[str, ...]], ...] = ()
    candidate_only_official_cases: Tuple[int, ...] = ()
    default_input_scale_only_cases: Tuple[int, ...] = ()
    cuda_only_official_cases: Tuple[int, ...] = ()
    official_case_min_cuda_capability: Tuple[Tuple[int, Tuple[int, int]], ...] = ()
    official_case_torch_versions: Tuple[Tuple[int, Tuple[str, ...]], ...] = ()

    def validate(self) -> None:
        if not re.fullmatch(r"[a-z0-9][a-z0-9_-]*", self.name):
            raise ValueError("candidate name must contain only lowercase letters, numbers, underscores, and hyphens")
        if not callable(self.model_factory):
            raise TypeError("candidate model_factory must be callable")
        if self.weight_loader is not None and not callable(self.weight_loader):
            raise TypeError("candidate weight_loader must be callable")
        if not isinstance(self.self_compiling, bool):
            raise TypeError("candidate self_compiling must be a bool")

        def ids_ok(ids):
            return isinstance(ids, tuple) and all(isinstance(i, int) and 1 <= i <= 14 for i in ids)

        for ids, label in ((self.unsupported_official_cases, "unsupported"),
                           (self.candidate_only_official_cases, "candidate-only"),
                           (self.default_input_scale_only_cases, "default-input-scale"),
                           (self.cuda_only_official_cases, "CUDA-only")):
            if not ids_ok(ids):
                raise ValueError(f"{label} official cases must contain ids 1 through 14")
        if len(set(self.unsupported_official_cases)) != len(self.unsupported_official_cases):
            raise ValueError("unsupported official cases must not contain duplicates")
        for pairs, label in ((self.official_case_dtypes, "dtype"),
                             (self.official_case_min_cuda_capability, "capability"),
                             (self.official_case_torch_versions, "version")):
            seen = set()
            for case_id, _ in pairs:
                if not isinstance(case_id, int) or not 1 <= case_id <= 14 or case_id in seen:
                    raise ValueError(f"{label} contracts need distinct case ids 1 through 14")
                seen.add(case_id)
        for _, dtypes in self.official_case_dtypes:
            if not dtypes or any(t not in ("float32", "float16", "bfloat16") for t in dtypes):
                raise ValueError("dtype contracts contain an unsupported dtype name")
        for _, cap in self.official_case_min_cuda_capability:
            if not (isinstance(cap, tuple) and len(cap) == 2 and all(isinstance(v, int) and v >= 0 for v in cap)):
                raise TypeError("CUDA capabilities must be non-negative integer pairs")


def validate_candidate_execution(spec: CandidateSpec, official_case_id: Optional[int], *, compile_user: bool = False,
                                 dtype_name: Optional[str] = None, candidate_only: bool = False,
                                 input_scale: float = 1.0, device_type: Optional[str] = None,
                                 cuda_capability: Optional[Tuple[int, int]] = None,
                                 torch_version: Optional[str] = None) -> None:
    """Refuse a run that breaks the candidate's declared contract, before any
    model or input is allocated (restates ``validate_candidate_execution``,
    src/infra/candidate.py:165-232; same checks, same order)."""
    if spec.self_compiling and compile_user:
        raise ValueError(f"candidate {spec.name!r} compiles itself; remove --compile-user to avoid nested compilation")
    if official_case_id in spec.unsupported_official_cases:
        raise ValueError(f"candidate {spec.name!r} explicitly does not support official case {official_case_id}; "
                         "refusing before model/input allocation")
    dtypes = dict(spec.official_case_dtypes).get(official_case_id)
    if dtypes is not None and dtype_name not in dtypes:
        raise ValueError(f"candidate {spec.name!r} supports official case {official_case_id} only with "
                         f"{', '.join(dtypes)}; received {dtype_name}; refusing before model/input allocation")
    if official_case_id in spec.candidate_only_official_cases and not candidate_only:
        raise ValueError(f"official case {official_case_id} has no runnable dense baseline; "
                         "use the candidate-only runner")
    if official_case_id in spec.default_input_scale_only_cases and input_scale != 1.0:
        raise ValueError(f"official case {official_case_id} is validated only at the default input scale 1.0")
    if official_case_id in spec.cuda_only_official_cases and device_type != "cuda":
        raise ValueError(f"official case {official_case_id} requires CUDA; refusing before model/input allocation")
    cap = dict(spec.official_case_min_cuda_capability).get(official_case_id)
    if cap is not None and (cuda_capability is None or tuple(cuda_capability) < tuple(cap)):
        raise ValueError(f"official case {official_case_id} requires CUDA capability {cap} or newer; "
                         "refusing before model/input allocation")
    versions = dict(spec.official_case_torch_versions).get(official_case_id)
    if versions is not None and torch_version not in versions:
        raise ValueError(f"official case {official_case_id} requires PyTorch {', '.join(versions)}; "
                         "refusing before model/input allocation")
