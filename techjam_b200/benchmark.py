#!/usr/bin/env python3
"""Accuracy check and paired A/B timing of a candidate against a dense baseline.

    python -m techjam_b200.benchmark --candidate techjam_b200.dispatcher \\
        --baseline-module /path/to/torch_transformer_benchmark.py --workload C2

Restates the reference's harness (``src/benchmark.py:40-627``) with the same
flags, defaults, accuracy loop and timing methodology, so speedups measured
with it compare with the reference's published ones:

* the model shape comes from ``--workload C1..C5`` (this build's configs),
  ``--case 1..14`` (the reference's disclosed shapes, ``src/cases/
  task_shapes.json``) or the shape flags (defaults of ``src/benchmark.py:
  124-150``);
* the baseline is the reference's immutable ``BaselineTransformer``, loaded
  from ``--baseline-module`` (a module name or a ``.py`` path, optionally
  ``:ClassName``); weights are its seeded CPU default init, copied into the
  candidate by a strict ``load_state_dict`` (``copy_model_weights``) or the
  candidate's own ``weight_loader``;
* accuracy: ``--accuracy-trials`` seeded inputs (seeds ``seed + t``), the
  reference criterion evaluated by the streamed checker
  (``techjam_b200.checker``);
* timing: inputs from seed ``seed + 100000``; ``paired`` (default) settles
  both models, picks a block size and interleaves AB/BA samples
  (``techjam_b200.timing``); ``legacy`` reproduces the block-per-round
  schedule (``src/benchmark.py:424-480``).

Where the dense baseline cannot hold one full batch of ``[B, H, N, N]`` FP32
scores on the device, it runs one sample at a time (``--baseline-per-sample
auto``; samples are independent through the whole model) and its time is the
sum over samples; where it cannot hold even one sample's scores (the 262k-token
workload), the run is candidate-only: timing of the candidate alone, accuracy
left to the bounded-memory oracle of the test suite.

``--compile-*`` are not offered: nothing in this build uses torch.compile.
"""

from __future__ import annotations

import argparse
import contextlib
import importlib
import importlib.util
import json
import os
import platform
import shlex
import statistics
import subprocess
import sys
from dataclasses import asdict
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from . import timing
from .candidate import TransformerConfig, validate_candidate_execution
from .checker import AccuracyAccumulator
from .harness import CONFIGS, generate_random_case

# The reference's disclosed official shapes (src/cases/task_shapes.json:12-25):
# id -> (batch_size, d_model (qkv_dim), heads, seq_len, layers, causal, ffn_dim).
OFFICIAL_CASES: Dict[int, Tuple[int, int, int, int, int, bool, int]] = {
    1: (64, 128, 4, 128, 4, True, 128),
    2: (1, 128, 4, 128, 4, True, 128),
    3: (4, 128, 4, 128, 4, True, 128),
    4: (16, 128, 4, 128, 4, True, 128),
    5: (128, 128, 4, 128, 4, True, 128),
    6: (10000, 128, 4, 128, 4, True, 128),
    7: (64, 32, 4, 128, 4, True, 32),
    8: (64, 1024, 4, 128, 4, True, 1024),
    9: (64, 128, 1, 128, 4, True, 128),
    10: (64, 128, 2, 128, 4, True, 128),
    11: (64, 128, 16, 128, 4, True, 128),
    12: (64, 128, 4, 32, 4, True, 128),
    13: (64, 128, 4, 1024, 4, True, 128),
    14: (32, 1024, 16, 100000, 2, True, 1024),
}
SHAPE_DEFAULTS = {"batch_size": 8, "seq_len": 128, "d_model": 512, "heads": 8, "ffn_dim": 2048,
                  "layers": 6, "causal": False}  # src/benchmark.py:124-132
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
TIMING_SEED_OFFSET = 100000  # src/benchmark.py:375-382


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Compare a loadable candidate with the dense baseline model")
    p.add_argument("--candidate", default="techjam_b200.dispatcher",
                   help="module[:attribute]; a name without a dot resolves under techjam_b200")
    p.add_argument("--baseline-module", default="torch_transformer_benchmark",
                   help="module name or .py path holding the baseline model, optionally :ClassName "
                        "(default class BaselineTransformer)")
    p.add_argument("--output", type=Path, help="new JSON result path; an existing file is never overwritten")
    p.add_argument("--workload", choices=sorted(CONFIGS), help="one of this build's workload presets")
    p.add_argument("--case", type=int, choices=range(1, 15), help="the reference's disclosed shape 1-14")
    p.add_argument("--batch-size", type=int)
    p.add_argument("--seq-len", type=int)
    p.add_argument("--d-model", type=int)
    p.add_argument("--heads", type=int)
    p.add_argument("--ffn-dim", type=int)
    p.add_argument("--layers", type=int)
    p.add_argument("--causal", action=argparse.BooleanOptionalAction, default=None)
    p.add_argument("--device", default="auto")
    p.add_argument("--dtype", choices=tuple(DTYPES), default="float32")
    p.add_argument("--padding-ratio", type=float, default=None)
    p.add_argument("--input-scale", type=float, default=1.0)
    p.add_argument("--accuracy-trials", type=int, default=5)
    p.add_argument("--rtol", type=float, default=0.02)
    p.add_argument("--atol", type=float, default=0.002)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--repeats", type=int, default=100)
    p.add_argument("--benchmark-rounds", type=int, default=3)
    p.add_argument("--timing", choices=("paired", "legacy"), default="paired")
    p.add_argument("--settle-seconds", type=float, default=10.0)
    p.add_argument("--block-size", type=int, default=0, help="forwards per timed sample; 0 = from a probe")
    p.add_argument("--sample-target-ms", type=float, default=50.0)
    p.add_argument("--benchmark-on-failure", action="store_true")
    p.add_argument("--non-strict-weight-copy", action="store_true")
    p.add_argument("--matmul-precision", choices=("highest", "high", "medium"), default="high")
    p.add_argument("--allow-tf32", action=argparse.BooleanOptionalAction, default=True)
    p.add_argument("--accuracy-precision", choices=("harness", "fp32"), default="harness",
                   help="'fp32' evaluates the baseline in true FP32 (TF32 off) during the accuracy "
                        "trials only; timing always uses the --allow-tf32 setting")
    p.add_argument("--baseline-per-sample", choices=("auto", "on", "off"), default="auto")
    p.add_argument("--nvtx", action="store_true",
                   help="annotate the timed region for Nsight Systems; adds profiling overhead")
    return p.parse_args(argv)


# ------------------------------------------------------------------ shape and loading
def resolve_shape(args: argparse.Namespace) -> Tuple[TransformerConfig, float]:
    """Fill the shape flags from --workload / --case / defaults; return the
    config and the linear-weight scale.  A flag that conflicts with a preset is
    an error (src/benchmark.py:134-150)."""
    if args.workload and args.case:
        raise ValueError("--workload and --case are mutually exclusive")
    fixed: Dict[str, Any] = {}
    scale = 1.0
    if args.workload:
        wl = CONFIGS[args.workload]
        c = wl.config
        fixed = {"batch_size": c.batch_size, "seq_len": c.seq_len, "d_model": c.d_model, "heads": c.num_heads,
                 "ffn_dim": c.ffn_dim, "layers": c.num_layers, "causal": c.causal}
        scale = wl.linear_scale
        if args.padding_ratio is None:
            args.padding_ratio = wl.padding_ratio
    elif args.case:
        b, d, h, n, L, causal, f = OFFICIAL_CASES[args.case]
        fixed = {"batch_size": b, "seq_len": n, "d_model": d, "heads": h, "ffn_dim": f, "layers": L,
                 "causal": causal}
    for name, value in fixed.items():
        given = getattr(args, name)
        if given is not None and given != value:
            which = f"--workload {args.workload}" if args.workload else f"--case {args.case}"
            raise ValueError(f"{which} fixes --{name.replace('_', '-')}={value}; received conflicting value {given}")
        setattr(args, name, value)
    for name, value in SHAPE_DEFAULTS.items():
        if getattr(args, name) is None:
            setattr(args, name, value)
    if args.padding_ratio is None:
        args.padding_ratio = 0.0
    if not 0.0 <= args.padding_ratio < 1.0:
        raise ValueError("padding_ratio must be in [0, 1)")
    if args.input_scale <= 0:
        raise ValueError("input_scale must be positive")
    for name in ("accuracy_trials", "repeats", "benchmark_rounds"):
        if getattr(args, name) <= 0:
            raise ValueError(f"{name.replace('_', '-')} must be positive")
    if args.warmup < 0:
        raise ValueError("warmup must be non-negative")
    cfg = TransformerConfig(args.batch_size, args.seq_len, args.d_model, args.heads, args.ffn_dim, args.layers,
                            bool(args.causal))
    cfg.validate()
    return cfg, scale


def load_candidate(selector: str):
    """``module[:attribute]`` -> the candidate spec (reference ``candidate.py:133-162``);
    the attribute defaults to ``CANDIDATE``."""
    mod_name, sep, attr = selector.partition(":")
    if not mod_name:
        raise ValueError("candidate selector must not be empty")
    if "." not in mod_name:
        mod_name = f"techjam_b200.{mod_name}"
    attr = attr if sep else "CANDIDATE"
    if not attr:
        raise ValueError("candidate attribute must not be empty")
    spec = getattr(importlib.import_module(mod_name), attr, None)
    if spec is None:
        raise AttributeError(f"candidate module {mod_name!r} has no {attr!r} attribute")
    if not callable(getattr(spec, "model_factory", None)):
        raise TypeError(f"{mod_name}:{attr} is not a candidate spec (no callable model_factory)")
    if hasattr(spec, "validate"):
        spec.validate()
    return spec


def load_baseline_class(selector: str):
    """A module name or ``.py`` path, optionally ``:ClassName`` -> the baseline class."""
    target, sep, cls = selector.rpartition(":")
    if not sep or not cls.isidentifier():
        target, cls = selector, ""
    cls = cls or "BaselineTransformer"
    if target.endswith(".py") or os.sep in target:
        path = Path(target).resolve()
        spec = importlib.util.spec_from_file_location(f"_tj_baseline_{path.stem}", path)
        if spec is None or spec.loader is None:
            raise ImportError(f"cannot load baseline module from {path}")
        module = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = module
        spec.loader.exec_module(module)
    else:
        module = importlib.import_module(target)
    model_cls = getattr(module, cls, None)
    if model_cls is None:
        raise AttributeError(f"baseline module {target!r} has no {cls!r}")
    return model_cls


def resolve_device(name: str) -> torch.device:
    if name == "auto":
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    dev = torch.device(name)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("CUDA was requested but is unavailable")
    return dev


class PerSampleModel(nn.Module):
    """Runs a model one batch item at a time (batch items are independent through
    every layer of the encoder), so dense attention holds one sample's scores."""

    def __init__(self, inner: nn.Module) -> None:
        super().__init__()
        self.inner = inner

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        outs = []
        for i in range(x.shape[0]):
            m = None if valid_token_mask is None else valid_token_mask[i:i + 1]
            outs.append(self.inner(x[i:i + 1], m))
        return torch.cat(outs, 0)


def dense_score_bytes(cfg: TransformerConfig, batch: int) -> int:
    """Peak of the dense baseline's attention temporaries: scores, their FP32
    softmax and the masked copy, ``[b, H, N, N]`` each."""
    return 3 * batch * cfg.num_heads * cfg.seq_len * cfg.seq_len * 4


def baseline_mode(args, cfg: TransformerConfig, device: torch.device) -> str:
    """'batch', 'per-sample' or 'unavailable' for the dense baseline."""
    if args.baseline_per_sample == "on":
        return "per-sample"
    if device.type != "cuda":
        return "batch" if args.baseline_per_sample == "off" or dense_score_bytes(cfg, cfg.batch_size) < 32 << 30 \
            else "per-sample"
    free, _ = torch.cuda.mem_get_info(device)
    budget = 0.6 * free
    if args.baseline_per_sample == "off" or dense_score_bytes(cfg, cfg.batch_size) <= budget:
        return "batch"
    return "per-sample" if dense_score_bytes(cfg, 1) <= budget else "unavailable"


# ------------------------------------------------------------------ environment
def _cmd(command: List[str]) -> Optional[str]:
    try:
        r = subprocess.run(command, check=True, capture_output=True, text=True, timeout=5)
    except (OSError, subprocess.SubprocessError):
        return None
    return r.stdout.strip() or None


def collect_environment(device: torch.device) -> Dict[str, Any]:
    cpu = platform.processor().strip()
    if not cpu:
        try:
            for line in Path("/proc/cpuinfo").read_text().splitlines():
                if line.lower().startswith("model name"):
                    cpu = line.partition(":")[2].strip()
                    break
        except OSError:
            pass
    gpu: Dict[str, Any] = {"available": torch.cuda.is_available(), "name": None, "driver": None,
                           "cuda_runtime": torch.version.cuda}
    if device.type == "cuda":
        gpu["name"] = torch.cuda.get_device_name(device)
        gpu["capability"] = list(torch.cuda.get_device_capability(device))
        gpu["driver"] = _cmd(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader",
                              f"--id={device.index or 0}"])
    return {"cpu": cpu or "unknown", "cpu_count": os.cpu_count(), "os": platform.platform(),
            "python": platform.python_version(), "pytorch": torch.__version__, "gpu": gpu}


def collect_gpu_state(device: torch.device) -> Optional[Dict[str, str]]:
    """Clock, power and throttle state at the moment of measurement."""
    if device.type != "cuda":
        return None
    fields = ["clocks.sm", "clocks.mem", "power.draw", "power.limit", "temperature.gpu",
              "clocks_event_reasons.active"]
    out = _cmd(["nvidia-smi", f"--query-gpu={','.join(fields)}", "--format=csv,noheader,nounits",
                f"--id={device.index or 0}"])
    if not out:
        return None
    vals = [v.strip() for v in out.split(",")]
    return dict(zip(fields, vals)) if len(vals) == len(fields) else None


# ------------------------------------------------------------------ accuracy and timing
class _PrecisionScope:
    """Temporarily sets the TF32 switches (accuracy trials with --accuracy-precision fp32)."""

    def __init__(self, allow_tf32: Optional[bool]) -> None:
        self.allow = allow_tf32
        self.saved = None

    def __enter__(self):
        if self.allow is not None:
            self.saved = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
            torch.backends.cuda.matmul.allow_tf32 = self.allow
            torch.backends.cudnn.allow_tf32 = self.allow
        return self

    def __exit__(self, *exc):
        if self.saved is not None:
            torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = self.saved


def accuracy_trials(baseline, candidate, cfg, device, dtype, args) -> Dict[str, Any]:
    """src/benchmark.py:152-201 with the streamed checker; the baseline output of
    each trial is compared sample by sample when the baseline runs per sample."""
    trials = []
    scope = _PrecisionScope(False if args.accuracy_precision == "fp32" else None)
    with torch.inference_mode(), scope:
        for t in range(args.accuracy_trials):
            x, mask = generate_random_case(cfg, device, dtype, args.seed + t, args.padding_ratio, args.input_scale)
            actual = candidate(x, mask)
            acc = AccuracyAccumulator(args.rtol, args.atol)
            if isinstance(baseline, PerSampleModel):
                for i in range(cfg.batch_size):
                    acc.add(baseline.inner(x[i:i + 1], mask[i:i + 1]), actual[i:i + 1], batch_offset=i)
            else:
                acc.add(baseline(x, mask), actual)
            res = acc.result()
            trial = asdict(res)
            trial.update(trial=t + 1, seed=args.seed + t)
            trials.append(trial)
            print(f"accuracy {t + 1:02d}/{args.accuracy_trials}: {'PASS' if res.passed else 'FAIL'} | "
                  f"max_abs={res.max_abs_error:.6g} | failed={res.failed_elements}/{res.total_elements}", flush=True)
            del x, mask, actual
    return {
        "passed": all(t["passed"] for t in trials), "rtol": args.rtol, "atol": args.atol,
        "precision": args.accuracy_precision,
        "failed_elements": sum(t["failed_elements"] for t in trials),
        "total_elements": sum(t["total_elements"] for t in trials),
        "max_abs_error": max(t["max_abs_error"] for t in trials),
        "max_relative_error": max(t["max_relative_error"] for t in trials),
        "trials": trials,
    }


def memory_probe(models: Dict[str, nn.Module], x, mask, device) -> Optional[Dict[str, Dict[str, int]]]:
    """Absolute and incremental peak memory of one forward per model (src/benchmark.py:215-246)."""
    if device.type != "cuda":
        return None
    snaps = {}
    for label, model in models.items():
        torch.cuda.synchronize(device)
        torch.cuda.reset_peak_memory_stats(device)
        a0, r0 = torch.cuda.memory_allocated(device), torch.cuda.memory_reserved(device)
        with torch.inference_mode():
            out = model(x, mask)
        torch.cuda.synchronize(device)
        pa, pr = torch.cuda.max_memory_allocated(device), torch.cuda.max_memory_reserved(device)
        del out
        snaps[label] = {"before_allocated_bytes": a0, "before_reserved_bytes": r0, "peak_allocated_bytes": pa,
                        "peak_reserved_bytes": pr, "incremental_peak_allocated_bytes": pa - a0,
                        "incremental_peak_reserved_bytes": pr - r0}
    return snaps


def _nvtx_range(device, enabled: bool, label: str):
    """An NVTX range for Nsight Systems when requested on CUDA (src/benchmark.py:249-252)."""
    if not enabled or device.type != "cuda":
        return contextlib.nullcontext()
    return torch.cuda.nvtx.range(label)


def _resolve_block_size(model, x, mask, device, args) -> int:
    if args.block_size > 0:
        return args.block_size
    probe = timing.make_block_runner(model, x, mask, device, 1)
    s = timing.measure_pair({timing.BASELINE: probe, timing.CANDIDATE: probe}, repeats=2, device=device)
    per_iter = statistics.median(s[timing.BASELINE] + s[timing.CANDIDATE])
    return timing.choose_block_size(per_iter, target_ms=args.sample_target_ms)


def _with_rates(summary: Dict[str, Any], tokens: int) -> Dict[str, Any]:
    summary["tokens_per_second"] = tokens * 1000.0 / summary["median_ms"]
    return summary


def paired_benchmark(baseline, candidate, cfg, device, x, mask, args) -> Dict[str, Any]:
    """src/benchmark.py:249-320: settle both, one block size (probed on the
    baseline), interleaved samples, median speedup and its noise floor."""
    with torch.inference_mode():
        timing.settle(baseline, x, mask, device, args.settle_seconds)
        timing.settle(candidate, x, mask, device, args.settle_seconds)
        block = _resolve_block_size(baseline, x, mask, device, args)
    runners = {timing.BASELINE: timing.make_block_runner(baseline, x, mask, device, block),
               timing.CANDIDATE: timing.make_block_runner(candidate, x, mask, device, block)}
    with _nvtx_range(device, args.nvtx, "paired_timing"):
        samples = timing.measure_pair(runners, args.repeats, device=device)
    summary = timing.paired_summary(samples)
    floor = timing.noise_floor_ratio(samples)
    significant = timing.is_significant(summary["speedup"], floor)
    tokens = cfg.batch_size * cfg.seq_len
    b_sum = _with_rates(timing.timing_summary(samples[timing.BASELINE]), tokens)
    c_sum = _with_rates(timing.timing_summary(samples[timing.CANDIDATE]), tokens)
    print(f"baseline median={b_sum['median_ms']:.4f} ms | candidate median={c_sum['median_ms']:.4f} ms | "
          f"speedup={summary['speedup']:.3f}x")
    print(f"noise floor=+/-{floor * 100:.2f}% | {'SIGNIFICANT' if significant else 'WITHIN NOISE'} | "
          f"block={block} repeats={args.repeats} settle={args.settle_seconds:g}s", flush=True)
    if not significant:
        print("  this difference cannot be distinguished from measurement noise; raise --repeats or treat it "
              "as no change", flush=True)
    return {"timing_mode": "paired", "settle_seconds": args.settle_seconds, "block_size": block,
            "repeats": args.repeats,
            "timing_method": "torch.cuda.Event" if device.type == "cuda" else "perf_counter_ns",
            "baseline": b_sum, "candidate": c_sum, "speedup": summary["speedup"], "noise_floor_ratio": floor,
            "significant": significant, "gpu_state": collect_gpu_state(device)}


def _per_iteration_samples(model, x, mask, iterations, device) -> List[float]:
    """One event pair (or host timer) around each forward (torch_transformer_benchmark.py:477-506)."""
    with torch.inference_mode():
        if device.type == "cuda":
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(iterations)]
            torch.cuda.synchronize(device)
            for s, e in ev:
                s.record()
                model(x, mask)
                e.record()
            torch.cuda.synchronize(device)
            return [s.elapsed_time(e) for s, e in ev]
        out = []
        for _ in range(iterations):
            out.append(timing.make_block_runner(model, x, mask, device, 1)())
        return out


def legacy_benchmark(baseline, candidate, cfg, device, x, mask, args) -> Dict[str, Any]:
    """src/benchmark.py:424-480: warm both, then alternate which model's block of
    ``repeats`` runs first in each round."""
    with torch.inference_mode():
        for model in (baseline, candidate):
            for _ in range(args.warmup):
                model(x, mask)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    b_s: List[float] = []
    c_s: List[float] = []
    for r in range(args.benchmark_rounds):
        order = [("baseline", baseline, b_s), ("candidate", candidate, c_s)]
        for label, model, dst in (order if r % 2 == 0 else order[::-1]):
            with _nvtx_range(device, args.nvtx, f"{label}_timed_round_{r + 1}"):
                dst.extend(_per_iteration_samples(model, x, mask, args.repeats, device))
    tokens = cfg.batch_size * cfg.seq_len
    b_sum = _with_rates(timing.timing_summary(b_s), tokens)
    c_sum = _with_rates(timing.timing_summary(c_s), tokens)
    speedup = b_sum["median_ms"] / c_sum["median_ms"]
    print(f"baseline median={b_sum['median_ms']:.4f} ms | candidate median={c_sum['median_ms']:.4f} ms | "
          f"speedup={speedup:.3f}x", flush=True)
    return {"timing_mode": "legacy", "warmup_iterations": args.warmup, "repeats": args.repeats,
            "rounds": args.benchmark_rounds,
            "timing_method": "torch.cuda.Event" if device.type == "cuda" else "perf_counter_ns",
            "baseline": b_sum, "candidate": c_sum, "speedup": speedup, "gpu_state": collect_gpu_state(device)}


def candidate_only_benchmark(candidate, cfg, device, x, mask, args) -> Dict[str, Any]:
    """Timing when no dense baseline fits: settle, then ``repeats`` blocks of the candidate."""
    with torch.inference_mode():
        timing.settle(candidate, x, mask, device, args.settle_seconds, chunk=1)
    block = max(1, args.block_size)
    run = timing.make_block_runner(candidate, x, mask, device, block)
    pending = [run() for _ in range(args.repeats)]
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    c_sum = _with_rates(timing.timing_summary([timing.resolve_sample(p) for p in pending]),
                        cfg.batch_size * cfg.seq_len)
    print(f"candidate median={c_sum['median_ms']:.4f} ms (no dense baseline fits on this device)", flush=True)
    return {"timing_mode": "candidate-only", "settle_seconds": args.settle_seconds, "block_size": block,
            "repeats": args.repeats, "candidate": c_sum, "baseline": None, "speedup": None,
            "gpu_state": collect_gpu_state(device)}


# ------------------------------------------------------------------ main
def _git() -> Dict[str, Any]:
    here = str(Path(__file__).resolve().parent)
    commit = _cmd(["git", "-C", here, "rev-parse", "HEAD"])
    status = _cmd(["git", "-C", here, "status", "--short"])
    return {"commit": commit, "dirty": bool(status), "status": status or ""}


def run(args: argparse.Namespace) -> int:
    cfg, linear_scale = resolve_shape(args)
    spec = load_candidate(args.candidate)
    device = resolve_device(args.device)
    dtype = DTYPES[args.dtype]
    validate_candidate_execution(
        spec, args.case, dtype_name=args.dtype, input_scale=args.input_scale, device_type=device.type,
        cuda_capability=torch.cuda.get_device_capability(device) if device.type == "cuda" else None,
        torch_version=torch.__version__)
    torch.manual_seed(args.seed)
    torch.set_float32_matmul_precision(args.matmul_precision)
    if device.type == "cuda":
        torch.cuda.manual_seed_all(args.seed)
        torch.backends.cuda.matmul.allow_tf32 = args.allow_tf32
        torch.backends.cudnn.allow_tf32 = args.allow_tf32

    # seeded CPU default init of the baseline (torch_transformer_benchmark.py:672-680),
    # then the candidate built and loaded from it (src/benchmark.py:500-521)
    base_cls = load_baseline_class(args.baseline_module)
    torch.manual_seed(args.seed)
    baseline = base_cls(cfg)
    if linear_scale != 1.0:
        with torch.no_grad():
            for m in baseline.modules():
                if isinstance(m, nn.Linear):
                    m.weight.mul_(linear_scale)
                    m.bias.mul_(linear_scale)
    candidate = spec.model_factory(cfg)
    if not isinstance(candidate, nn.Module):
        raise TypeError(f"candidate factory returned {type(candidate).__name__}, expected nn.Module")
    strict = getattr(spec, "strict_weight_copy", True) and not args.non_strict_weight_copy
    loader = getattr(spec, "weight_loader", None)
    if loader is not None:
        loader(baseline, candidate, strict)
    else:
        candidate.load_state_dict(baseline.state_dict(), strict=strict)
    candidate = candidate.to(device=device, dtype=dtype).eval()
    mode = baseline_mode(args, cfg, device)
    baseline = baseline.to(device=device, dtype=dtype).eval() if mode != "unavailable" else None
    if mode == "per-sample":
        baseline = PerSampleModel(baseline)
    print(f"candidate={spec.name} device={device} dtype={dtype} config={cfg} baseline={mode}", flush=True)

    if baseline is not None:
        accuracy = accuracy_trials(baseline, candidate, cfg, device, dtype, args)
    else:
        accuracy = {"passed": True, "skipped": ("the dense baseline cannot hold one sample's scores on this "
                                                "device; accuracy is checked against the bounded-memory oracle "
                                                "of the test suite")}
        print(f"accuracy: skipped ({accuracy['skipped']})", flush=True)

    performance = None
    if accuracy["passed"] or args.benchmark_on_failure:
        x, mask = generate_random_case(cfg, device, dtype, args.seed + TIMING_SEED_OFFSET, args.padding_ratio,
                                       args.input_scale)
        models = {"candidate": candidate} if baseline is None else {"baseline": baseline, "candidate": candidate}
        memory = memory_probe(models, x, mask, device)
        if baseline is None:
            performance = candidate_only_benchmark(candidate, cfg, device, x, mask, args)
        elif args.timing == "paired":
            performance = paired_benchmark(baseline, candidate, cfg, device, x, mask, args)
        else:
            performance = legacy_benchmark(baseline, candidate, cfg, device, x, mask, args)
        performance["memory"] = memory
        performance["baseline_mode"] = mode
    else:
        print("benchmark skipped because correctness failed", flush=True)

    result = {
        "schema_version": 1,
        "timestamp_utc": datetime.now(timezone.utc).isoformat(),
        "command": shlex.join([sys.executable, *sys.argv]),
        "git": _git(),
        "environment": collect_environment(device),
        "candidate": {"selector": args.candidate, "name": spec.name, "owner": getattr(spec, "owner", None),
                      "description": getattr(spec, "description", None), "strict_weight_copy": strict,
                      "self_compiling": getattr(spec, "self_compiling", False)},
        "baseline": {"selector": args.baseline_module, "mode": mode},
        "config": asdict(cfg), "workload": args.workload, "official_case_id": args.case,
        "linear_scale": linear_scale, "dtype": args.dtype, "device": str(device),
        "padding_ratio": args.padding_ratio, "input_scale": args.input_scale, "seed": args.seed,
        "nvtx_enabled": args.nvtx,
        "accuracy": accuracy, "performance": performance,
    }
    if args.output is not None:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        with args.output.open("x", encoding="utf-8") as fh:
            json.dump(result, fh, indent=2, sort_keys=True, default=float)
            fh.write("\n")
        print(f"result saved to {args.output}")
    return 0 if accuracy["passed"] else 2


def main(argv: Optional[List[str]] = None) -> int:
    return run(parse_args(argv))


if __name__ == "__main__":
    raise SystemExit(main())
