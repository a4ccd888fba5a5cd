#!/usr/bin/env python3
"""Streamed validation of the B200 forward against the bounded-memory FP32 oracle.

    python tests/streamed_validation.py --config C4 --trials 5 [--route auto] [--json out.json]

TEST INFRASTRUCTURE (it imports ``oracle/``).  Restates the flow of the
reference's over-size validation runner (src/case14_fp32_reference.py:111-255):
the oracle model stays resident, every batch item of every seeded trial is
evaluated by the FP32 oracle one sample at a time (attention in query chunks,
memory linear in N), and each sample's output is reduced by the checker at
once, so no full-batch FP32 reference ever exists.  Differences from the
reference runner: the candidate runs the whole batch in one forward (as the
benchmark times it) and is compared slice by slice; the inputs are the
reference generator's full-batch draws (seeds ``seed + t``), i.e. exactly the
tensors the benchmark's accuracy loop would feed.

Before the trials, the oracle itself is checked against the dense FP32 model
on one sample truncated to ``--validate-dense-n`` tokens
(src/case14_fp32_reference.py:80-108).

Exit status 0 iff every element of every trial passes
``|err| <= 0.002 OR |err| <= 2% |ref|`` and every padded row is exactly 0.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from oracle.linear_memory import linear_memory_forward  # noqa: E402
from oracle.reference_model import EncoderShape, check_outputs, generate_random_case, seeded_encoder  # noqa: E402
from techjam_b200.dispatcher import CANDIDATE  # noqa: E402
from techjam_b200.harness import CONFIGS  # noqa: E402


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", choices=sorted(CONFIGS), default="C4")
    p.add_argument("--trials", type=int, default=5)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--route", choices=("auto", "exact", "poly"), default="auto")
    p.add_argument("--samples", type=int, default=0, help="check only the first K samples of each trial (0 = all)")
    p.add_argument("--q-chunk", type=int, default=0, help="oracle query chunk (0 = from the sequence length)")
    p.add_argument("--validate-dense-n", type=int, default=2048)
    p.add_argument("--json", type=Path)
    return p.parse_args(argv)


def _shape(name):
    c = CONFIGS[name].config
    return EncoderShape(c.batch_size, c.seq_len, c.d_model, c.num_heads, c.ffn_dim, c.num_layers, c.causal)


def dense_validation(oracle, cfg, seed, n, pr, dev):
    """The chunked oracle against the dense model on one sample of ``n`` tokens."""
    if n <= 0:
        return {"status": "skipped"}
    small = EncoderShape(1, min(n, cfg.seq_len), cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers, cfg.causal)
    x, mask = generate_random_case(small, dev, torch.float32, seed, pr)
    with torch.inference_mode():
        dense = oracle(x, mask)
        chunked = linear_memory_forward(oracle, x, mask, q_chunk=max(64, small.seq_len // 4))
    v = check_outputs(dense, chunked, rtol=0.0, atol=1e-4)
    return {"status": "pass" if v.passed else "fail", "tokens": small.seq_len, "max_abs_error": v.max_abs_error}


def run(args) -> dict:
    dev = torch.device("cuda")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    wl = CONFIGS[args.config]
    cfg = _shape(args.config)
    oracle = seeded_encoder(cfg, args.seed, wl.linear_scale).to(dev).eval()
    cand = CANDIDATE.model_factory(cfg)
    cand.load_state_dict(oracle.state_dict(), strict=True)
    cand = cand.to(dev).eval()
    cand.attention_route = args.route
    q_chunk = args.q_chunk or (256 if cfg.seq_len > 65536 else 2048)
    report = {"config": args.config, "route": args.route, "trials": [], "q_chunk": q_chunk,
              "dense_validation": dense_validation(oracle, cfg, args.seed, args.validate_dense_n,
                                                   wl.padding_ratio, dev)}
    print(f"dense validation: {report['dense_validation']}", flush=True)
    ok = report["dense_validation"]["status"] != "fail"
    n_samples = cfg.batch_size if args.samples <= 0 else min(args.samples, cfg.batch_size)
    t_oracle = t_cand = 0.0
    with torch.inference_mode():
        for t in range(args.trials):
            seed = args.seed + t
            x, mask = generate_random_case(cfg, dev, torch.float32, seed, wl.padding_ratio)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            got = cand(x, mask)
            torch.cuda.synchronize()
            t_cand += time.perf_counter() - t0
            err_word = cand.device_error()
            padded_zero = bool(torch.all(got[~mask] == 0))
            finite = bool(torch.isfinite(got).all())
            failed = total = 0
            max_abs = 0.0
            for b in range(n_samples):
                t0 = time.perf_counter()
                ref = linear_memory_forward(oracle, x[b:b + 1], mask[b:b + 1], q_chunk=q_chunk)
                torch.cuda.synchronize()
                t_oracle += time.perf_counter() - t0
                v = check_outputs(ref, got[b:b + 1])
                failed += v.failed_elements
                total += v.total_elements
                max_abs = max(max_abs, v.max_abs_error)
                del ref
            passed = failed == 0 and padded_zero and finite and err_word == 0
            ok &= passed
            report["trials"].append({"trial": t + 1, "seed": seed, "samples": n_samples, "passed": passed,
                                     "failed_elements": failed, "total_elements": total, "max_abs_error": max_abs,
                                     "padded_rows_zero": padded_zero, "finite": finite, "device_error": err_word})
            print(f"trial {t + 1}/{args.trials} seed {seed}: {'PASS' if passed else 'FAIL'} | samples={n_samples} "
                  f"| max_abs={max_abs:.4g} | failed={failed}/{total}", flush=True)
            del x, mask, got
    report.update(passed=ok, oracle_seconds=round(t_oracle, 2), candidate_seconds=round(t_cand, 3))
    return report


def main(argv=None) -> int:
    args = parse_args(argv)
    report = run(args)
    print(json.dumps({k: v for k, v in report.items() if k != "trials"}), flush=True)
    if args.json is not None:
        args.json.parent.mkdir(parents=True, exist_ok=True)
        args.json.write_text(json.dumps(report, indent=1) + "\n")
    return 0 if report["passed"] else 2


if __name__ == "__main__":
    sys.exit(main())
