"""``bench.py``'s rate arithmetic on synthetic kernel timings (no GPU): the
dominant kernel's roofline figure, the per-GPU attention rate, and the
polynomial route's exact-equivalent rate, which alone may exceed the peak."""

import pytest

import bench
from techjam_b200 import _lib
from techjam_b200.harness import CONFIGS, work

NAMES = _lib.KERNEL_CLASSES


def _timings(ms_by_class, launches_per_step, steps):
    kms = [0.0] * len(NAMES)
    kcnt = [0] * len(NAMES)
    for n, v in ms_by_class.items():
        kms[NAMES.index(n)] = v
        kcnt[NAMES.index(n)] = launches_per_step.get(n, 1) * steps
    return kms, kcnt


def test_exact_route_rates():
    cfg = CONFIGS["C2"].config
    lengths = [1536] * cfg.batch_size
    kms, kcnt = _timings({"prep": 0.013, "layernorm": 0.28, "gemm_qkv": 0.47, "attention": 0.71, "gemm_out": 0.26,
                          "gemm_ffn_in": 0.62, "gemm_ffn_out": 0.53, "layernorm_final": 0.046},
                         {"layernorm": 8, "gemm_qkv": 4, "attention": 4, "gemm_out": 4, "gemm_ffn_in": 4,
                          "gemm_ffn_out": 4}, steps=10)
    r = bench.kernel_rates(cfg, lengths, lengths, kms, kcnt, 10, 1)
    w = work(cfg, lengths)
    assert r["dominant"] == "attention"
    assert r["kernels"]["attention"]["launches_per_step"] == 4
    # per-launch figure: a quarter of the step's attention flops in a quarter of its time
    assert r["achieved"] == pytest.approx(w["attn_flops"] / 0.71e-3 / 1e12, rel=1e-9)
    assert r["attn_tflops"] == pytest.approx(r["achieved"], rel=1e-9)
    assert r["attn_exact_eq"] is None
    assert r["kernels"]["gemm_ffn_out"]["tflops"] == pytest.approx(w["gemm_ffn_out_flops"] / 0.53e-3 / 1e12, abs=0.1)
    assert sum(k["share"] for k in r["kernels"].values()) == pytest.approx(1.0, abs=1e-3)


@pytest.mark.parametrize("world,prefix_here", [(1, True), (8, True), (8, False)])
def test_polynomial_route_rates(world, prefix_here):
    cfg = CONFIGS["C5"].config
    lengths = [cfg.seq_len] * cfg.batch_size
    mine = [cfg.seq_len // world] * cfg.batch_size
    kms, kcnt = _timings({"gemm_qkv": 5.2 / world, "attention": 0.9 if prefix_here else 0.0, "gemm_ffn_in": 7.7 / world,
                          "poly": 51.4 / world}, {"poly": 2}, steps=10)
    r = bench.kernel_rates(cfg, lengths, mine, kms, kcnt, 10, world, poly_prefix_here=prefix_here)
    assert r["dominant"] == "poly"
    # executed tensor work per GPU stays below the B200 peak; the exact-equivalent rate does not
    assert 100 < r["attn_tflops"] < 1700
    assert r["attn_exact_eq"] > 2000
    pre = min(4096, cfg.seq_len // world) if prefix_here else 0
    poly_flops = 2.0 * 4224 * 80 * cfg.batch_size * cfg.num_heads * (2 * (cfg.seq_len // world) - pre)
    assert r["kernels"]["poly"]["tflops"] == pytest.approx(poly_flops / (51.4 / world * 1e-3) / 1e12, abs=0.1)
