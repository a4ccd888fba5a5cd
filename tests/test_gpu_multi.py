"""Sequence-sharded forward on 2 GPUs (NCCL), against the single-GPU forward
and the bounded-memory FP32 oracle.  Skipped unless two GPUs are visible."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, results):
    import datetime

    from oracle.reference_model import EncoderShape
    from techjam_b200.dispatcher import DispatchingTransformer
    from techjam_b200.harness import generate_random_case, seeded_model
    from techjam_b200.sharding import (SeqShardComm, forward_seqshard, seqshard_routes, take_tokens, token_range,
                                       token_ranges)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        cfg = EncoderShape(1, 16384, 1024, 16, 4096, 1, True)
        model = seeded_model(DispatchingTransformer, cfg, 1234, 0.5).to(dev)
        x, _ = generate_random_case(cfg, dev, torch.float32, 77, 0.0)
        comm = SeqShardComm(dev)
        rng = token_range(cfg.seq_len, WORLD, rank)
        outs = {}
        with torch.inference_mode():
            for route in ("exact", "auto"):
                y = forward_seqshard(model, comm, x[:, rng.start:rng.stop].contiguous(), route)
                parts = [torch.empty_like(y) for _ in range(WORLD)]
                dist.all_gather(parts, y)
                outs[route] = torch.cat(parts, dim=1).cpu()
                if route == "exact":
                    assert seqshard_routes(model) == [-1]  # the exact route runs no guard
            # zig-zag layout on the exact route: rank r holds chunks r and 3-r of 4096 tokens
            zz = token_ranges(cfg.seq_len, WORLD, rank, "zigzag")
            y = forward_seqshard(model, comm, take_tokens(x, zz), "exact", "zigzag")
            parts = [torch.empty_like(y) for _ in range(WORLD)]
            dist.all_gather(parts, y)
            full = torch.empty_like(x)
            for r, part in enumerate(parts):
                col = 0
                for rg in token_ranges(cfg.seq_len, WORLD, r, "zigzag"):
                    full[:, rg.start:rg.stop] = part[:, col:col + len(rg)]
                    col += len(rg)
            outs["exact_zigzag"] = full.cpu()
            # the pooled guard admitted the polynomial route (sigma ~0.08 at 0.5x weights) ...
            assert seqshard_routes(model) == [1]
            # ... and a second forward reuses the cached verdict (no guard, no host read) with the same result
            y2 = forward_seqshard(model, comm, x[:, rng.start:rng.stop].contiguous(), "auto")
            parts = [torch.empty_like(y2) for _ in range(WORLD)]
            dist.all_gather(parts, y2)
            outs["auto_cached"] = torch.cat(parts, dim=1).cpu()
            torch.cuda.synchronize(dev)
            assert model.device_error() == 0
        if rank == 0:
            results.put({k: v for k, v in outs.items()})
        dist.barrier(device_ids=[rank])
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_sequence_sharded_forward_two_gpus():
    from oracle import linear_memory
    from oracle.reference_model import EncoderShape, check_outputs, generate_random_case, seeded_encoder

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    outs = results.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    dev = torch.device("cuda", 0)
    cfg = EncoderShape(1, 16384, 1024, 16, 4096, 1, True)
    from techjam_b200.dispatcher import DispatchingTransformer
    from techjam_b200.harness import seeded_model
    single = seeded_model(DispatchingTransformer, cfg, 1234, 0.5).to(dev)
    oracle = seeded_encoder(cfg, 1234, 0.5).to(dev)
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.inference_mode():
            x, _ = generate_random_case(cfg, dev, torch.float32, 77, 0.0)
            single.attention_route = "exact"
            ref_exact = single(x, None).cpu()
            ref = linear_memory.linear_memory_forward(oracle, x, None, q_chunk=1024).cpu()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    # exact route: same kernels, same key tiles in the same order -> identical
    assert torch.equal(outs["exact"], ref_exact)
    assert torch.equal(outs["exact_zigzag"], ref_exact)
    assert torch.equal(outs["auto_cached"], outs["auto"])
    for route in ("exact", "auto"):
        v = check_outputs(ref, outs[route])
        assert v.passed, f"{route}: {v.failed_elements} failed, max_abs={v.max_abs_error:.3g}"
