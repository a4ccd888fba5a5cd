"""Host logic of multi-GPU sharding, run as two gloo ranks on the CPU."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from techjam_b200.harness import CONFIGS, generate_random_case, valid_lengths
from techjam_b200.sharding import sample_cost, shard_samples, token_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        for name in ("C2", "C3"):
            wl = CONFIGS[name]
            cfg = wl.config
            _, mask = generate_random_case(cfg, torch.device("cpu"), torch.float32, 101234, wl.padding_ratio)
            lengths = valid_lengths(mask, cfg.batch_size, cfg.seq_len)
            mine = shard_samples(lengths, world, rank, cfg.d_model, cfg.ffn_dim)
            gathered = [None] * world
            dist.all_gather_object(gathered, mine)
            out[name] = (gathered, lengths)
        rng = token_range(262144, world, rank)
        spans = [None] * world
        dist.all_gather_object(spans, (rng.start, rng.stop))
        out["C5"] = spans
        if rank == 0:
            results.put(out)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_partitions_and_balances():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    out = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for name in ("C2", "C3"):
        gathered, lengths = out[name]
        flat = sorted(i for part in gathered for i in part)
        assert flat == list(range(len(lengths)))  # every sample exactly once
        cfg = CONFIGS[name].config
        loads = [sum(sample_cost(lengths[i], cfg.d_model, cfg.ffn_dim) for i in part) for part in gathered]
        assert max(loads) / (sum(loads) / 2) < 1.05  # balanced within 5%
    assert out["C5"] == [(0, 131072), (131072, 262144)]


def test_token_range_rejects_uneven_split():
    with pytest.raises(ValueError):
        token_range(1000, 3, 0)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_zigzag_ranges_partition_and_balance_causal_work(world):
    """Zig-zag: rank r holds chunks r and 2P-1-r; together the ranks cover
    every token once, and each does exactly 1/P of the causal attention work
    (the contiguous split gives the last rank (2P-1)/P^2 of it)."""
    from techjam_b200.sharding import causal_work, take_tokens, token_ranges
    S = 262144
    parts = [token_ranges(S, world, r, "zigzag") for r in range(world)]
    covered = sorted(t for rs in parts for rg in rs for t in (rg.start, rg.stop - 1))
    assert sorted(p for rs in parts for rg in rs for p in range(rg.start, rg.stop, 4096)) == list(range(0, S, 4096))
    assert covered[0] == 0 and covered[-1] == S - 1
    assert all(sum(len(rg) for rg in rs) == S // world for rs in parts)
    work = [causal_work(rs) for rs in parts]
    assert len(set(work)) == 1 and sum(work) == S * (S + 1) // 2
    contiguous = [causal_work(token_ranges(S, world, r)) for r in range(world)]
    assert max(contiguous) / (sum(contiguous) / world) == pytest.approx((2 * world - 1) / world, rel=1e-4)
    # local rows are the two chunks back to back
    x = torch.arange(S).view(1, S, 1)
    local = take_tokens(x, parts[1]).view(-1).tolist()
    assert local == list(parts[1][0]) + list(parts[1][1])
    with pytest.raises(ValueError):
        token_ranges(S + 512, world, 0, "zigzag")


def _gather_main(rank, world, port, results):
    from techjam_b200.sharding import gather_batch_outputs, sample_owners

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = [5, 17, 3, 11, 9, 2, 13]
        owners = sample_owners(lengths, world, 16, 64)
        mine = [i for i, r in enumerate(owners) if r == rank]
        assert mine == shard_samples(lengths, world, rank, 16, 64)
        # every sample's "output" is its index, so rank 0 can check placement
        out_local = torch.stack([torch.full((4, 3), float(i)) for i in mine]) if mine else torch.empty(0, 4, 3)
        full = gather_batch_outputs(out_local, owners)
        part = gather_batch_outputs(out_local, owners, lengths=[2] * len(lengths))  # valid prefixes only
        if rank == 0:
            results.put((owners, full, part))
        else:
            assert full is None and part is None
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_batch_output_gather_lands_every_sample_on_rank0(world):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    owners, full, part = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(set(owners)) == world  # every rank owns a sample
    assert full.shape == (7, 4, 3)
    for i in range(7):
        assert torch.all(full[i] == float(i))
        assert torch.all(part[i, :2] == float(i)) and torch.all(part[i, 2:] == 0)
