"""Multi-GPU execution: one process per GPU (torchrun), NCCL over NVLink.

Two ways the encoder forward shards (the reference has neither; it streams
batch and prefix chunks through one GPU, src/implementations/extreme.py:136-204):

* **Batch sharding** (independent samples): ``shard_samples`` assigns whole
  samples to ranks by a longest-processing-time rule on their algorithmic cost
  (ragged lengths make a contiguous split unbalanced); each rank then runs an
  ordinary forward on its samples, with no collective inside the forward;
  ``gather_batch_outputs`` then lands every sample's output rows in rank 0's
  ``[B, N, d]`` buffer (NCCL point-to-point).
* **Sequence sharding** (one long sequence per sample): ``SeqShardComm`` joins
  libtj's own NCCL communicator (the unique id travels over the existing
  torch.distributed group) and ``forward_seqshard`` runs rank r's tokens --
  the contiguous range ``[r*S/P, (r+1)*S/P)``, or (``layout="zigzag"``, exact
  route) chunks r and 2P-1-r of S/(2P) tokens, which gives every rank the same
  causal attention work; libtj exchanges the polynomial prefix state (or the
  K/V shards on the exact route) with NCCL on the compute stream.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib
from .model import _ROUTES, B200Transformer


def sample_cost(length: int, d_model: int, ffn_dim: int) -> float:
    """Algorithmic flops of one causal sample per layer (GEMMs + exact attention)."""
    return 2.0 * length * (4 * d_model * d_model + 2 * d_model * ffn_dim) + 2.0 * d_model * length * (length + 1)


def shard_samples(lengths: Sequence[int], world: int, rank: int, d_model: int, ffn_dim: int) -> List[int]:
    """Samples of ``rank`` under a longest-processing-time assignment (deterministic)."""
    loads = [0.0] * world
    owner = {}
    order = sorted(((sample_cost(int(l), d_model, ffn_dim), i) for i, l in enumerate(lengths)), reverse=True)
    for cost, i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        loads[r] += cost
        owner[i] = r
    return sorted(i for i, r in owner.items() if r == rank)


def sample_owners(lengths: Sequence[int], world: int, d_model: int, ffn_dim: int) -> List[int]:
    """Owning rank of every sample under ``shard_samples``'s assignment."""
    owner = [0] * len(lengths)
    for r in range(world):
        for i in shard_samples(lengths, world, r, d_model, ffn_dim):
            owner[i] = r
    return owner


def gather_batch_outputs(out_local: torch.Tensor, owners: Sequence[int], out_full=None, dst: int = 0,
                         lengths: Optional[Sequence[int]] = None):
    """Assemble the batch-sharded forward's output on rank ``dst``.

    ``out_local`` is this rank's ``[n_local, N, d]`` output (its samples in
    ascending sample order, as ``shard_samples`` lists them); ``owners[i]`` is
    the rank of sample i.  Rank ``dst`` receives every other rank's samples
    straight into ``out_full`` ``[B, N, d]`` (made here when not given) with
    point-to-point NCCL transfers -- one message per sample, issued as one
    batch so they proceed concurrently -- and copies its own rows locally; it
    returns ``out_full``.  The other ranks return None.  Every rank must call
    this with the same ``owners`` (and ``lengths``).  With ``lengths`` only
    each sample's first ``lengths[i]`` rows (its valid prefix) move; the
    padded rows of ``out_full`` are left as they are, so the caller passes a
    zero-filled buffer (the forward writes padded rows as exact zeros).  The reference returns the whole batch's
    output from one forward (torch_transformer_benchmark.py:162-172); this is
    the step that gives the sharded forward the same result tensor.
    """
    rank = dist.get_rank()
    world = dist.get_world_size()
    if len(owners) == 0 or max(owners) >= world:
        raise ValueError("owners must name a rank of the process group for every sample")
    mine = [i for i, r in enumerate(owners) if r == rank]
    if out_local.shape[0] != len(mine):
        raise ValueError(f"rank {rank} holds {out_local.shape[0]} samples, the assignment gives it {len(mine)}")
    ops = []
    if rank == dst:
        if out_full is None:
            out_full = torch.zeros((len(owners),) + tuple(out_local.shape[1:]), dtype=out_local.dtype,
                                   device=out_local.device)
        for k, i in enumerate(mine):
            n = out_local.shape[1] if lengths is None else int(lengths[i])
            out_full[i, :n].copy_(out_local[k, :n])
        for i, r in enumerate(owners):
            n = out_local.shape[1] if lengths is None else int(lengths[i])
            if r != dst and n > 0:
                ops.append(dist.P2POp(dist.irecv, out_full[i, :n], r))
    else:
        for k, i in enumerate(mine):
            n = out_local.shape[1] if lengths is None else int(lengths[i])
            if n > 0:
                ops.append(dist.P2POp(dist.isend, out_local[k, :n].contiguous(), dst))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return out_full if rank == dst else None


def token_range(seq_len: int, world: int, rank: int) -> range:
    """Global token positions held by ``rank`` under sequence sharding."""
    if seq_len % world:
        raise ValueError(f"seq_len {seq_len} not divisible by {world} ranks")
    per = seq_len // world
    return range(rank * per, (rank + 1) * per)


_LAYOUTS = {"contiguous": 0, "zigzag": 1}


def token_ranges(seq_len: int, world: int, rank: int, layout: str = "contiguous") -> List[range]:
    """Global token positions held by ``rank``, in local row order: one range
    (contiguous) or chunks ``rank`` and ``2*world-1-rank`` of ``seq_len/(2*world)``
    tokens (zig-zag; each chunk a multiple of 256 tokens)."""
    if layout == "contiguous":
        return [token_range(seq_len, world, rank)]
    if layout != "zigzag":
        raise ValueError(f"unknown layout {layout!r}")
    if seq_len % (512 * world):
        raise ValueError(f"zig-zag sharding needs seq_len a multiple of {512 * world} for {world} ranks")
    h = seq_len // (2 * world)
    return [range(rank * h, (rank + 1) * h), range((2 * world - 1 - rank) * h, (2 * world - rank) * h)]


def take_tokens(x: torch.Tensor, ranges: Sequence[range]) -> torch.Tensor:
    """The rows of ``x`` ([B, S, ...]) at ``ranges``, in order, contiguous."""
    return torch.cat([x[:, r.start:r.stop] for r in ranges], dim=1).contiguous()


def causal_work(ranges: Sequence[range]) -> int:
    """Causal attention work of a rank's queries: sum over them of (position + 1)."""
    return sum((r.start + r.stop + 1) * len(r) // 2 for r in ranges)


class SeqShardComm:
    """libtj's NCCL communicator for the ranks of a torch.distributed group."""

    def __init__(self, device: torch.device, timeout_ms: int = 120_000) -> None:
        if not dist.is_initialized():
            raise RuntimeError("SeqShardComm needs an initialised torch.distributed process group")
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.device = device
        uid = torch.zeros(128, dtype=torch.uint8)
        if self.rank == 0:
            buf = (ctypes.c_uint8 * 128)()
            _lib.call("tj_nccl_unique_id", buf)
            uid = torch.tensor(list(buf), dtype=torch.uint8)
        uid = uid.to(device) if dist.get_backend() == "nccl" else uid
        dist.broadcast(uid, src=0)
        raw = (ctypes.c_uint8 * 128)(*uid.cpu().tolist())
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.call("tj_comm_create", raw, self.rank, self.world, timeout_ms, ctypes.byref(ptr))
        self.ptr = ptr
        self._ws = {}

    def close(self) -> None:
        if self.ptr:
            _lib.load().tj_comm_destroy(self.ptr)
            self.ptr = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def forward_seqshard(model: B200Transformer, comm: SeqShardComm, x_local: torch.Tensor,
                     route: str = "auto", layout: str = "contiguous") -> torch.Tensor:
    """Rank ``comm.rank``'s shard of the forward: ``x_local`` holds its tokens
    of every sample (``token_ranges(S, P, rank, layout)``; [B, S/P, d] FP32,
    causal, no padding); returns the matching output rows.  The zig-zag
    layout takes the exact route only."""
    if layout not in _LAYOUTS:
        raise ValueError(f"unknown layout {layout!r}")
    if layout == "zigzag" and route != "exact":
        raise ValueError("the zig-zag layout balances the exact route; pass route='exact'")
    if x_local.device != comm.device or x_local.dtype != torch.float32 or x_local.ndim != 3:
        raise ValueError("x_local must be FP32 [B, S/P, d] on the communicator's device")
    x_local = x_local.contiguous()
    batch, s_loc, _ = x_local.shape
    handle = model._ensure_packed(x_local.device)
    key = (batch, s_loc, route)
    ws = comm._ws.get(key)
    if ws is None:
        nbytes = ctypes.c_size_t()
        _lib.call("tj_workspace_bytes_seqshard", handle.ptr, comm.ptr, batch, s_loc, _ROUTES[route],
                  ctypes.byref(nbytes))
        ws = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=x_local.device)
        comm._ws = {key: ws}
    out = torch.empty_like(x_local)
    stream = torch.cuda.current_stream(x_local.device)
    with torch.cuda.device(x_local.device):
        _lib.call("tj_forward_seqshard", handle.ptr, comm.ptr, x_local.data_ptr(), out.data_ptr(), batch, s_loc,
                  _ROUTES[route], _LAYOUTS[layout], ws.data_ptr(), ws.numel(),
                  ctypes.c_void_p(stream.cuda_stream))
    return out


def seqshard_routes(model: B200Transformer) -> List[int]:
    """Each layer's cached sequence-sharded route: 1 polynomial, 0 exact, -1 not evaluated yet."""
    handle = model._handle
    if handle is None:
        return [-1] * model.config.num_layers
    out = []
    for layer in range(model.config.num_layers):
        r = ctypes.c_int()
        _lib.call("tj_seqshard_route", handle.ptr, layer, ctypes.byref(r))
        out.append(int(r.value))
    return out
