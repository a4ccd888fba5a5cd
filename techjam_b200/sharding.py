"""Multi-GPU execution: one process per GPU (torchrun), NCCL over NVLink.

Two ways the encoder forward shards (the reference has neither; it streams
batch and prefix chunks through one GPU, src/implementations/extreme.py:136-204):

* **Batch sharding** (independent samples): ``shard_samples`` assigns whole
  samples to ranks by a longest-processing-time rule on their algorithmic cost
  (ragged lengths make a contiguous split unbalanced); each rank then runs an
  ordinary forward on its samples.  No data-path collective.
* **Sequence sharding** (one long sequence per sample): ``SeqShardComm`` joins
  libtj's own NCCL communicator (the unique id travels over the existing
  torch.distributed group) and ``forward_seqshard`` runs rank r's token range
  ``[r*S/P, (r+1)*S/P)``; libtj exchanges the polynomial prefix state (or the
  K/V shards on the exact route) with NCCL on the compute stream.
"""

from __future__ import annotations

import ctypes
from typing import List, Sequence

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


def token_range(seq_len: int, world: int, rank: int) -> range:
    """Global token positions held by ``rank`` under sequence sharding."""
    if seq_len % world:
        raise ValueError(f"seq_len {seq_len} not divisible by {world} ranks")
    per = seq_len // world
    return range(rank * per, (rank + 1) * per)


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
                     route: str = "auto") -> torch.Tensor:
    """Rank ``comm.rank``'s shard of the forward: ``x_local`` holds its token
    range of every sample ([B, S/P, d] FP32, causal, no padding); returns the
    matching output rows."""
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
                  _ROUTES[route], ws.data_ptr(), ws.numel(), ctypes.c_void_p(stream.cuda_stream))
    return out
