"""Kernel-level building blocks over torch CUDA tensors (thin ctypes wrappers).

Each function checks shapes/dtypes/devices, allocates its outputs with torch
and calls the matching ``libtj.so`` entry point on the current stream.  These
are the same kernels ``tj_forward`` chains; they are exposed for tests,
profiling and callers composing their own pipelines.
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple, Optional

import torch

from . import _lib


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and (t.device.type != "cuda" or not t.is_contiguous()):
            raise ValueError("techjam_b200.ops needs contiguous CUDA tensors")


class MaskInfo(NamedTuple):
    lengths: torch.Tensor     # int32 [B]
    general: torch.Tensor     # uint8 [B]
    tile_list: torch.Tensor   # int32 [n_tiles]
    n_live: torch.Tensor      # int32 [1]
    tile_live: torch.Tensor   # uint8 [n_tiles]
    mask: Optional[torch.Tensor]
    batch: int
    seq_len: int


def prepare_mask(mask: Optional[torch.Tensor], batch: int, seq_len: int, device=None) -> MaskInfo:
    """Per-sample valid lengths, non-prefix flags and the live 128-row tile list."""
    if mask is not None:
        _need_cuda(mask)
        if mask.dtype != torch.bool or mask.shape != (batch, seq_len):
            raise ValueError("mask must be bool [B, N]")
        device = mask.device
    device = torch.device(device or "cuda")
    n_tiles = (batch * seq_len + 127) // 128
    lengths = torch.empty(batch, dtype=torch.int32, device=device)
    general = torch.empty(batch, dtype=torch.uint8, device=device)
    tile_list = torch.zeros(max(n_tiles, 1), dtype=torch.int32, device=device)
    n_live = torch.zeros(1, dtype=torch.int32, device=device)
    tile_live = torch.zeros(max(n_tiles, 1), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        _lib.call("tj_prepare_mask", _ptr(mask), batch, seq_len, lengths.data_ptr(), general.data_ptr(),
                  tile_list.data_ptr(), n_live.data_ptr(), tile_live.data_ptr(), _stream(lengths))
    return MaskInfo(lengths, general, tile_list, n_live, tile_live, mask, batch, seq_len)


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, info: MaskInfo, eps: float = 1e-5,
              out_fp16: bool = True) -> torch.Tensor:
    """LayerNorm of x [B*N, d] (fp32); invalid rows are written as zeros."""
    _need_cuda(x, weight, bias)
    rows, d = x.shape
    if rows != info.batch * info.seq_len:
        raise ValueError("x rows must equal B*N")
    out = torch.zeros(rows, d, dtype=torch.float16 if out_fp16 else torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("tj_layernorm", x.data_ptr(), weight.data_ptr(), bias.data_ptr(), info.batch, info.seq_len, d,
                  float(eps), out.data_ptr(), int(out_fp16), info.lengths.data_ptr(), _ptr(info.mask),
                  info.tile_live.data_ptr(), _stream(x))
    return out


def gemm(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, info: MaskInfo, epilogue: int,
         resid: Optional[torch.Tensor] = None, heads: int = 0, err: Optional[torch.Tensor] = None):
    """tcgen05 GEMM ``a @ w.T + bias`` (fp16 operands, fp32 accumulate) with a fused epilogue.

    Returns fp16 [M, N] (GELU/plain), fp32 [M, N] (residual) or a (q, k, v)
    tuple of fp16 [B, H, N, hd] (QKV scatter).
    """
    _need_cuda(a, w, bias, resid)
    if a.dtype != torch.float16 or w.dtype != torch.float16 or bias.dtype != torch.float32:
        raise ValueError("a, w must be fp16 and bias fp32")
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or bias.shape != (n,) or m != info.batch * info.seq_len:
        raise ValueError("shape mismatch")
    err = err if err is not None else torch.zeros(1, dtype=torch.int32, device=a.device)
    out = q = kk = v = None
    if epilogue == _lib.EPI_QKV:
        d = n // 3
        hd = d // heads
        q, kk, v = (torch.zeros(info.batch, heads, info.seq_len, hd, dtype=torch.float16, device=a.device)
                    for _ in range(3))
    elif epilogue == _lib.EPI_RESID:
        out = torch.empty(m, n, dtype=torch.float32, device=a.device)
        if resid is None:
            raise ValueError("residual epilogue needs resid")
    else:
        out = torch.empty(m, n, dtype=torch.float16, device=a.device)
    with torch.cuda.device(a.device):
        _lib.call("tj_gemm_f16", a.data_ptr(), w.data_ptr(), bias.data_ptr(), info.batch, info.seq_len, n, k,
                  epilogue, _ptr(out), _ptr(resid), _ptr(q), _ptr(kk), _ptr(v), heads, info.tile_list.data_ptr(),
                  info.n_live.data_ptr(), info.lengths.data_ptr(), _ptr(info.mask), err.data_ptr(), _stream(a))
    return (q, kk, v) if epilogue == _lib.EPI_QKV else out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, info: MaskInfo, causal: bool,
              err: Optional[torch.Tensor] = None, sched: Optional[torch.Tensor] = None,
              dynamic: bool = True) -> torch.Tensor:
    """Flash attention over fp16 [B, H, N, hd]; returns the fp16 context [B*N, H*hd].

    ``sched``: two zeroed int32 words for the dynamic work scheduler (made
    here when not given); ``dynamic=False`` uses the static item assignment.
    """
    _need_cuda(q, k, v)
    b, h, n, hd = q.shape
    if q.dtype != torch.float16 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must be fp16 [B, H, N, hd]")
    err = err if err is not None else torch.zeros(1, dtype=torch.int32, device=q.device)
    if dynamic and sched is None:
        sched = torch.zeros(2, dtype=torch.int32, device=q.device)
    ctx = torch.zeros(b * n, h * hd, dtype=torch.float16, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("tj_attention_f16", q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx.data_ptr(), b, h, n, hd,
                  int(causal), info.lengths.data_ptr(), _ptr(info.mask), info.general.data_ptr(), err.data_ptr(),
                  _ptr(sched) if dynamic else None, _stream(q))
    return ctx


class PolyStatus(NamedTuple):
    admit: bool
    c0: float
    c1: float
    c2: float
    sigma: float
    max_abs: float


def poly_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_prefix: int = 4096,
                   err: Optional[torch.Tensor] = None):
    """Guarded polynomial causal attention (head_dim 64, no padding).

    Returns (ctx fp16 [B*N, H*64], PolyStatus).  Queries below ``exact_prefix``
    -- or all of them if the device-side guard rejects the route -- come from
    the exact flash kernel.
    """
    _need_cuda(q, k, v)
    b, h, n, hd = q.shape
    if hd != 64 or q.dtype != torch.float16 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must be fp16 [B, H, N, 64]")
    nbytes = ctypes.c_size_t()
    _lib.call("tj_poly_workspace_bytes", b, h, n, exact_prefix, ctypes.byref(nbytes))
    ws = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=q.device)
    err = err if err is not None else torch.zeros(1, dtype=torch.int32, device=q.device)
    lengths = torch.full((b,), n, dtype=torch.int32, device=q.device)
    ctx = torch.zeros(b * n, h * hd, dtype=torch.float16, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("tj_poly_attention_f16", q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx.data_ptr(),
                  lengths.data_ptr(), b, h, n, exact_prefix, ws.data_ptr(), ws.numel(), err.data_ptr(), _stream(q))
    head = ws[:24].cpu()
    admit = int(head[:4].view(torch.int32).item())
    c0, c1, c2, sigma, max_abs = (float(v) for v in head[4:24].view(torch.float32))
    return ctx, PolyStatus(bool(admit), c0, c1, c2, sigma, max_abs)
