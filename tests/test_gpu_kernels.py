"""Kernel-level parity on the GPU: each libtj building block vs a plain PyTorch
FP32 evaluation of the same operation on the same (seeded) inputs."""

import math

import pytest
import torch
import torch.nn.functional as F

from techjam_b200 import _lib, ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _right_padded(b, n, lo, gen):
    lengths = torch.randint(lo, n + 1, (b,), generator=gen)
    return torch.arange(n)[None, :] < lengths[:, None]


def test_prepare_mask_lengths_and_tiles():
    gen = torch.Generator().manual_seed(0)
    for b, n in ((3, 200), (4, 512), (2, 1000)):
        mask = _right_padded(b, n, 1, gen)
        mask[0] = False  # an empty sample
        general = mask.clone()
        general[-1, 0] = False  # a hole -> not a prefix
        for m in (mask, general, None):
            info = ops.prepare_mask(None if m is None else m.to(DEV), b, n, DEV)
            mm = torch.ones(b, n, dtype=torch.bool) if m is None else m
            pos = torch.arange(1, n + 1)[None, :]
            exp_len = (mm.long() * pos).amax(1)
            assert torch.equal(info.lengths.cpu().long(), exp_len)
            exp_gen = (mm.sum(1) != exp_len).to(torch.uint8)
            assert torch.equal(info.general.cpu(), exp_gen)
            rows = torch.arange(b * n)
            valid_row = (rows % n) < exp_len[rows // n]
            n_tiles = (b * n + 127) // 128
            exp_live = torch.zeros(n_tiles, dtype=torch.bool)
            exp_live.index_put_((rows[valid_row] // 128,), torch.tensor(True))
            assert torch.equal(info.tile_live.cpu()[:n_tiles].bool(), exp_live)
            nl = int(info.n_live.item())
            assert nl == int(exp_live.sum())
            assert torch.equal(info.tile_list.cpu()[:nl], torch.nonzero(exp_live).flatten().int())


@pytest.mark.parametrize("d", [256, 768, 1024])
def test_layernorm_matches_torch(d):
    gen = torch.Generator().manual_seed(d)
    b, n = 3, 333
    x = torch.randn(b * n, d, generator=gen) * 2 + 0.5
    w = torch.randn(d, generator=gen)
    bb = torch.randn(d, generator=gen)
    mask = _right_padded(b, n, 100, gen)
    info = ops.prepare_mask(mask.to(DEV), b, n)
    ref = F.layer_norm(x, (d,), w, bb, 1e-5)
    valid = mask.reshape(-1)
    for fp16 in (True, False):
        got = ops.layernorm(x.to(DEV), w.to(DEV), bb.to(DEV), info, 1e-5, out_fp16=fp16).float().cpu()
        tol = 4e-3 if fp16 else 2e-5
        torch.testing.assert_close(got[valid], ref[valid], atol=tol, rtol=tol)
        live = info.tile_live.cpu().bool()
        rows = torch.arange(b * n)
        zero_rows = (~valid) & (live[rows // 128] if fp16 else torch.ones_like(valid))
        assert torch.all(got[zero_rows] == 0)


def _gemm_case(b, n, k, nout, seed, lo=1):
    gen = torch.Generator().manual_seed(seed)
    a = (torch.randn(b * n, k, generator=gen)).half()
    w = (torch.randn(nout, k, generator=gen) / math.sqrt(k)).half()
    bias = torch.randn(nout, generator=gen) * 0.1
    mask = _right_padded(b, n, lo, gen)
    ref = a.float() @ w.float().t() + bias
    return a, w, bias, mask, ref


@pytest.mark.parametrize("b,n,k,nout", [(3, 200, 256, 512), (2, 512, 1024, 1024), (16, 1024, 1024, 4096),
                                         (4, 256, 2048, 512), (3, 1000, 512, 4096), (5, 700, 1024, 3072)])
def test_gemm_gelu_and_plain(b, n, k, nout):
    """Small shapes take the 1-CTA kernel; the large ones the 2-SM pair kernel
    (ragged lengths give odd live-tile counts: the pair's ghost half)."""
    a, w, bias, mask, ref = _gemm_case(b, n, k, nout, seed=b * 7 + n)
    info = ops.prepare_mask(mask.to(DEV), b, n)
    valid = mask.reshape(-1)
    for epi, fn in ((_lib.EPI_PLAIN16, lambda t: t), (_lib.EPI_GELU, lambda t: F.gelu(t, approximate="none"))):
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        got = ops.gemm(a.to(DEV), w.to(DEV), bias.to(DEV), info, epi, err=err).float().cpu()
        assert int(err.item()) == 0
        torch.testing.assert_close(got[valid], fn(ref)[valid], atol=3e-3, rtol=3e-3)
        live = info.tile_live.cpu().bool()
        rows = torch.arange(b * n)
        assert torch.all(got[(~valid) & live[rows // 128]] == 0)


@pytest.mark.parametrize("b,n,k,nout", [(3, 200, 256, 256), (16, 1024, 4096, 1024), (2, 2048, 1024, 1024)])
def test_gemm_residual(b, n, k, nout):
    a, w, bias, mask, ref = _gemm_case(b, n, k, nout, seed=11 + n)
    resid = torch.randn(b * n, nout)
    info = ops.prepare_mask(mask.to(DEV), b, n)
    got = ops.gemm(a.to(DEV), w.to(DEV), bias.to(DEV), info, _lib.EPI_RESID, resid=resid.to(DEV)).cpu()
    valid = mask.reshape(-1)
    torch.testing.assert_close(got[valid], (ref + resid)[valid], atol=1e-3, rtol=1e-4)
    live = info.tile_live.cpu().bool()
    rows = torch.arange(b * n)
    assert torch.all(got[(~valid) & live[rows // 128]] == 0)


@pytest.mark.parametrize("b,n,d,heads", [(3, 200, 256, 8), (2, 512, 1024, 16), (4, 256, 512, 8), (2, 256, 512, 4)])
def test_gemm_qkv_scatter(b, n, d, heads):
    a, w, bias, mask, ref = _gemm_case(b, n, d, 3 * d, seed=3 + d)
    info = ops.prepare_mask(mask.to(DEV), b, n)
    q, k, v = ops.gemm(a.to(DEV), w.to(DEV), bias.to(DEV), info, _lib.EPI_QKV, heads=heads)
    hd = d // heads
    valid = mask
    for i, t in enumerate((q, k, v)):
        exp = ref[:, i * d:(i + 1) * d].reshape(b, n, heads, hd).transpose(1, 2)
        got = t.float().cpu()
        vm = valid[:, None, :, None].expand_as(exp)
        torch.testing.assert_close(got[vm], exp[vm], atol=3e-3, rtol=3e-3)


def _attn_ref(q, k, v, mask, causal):
    """Plain fp32 softmax attention (masked keys -inf, invalid query rows ignored)."""
    b, h, n, hd = q.shape
    s = (q.float() @ k.float().transpose(-1, -2)) * hd ** -0.5
    if causal:
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return (p @ v.float()).transpose(1, 2).reshape(b * n, h * hd)


@pytest.mark.parametrize("b,h,n,hd,causal,kind", [
    (2, 4, 384, 64, True, "prefix"), (2, 2, 300, 32, True, "prefix"), (1, 2, 256, 128, True, "prefix"),
    (2, 4, 384, 64, False, "prefix"), (2, 3, 250, 64, True, "general"), (2, 2, 200, 64, False, "general"),
    (1, 16, 2048, 64, True, "none"), (3, 2, 1000, 128, False, "prefix"),
    # more than two query-tile pairs at head_dim 64: the per-pair (column-split) kernel
    (2, 4, 700, 64, True, "prefix"), (2, 3, 640, 64, True, "general"), (2, 2, 600, 64, False, "general"),
    (2, 2, 777, 64, False, "prefix"), (3, 2, 1100, 64, True, "none"),
])
def test_attention_matches_fp32(b, h, n, hd, causal, kind):
    gen = torch.Generator().manual_seed(b * 100 + n + hd)
    q, k, v = (torch.randn(b, h, n, hd, generator=gen).half() for _ in range(3))
    if kind == "none":
        mask = torch.ones(b, n, dtype=torch.bool)
    elif kind == "prefix":
        mask = _right_padded(b, n, n // 3, gen)
    else:
        mask = torch.rand(b, n, generator=gen) > 0.3
        mask[:, 0] = True
    info = ops.prepare_mask(None if kind == "none" else mask.to(DEV), b, n)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), info, causal, err=err).float().cpu()
    assert int(err.item()) == 0
    ref = _attn_ref(q, k, v, mask, causal)
    rows_ok = mask.reshape(-1)
    torch.testing.assert_close(got[rows_ok], ref[rows_ok], atol=4e-3, rtol=1e-2)


@pytest.mark.parametrize("b,h,n,hd,causal", [(4, 8, 2048, 64, True), (16, 4, 256, 64, True), (3, 4, 1500, 32, True),
                                             (2, 4, 1100, 64, False)])
def test_attention_scheduler_static_equals_dynamic(b, h, n, hd, causal):
    """The persistent kernel's work items are independent: claiming them
    through the atomic scheduler or by static round-robin gives bit-identical
    contexts, and the scheduler words are zero again after every launch."""
    gen = torch.Generator().manual_seed(b * 31 + n)
    q, k, v = (torch.randn(b, h, n, hd, generator=gen).half().to(DEV) for _ in range(3))
    mask = _right_padded(b, n, n // 2, gen)
    info = ops.prepare_mask(mask.to(DEV), b, n)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    sched = torch.zeros(2, dtype=torch.int32, device=DEV)
    dyn = [ops.attention(q, k, v, info, causal, err=err, sched=sched) for _ in range(3)]
    torch.cuda.synchronize()
    assert sched.tolist() == [0, 0]
    static = ops.attention(q, k, v, info, causal, err=err, dynamic=False)
    assert int(err.item()) == 0
    for d in dyn:
        assert torch.equal(d, static)
    ref = _attn_ref(q.cpu(), k.cpu(), v.cpu(), mask, causal)
    rows_ok = mask.reshape(-1)
    torch.testing.assert_close(static.float().cpu()[rows_ok], ref[rows_ok], atol=4e-3, rtol=1e-2)


@pytest.mark.parametrize("hd", [32, 64, 128])
@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("layout", ["contiguous", "zigzag"])
def test_sharded_attention_layouts_on_one_gpu(hd, world, layout):
    """The sequence-sharded attention (local queries at their global positions
    over every shard's K/V, as the multi-GPU forward runs it after its K/V
    all-gather), emulated rank by rank on one GPU: each shard's context rows
    equal the unsharded causal attention's rows bit for bit, for both token
    layouts and every head_dim (persistent kernel for <= 64, per-pair for 128)."""
    from techjam_b200.sharding import token_ranges
    b, h, s = 2, 2, world * 512
    gen = torch.Generator(device=DEV).manual_seed(hd * 10 + world)
    q, k, v = (torch.randn(b, h, s, hd, device=DEV, generator=gen).half() for _ in range(3))
    full_info = ops.prepare_mask(None, b, s, DEV)
    ref = ops.attention(q, k, v, full_info, causal=True)  # [b*s, h*hd]
    lengths = torch.full((b,), s, dtype=torch.int32, device=DEV)
    general = torch.zeros(b, dtype=torch.uint8, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    sched = torch.zeros(2, dtype=torch.int32, device=DEV)
    parts = [token_ranges(s, world, r, layout) for r in range(world)]
    rows = [torch.cat([torch.arange(rg.start, rg.stop) for rg in rs]).to(DEV) for rs in parts]
    k_all = torch.stack([k[:, :, idx] for idx in rows]).contiguous()
    v_all = torch.stack([v[:, :, idx] for idx in rows]).contiguous()
    s_loc = s // world
    for r in range(world):
        q_loc = q[:, :, rows[r]].contiguous()
        ctx = torch.zeros(b * s_loc, h * hd, dtype=torch.float16, device=DEV)
        _lib.call("tj_attention_shard_f16", q_loc.data_ptr(), k_all.data_ptr(), v_all.data_ptr(), ctx.data_ptr(),
                  b, h, s_loc, hd, lengths.data_ptr(), general.data_ptr(), err.data_ptr(), sched.data_ptr(), r, world,
                  1 if layout == "zigzag" else 0, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        want = ref.view(b, s, h * hd)[:, rows[r]].reshape(b * s_loc, h * hd)
        assert torch.equal(ctx, want), f"rank {r}: max diff {(ctx.float() - want.float()).abs().max().item()}"
