"""Paged latent-history kernel (hla_s6_history_attention) vs the reference fixtures and the oracle.

Tolerances: bf16 outputs within 2e-2 max-abs / 1e-2 relative, LSE within
1e-3; empty rows exactly o = 0, lse = -inf.  Cases follow the reference's GPU op test
(test_s6_ops_gpu.py:43-57: widths, blocks, splits, batches 1/8/33, ctx {5000, 1000, 17, 1, 0})
and its CPU fixtures (poisoned null block, stale table columns, NaN-filled caches).
"""
import math

import numpy as np
import pytest
import torch

import cases
from conftest import GOLDEN, pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu
CUDA, BF16, I32 = 'cuda', torch.bfloat16, torch.int32
SCALE = 1 / math.sqrt(128)
O_TOL = dict(atol=2e-2, rtol=1e-2)
LSE_ATOL = 1e-3


def ops():
    return pkg('s6_ops')


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


def check(o, lse, o_ref, lse_ref, ctx):
    T, H, W = o.shape
    assert o.dtype == BF16 and lse.dtype == torch.float32 and lse.shape == (H, T) and lse.is_contiguous()
    o, lse = o.float().cpu().numpy(), lse.cpu().numpy()
    assert np.isfinite(o).all() and not np.isnan(lse).any()
    empty = np.asarray(ctx) <= 0
    assert (o[empty] == 0).all() and (lse[:, empty] == -np.inf).all()
    np.testing.assert_allclose(o, o_ref, **O_TOL)
    np.testing.assert_allclose(lse[:, ~empty], lse_ref[:, ~empty], atol=LSE_ATOL, rtol=0)


def run(q, cache, table, ctx, splits, scale=SCALE, empty=None):
    T, H, W = q.shape
    ws = ops().S6Workspace(H, W, max(T, 1) * splits)
    return ops().history_attention(q, cache, table, ctx, scale, splits, ws, None, None, 'b200', empty=empty)


@pytest.mark.parametrize('name', ['hist_h16_w512_p16', 'hist_h16_w256_p16', 'hist_h16_w512_p32'])
@pytest.mark.parametrize('splits', [1, 4, 16])
def test_history_matches_reference_fixture(name, splits):
    inp, scale = cases.history_cases()[name]
    g = np.load(GOLDEN / f'{name}.npz')
    assert str(g['input_sha256']) == cases.digest(inp)
    o, lse = run(dev(inp['q'], BF16), dev(inp['cache'], BF16), dev(inp['block_table']), dev(inp['ctx']), splits,
                 scale=float(scale))
    check(o, lse, g['o'], g['lse'], inp['ctx'])


def random_case(seed, width, block, batch, ctx_values, num_blocks=1024, heads=16, nan_tail=False):
    rng = np.random.default_rng(seed)
    ctx = np.array((list(ctx_values) * 64)[:batch], dtype=np.int32)
    maxb = -(-max(int(ctx.max()), 1) // block)
    cache = orc.bf16(rng.standard_normal((num_blocks, 1, block, 2 * width), dtype=np.float32))
    table = rng.integers(0, num_blocks, (batch, maxb + 1)).astype(np.int32)
    q = orc.bf16(rng.standard_normal((batch, heads, width), dtype=np.float32))
    return q, cache, table, ctx


@pytest.mark.parametrize('width', [512, 256])
@pytest.mark.parametrize('block', [16, 32])
@pytest.mark.parametrize('splits', [1, 4, 16])
def test_history_matches_oracle_reference_grid(width, block, splits):
    for batch in (1, 8, 33):
        q, cache, table, ctx = random_case(batch * 7 + width + block, width, block, batch, [5000, 1000, 17, 1, 0])
        o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
        o, lse = run(dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx), splits)
        check(o, lse, o_ref, lse_ref, ctx)


def test_history_width_1024():
    q, cache, table, ctx = random_case(3, 1024, 16, 8, [3000, 17, 0, 1, 700], num_blocks=256)
    o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
    o, lse = run(dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx), 8)
    check(o, lse, o_ref, lse_ref, ctx)


def test_nan_rows_past_ctx_and_poisoned_stale_columns_never_leak():
    """Rows past ctx inside the last page are NaN, stale columns point at a +inf null block."""
    width, block = 512, 16
    q, cache, table, ctx = random_case(5, width, block, 9, [37, 16, 1, 200, 0, 15, 33, 100, 250], num_blocks=64)
    cache[0] = np.inf
    flat = cache.reshape(-1, 2 * width)
    used = set()
    for t, n in enumerate(ctx):
        pages = -(-int(n) // block)
        table[t, pages:] = 0
        for j in range(int(n)):
            used.add(int(table[t, j // block]) * block + j % block)
    for s in range(block, flat.shape[0]):
        if s not in used:
            flat[s] = np.nan
    o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
    for splits in (1, 16):
        o, lse = run(dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx), splits)
        check(o, lse, o_ref, lse_ref, ctx)


def test_empty_mask_and_all_empty_batch():
    q, cache, table, ctx = random_case(9, 512, 16, 5, [40, 0, 9, 300, 2], num_blocks=64)
    empty = torch.tensor([False, True, True, False, False], device=CUDA)
    o, lse = run(dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx), 4, empty=empty)
    o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
    o_ref[2] = 0
    lse_ref[:, 2] = -np.inf
    ctx2 = ctx.copy()
    ctx2[2] = 0
    check(o, lse, o_ref, lse_ref, ctx2)
    zero = np.zeros_like(ctx)
    o, lse = run(dev(q, BF16), dev(cache, BF16), dev(table), dev(zero), 16)
    assert (o == 0).all() and (lse == -np.inf).all()


def test_fewer_query_heads_than_sixteen():
    q, cache, table, ctx = random_case(10, 256, 16, 4, [100, 3, 0, 64], num_blocks=64, heads=6)
    o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
    o, lse = run(dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx), 4)
    check(o, lse, o_ref, lse_ref, ctx)


def test_strided_query_and_kv_variant():
    """einsum-shaped q (head stride T*W) and the k/v-halves entry point."""
    q, cache, table, ctx = random_case(11, 512, 16, 6, [300, 1, 0, 77, 16, 1000], num_blocks=128)
    qt = dev(q, BF16).transpose(0, 1).contiguous().transpose(0, 1)   # [T,H,W] with head stride T*W
    assert qt.stride(1) == q.shape[0] * q.shape[2]
    c = dev(cache, BF16)
    ws = ops().S6Workspace(16, 512, 6 * 16)
    o, lse = ops().history_attention_kv(qt, c[..., :512], c[..., 512:], dev(table), dev(ctx), SCALE, 16, ws, None,
                                        None, 'b200')
    o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
    check(o, lse, o_ref, lse_ref, ctx)


def test_workspace_overflow_raises():
    q, cache, table, ctx = random_case(12, 512, 16, 4, [10], num_blocks=8)
    ws = ops().S6Workspace(16, 512, 4 * 2)
    with pytest.raises(RuntimeError, match='overflow'):
        ops().history_attention(dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx), SCALE, 16, ws, None, None,
                                'b200')


def test_history_replays_inside_cuda_graph():
    """Graph capture with changing ctx / cache / q contents (test_s6_ops_gpu.py:121-151)."""
    torch.manual_seed(1)
    width, block, batch, splits, num_blocks = 512, 16, 8, 16, 256
    ws = ops().S6Workspace(16, width, batch * splits)
    ws.ensure(CUDA)
    cache = torch.randn(num_blocks, 1, block, 2 * width, dtype=BF16, device=CUDA)
    table = torch.randint(0, num_blocks, (batch, 64), dtype=I32, device=CUDA)
    ctx = torch.randint(0, 1000, (batch,), dtype=I32, device=CUDA)
    q = torch.randn(batch, 16, width, dtype=BF16, device=CUDA)

    def go():
        return ops().history_attention(q, cache, table, ctx, SCALE, splits, ws, None, None, 'b200')

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        go()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o, lse = go()
    for _ in range(3):
        ctx.copy_(torch.randint(0, 1000, (batch,), dtype=I32, device=CUDA))
        ctx[0] = 0
        cache.copy_(torch.randn_like(cache))
        q.copy_(torch.randn_like(q))
        graph.replay()
        torch.cuda.synchronize()
        o_ref, lse_ref = orc.history_attention(q.float().cpu().numpy(), cache.float().cpu().numpy(),
                                               table.cpu().numpy(), ctx.cpu().numpy(), SCALE)
        check(o, lse, o_ref, lse_ref, ctx.cpu().numpy())


def test_full_size_decode_call_spot_rows():
    """Config-2 shape (T=64, ctx_latent 8160, shuffled pages): spot rows against the oracle,
    plus a size-independent property: identical rows give identical outputs."""
    T, width, block = 64, 512, 16
    ctx_lat = 8160
    pages = -(-ctx_lat // block)
    nb = T * pages + 1
    g = torch.Generator(device=CUDA).manual_seed(3)
    cache = torch.randn(nb, 1, block, 2 * width, dtype=BF16, device=CUDA, generator=g)
    perm = torch.randperm(nb - 1, device=CUDA, generator=g).to(I32) + 1
    table = perm.view(T, pages)
    table[5] = table[4]                       # rows 4 and 5 read the same pages
    q = torch.randn(T, 16, width, dtype=BF16, device=CUDA, generator=g)
    q[5] = q[4]
    ctx = torch.full((T,), ctx_lat, dtype=I32, device=CUDA)
    splits = ops().num_kv_splits(8192, T, 512, torch.cuda.get_device_properties(0).multi_processor_count)
    o, lse = run(q, cache, table, ctx, splits)
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    # stream-K cuts rows 4 and 5 at different page boundaries (different fp32 summation order)
    torch.testing.assert_close(o[4].float(), o[5].float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(lse[:, 4], lse[:, 5], atol=1e-4, rtol=0)
    o1, lse1 = run(q, cache, table, ctx, 1)   # one CTA per row: identical rows, identical bits
    assert torch.equal(o1[4], o1[5]) and torch.equal(lse1[:, 4], lse1[:, 5])
    torch.testing.assert_close(o1.float(), o.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(lse1, lse, atol=LSE_ATOL, rtol=0)
    rows = [0, 4, 37, 63]
    qc = q[rows].float().cpu().numpy()
    tc = table[rows].cpu().numpy()
    used = np.unique(tc)
    remap = {int(b): i for i, b in enumerate(used)}
    sub = cache[torch.from_numpy(used).to(CUDA).long()].float().cpu().numpy()
    tsub = np.vectorize(remap.get)(tc).astype(np.int32)
    o_ref, lse_ref = orc.history_attention(qc, sub, tsub, np.full(len(rows), ctx_lat), SCALE)
    np.testing.assert_allclose(o[rows].float().cpu().numpy(), o_ref, **O_TOL)
    np.testing.assert_allclose(lse[:, rows].cpu().numpy(), lse_ref, atol=LSE_ATOL, rtol=0)


@pytest.mark.parametrize('splits', [1, 16])
def test_block_id_outside_the_cache_is_reported(splits):
    """A block-table entry at or past num_blocks (or negative) inside a row's pages: the reference's torch
    indexing raises IndexError; the kernel reads that page as zeros - never outside the cache - and sets
    HLA_S6_ERR_BLOCK in the error word.  A valid table leaves the word at 0."""
    lib = pkg('_lib')
    q, cache, table, ctx = random_case(3, 512, 16, 8, [300, 40, 0, 17], num_blocks=64)
    T, H, W = q.shape
    qd, cd, cx = dev(q, BF16), dev(cache, BF16), dev(ctx)
    for bad, expect in ((None, 0), (64, lib.ERR_BLOCK), (-3, lib.ERR_BLOCK)):
        tab = table.copy()
        if bad is not None:
            tab[1, 1] = bad                                 # row 1 (ctx 40) reads pages 0..2
        td = dev(tab)
        err = torch.zeros(1, dtype=I32, device=CUDA)
        ws = torch.empty(T * splits * H * (W + 1), dtype=torch.float32, device=CUDA)
        o = torch.empty(T, H, W, dtype=BF16, device=CUDA)
        lse = torch.empty(H, T, dtype=torch.float32, device=CUDA)
        lib.call('hla_s6_history_attention', lib.ptr(qd), qd.stride(0), qd.stride(1), lib.ptr(cd), cd.shape[0],
                 cd.stride(0), cd.stride(2), lib.ptr(td), td.stride(0), td.shape[1], lib.ptr(cx), None, T, H, W, 16,
                 SCALE, splits, lib.ptr(ws), ws.numel(), lib.ptr(o), o.stride(0), o.stride(1), lib.ptr(lse),
                 lib.ptr(err), lib.stream_of(qd))
        torch.cuda.synchronize()
        assert int(err.item()) == expect
        assert torch.isfinite(o.float()).all()
        if bad is None:
            o_ref, lse_ref = orc.history_attention(q, cache, tab, ctx, SCALE)
            check(o, lse, o_ref, lse_ref, ctx)


@pytest.mark.parametrize('width,block', [(512, 16), (256, 32), (512, 32)])
def test_tail_stealing_split_matches_oracle_and_repeats_bit_exactly(width, block):
    """A step with about as many rows as the split kernel has CTAs (160 rows, empty ones among them, over
    16 pages per CTA) runs the tail-stealing kernel: the last eighth of each CTA's pages is taken by
    whichever CTA is free first.  Partial slots belong to units, not to CTAs, so three calls in a row on
    the same workspace give bit-identical outputs (the pool's counters are re-zeroed by each launch's
    last CTA), equal to the oracle within the output tolerances."""
    q, cache, table, ctx = random_case(11 + width + block, width, block, 160, [3000, 700, 40, 5, 0])
    o_ref, lse_ref = orc.history_attention(q, cache, table, ctx, SCALE)
    qd, cd, td, xd = dev(q, BF16), dev(cache, BF16), dev(table), dev(ctx)
    outs = [run(qd, cd, td, xd, 64) for _ in range(3)]
    for o, lse in outs:
        check(o, lse, o_ref, lse_ref, ctx)
        assert torch.equal(o, outs[0][0]) and torch.equal(lse, outs[0][1])
