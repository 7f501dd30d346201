"""Per-head paged history read MLA-style - the LLA serving path (reference s6_ops.py:128-161 with mla=True,
as lla_layer.attend calls it at lla_layer.py:67-74) - on the B200 per-head reader, against the reference's
own outputs (golden fixtures, poisoned stale blocks and rows past ctx) and the oracle.  GPU."""
import math

import numpy as np
import pytest
import torch

import cases
from conftest import GOLDEN, pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu
CUDA, BF16 = 'cuda', torch.bfloat16
O_TOL = dict(atol=2e-2, rtol=1e-2)
LSE_ATOL = 1e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


def run(q, cache, r, table, ctx, scale, splits, empty=None):
    ops = pkg('s6_ops')
    T, H = q.shape[:2]
    ws = ops.S6Workspace(H, r, T * splits)
    return ops.history_attention_kv(q, cache, cache[..., :r], table, ctx, scale, splits, ws, None, None, 'b200',
                                    empty, mla=True)


@pytest.mark.parametrize('name,kw', [('heads_lla', dict()),
                                     ('heads_gqa', dict(seed=102, kv_heads=4, rank=64, d_rope=32, ctx=(40, 0, 16, 333)))])
@pytest.mark.parametrize('splits', [1, 4])
def test_matches_reference_fixture(name, kw, splits):
    hc = cases.heads_case(**kw)
    g = np.load(GOLDEN / f'{name}.npz')
    assert str(g['input_sha256']) == cases.digest(hc)
    r = int(hc['rank'])
    o, lse = run(dev(hc['q'], BF16), dev(hc['cache'], BF16), r, dev(hc['block_table']), dev(hc['ctx']),
                 float(g['scale']), splits)
    o, lse = o.float().cpu().numpy(), lse.cpu().numpy()
    assert np.isfinite(o).all()
    np.testing.assert_allclose(o, g['o'], **O_TOL)
    np.testing.assert_allclose(lse, g['lse'], atol=LSE_ATOL, rtol=0)
    empty = hc['ctx'] == 0
    assert (o[empty] == 0).all() and (lse[:, empty] == -np.inf).all()


@pytest.mark.parametrize('rank,d_rope,kvh,ctx', [(512, 64, 16, [8191, 1, 4000, 16, 17, 0, 2500, 8192]),
                                                 (256, 32, 16, [3000] * 12), (64, 32, 2, [100, 7, 1000]),
                                                 # key width 80, not a multiple of 32: 16-column slabs, 32-byte swizzle
                                                 (64, 16, 16, [300, 0, 17, 5000, 33])])
def test_matches_oracle(rank, d_rope, kvh, ctx):
    rng = np.random.default_rng(rank + len(ctx))
    T, H, page, Lk = len(ctx), 16, 16, rank + d_rope
    need = [-(-max(c, 1) // page) for c in ctx]
    nb = sum(need) + 1
    cache = orc.bf16(rng.standard_normal((nb, kvh, page, Lk), dtype=np.float32))
    table = np.zeros((T, max(need)), dtype=np.int32)
    perm = rng.permutation(np.arange(1, nb))
    k = 0
    for t in range(T):
        table[t, :need[t]] = perm[k:k + need[t]]
        k += need[t]
    q = orc.bf16(rng.standard_normal((T, H, Lk), dtype=np.float32))
    scale = 1 / math.sqrt(128)
    ctx = np.asarray(ctx, dtype=np.int32)
    props = torch.cuda.get_device_properties(0)
    splits = pkg('s6_ops').num_kv_splits(int(ctx.max()), T, 512, props.multi_processor_count)
    o, lse = run(dev(q, BF16), dev(cache, BF16), rank, dev(table), dev(ctx), scale, splits)
    o_ref, lse_ref = orc.history_attention_kv(q, cache, cache[..., :rank], table, ctx, scale)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, **O_TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=LSE_ATOL, rtol=0)


def test_layout_contract():
    ops = pkg('s6_ops')
    cache = torch.zeros(4, 16, 16, 160, dtype=BF16, device=CUDA)
    other = torch.zeros(4, 16, 16, 128, dtype=BF16, device=CUDA)
    q = torch.zeros(2, 16, 160, dtype=BF16, device=CUDA)
    table = torch.zeros(2, 2, dtype=torch.int32, device=CUDA)
    ctx = torch.ones(2, dtype=torch.int32, device=CUDA)
    ws = ops.S6Workspace(16, 128, 8)
    with pytest.raises(ValueError, match='MLA row layout'):     # v not a prefix of k's rows
        ops.history_attention_kv(q, cache, other, table, ctx, 0.1, 4, ws, None, None, 'b200', mla=True)
    with pytest.raises(RuntimeError, match='overflow'):
        ops.history_attention_kv(q, cache, cache[..., :128], table, ctx, 0.1, 64, ws, None, None, 'b200', mla=True)


def test_replays_inside_cuda_graph():
    """Per-head MLA read captured in a CUDA graph, replayed with changing ctx / cache / q contents (the case of the
    reference's test_s6_ops_gpu.py:78-110): the stream-K plan and slot ranges follow the new lengths on the device."""
    torch.manual_seed(6)
    ops = pkg('s6_ops')
    rank, d_rope, block, batch, splits, num_blocks = 512, 64, 16, 8, 8, 256
    ws = ops.S6Workspace(16, rank, batch * splits)
    ws.ensure(CUDA)
    cache = torch.randn(num_blocks, 16, block, rank + d_rope, dtype=BF16, device=CUDA)
    table = torch.randint(0, num_blocks, (batch, 64), dtype=torch.int32, device=CUDA)
    ctx = torch.randint(0, 1000, (batch,), dtype=torch.int32, device=CUDA)
    q = torch.randn(batch, 16, rank + d_rope, dtype=BF16, device=CUDA)
    scale = 1 / math.sqrt(128)

    def go():
        return ops.history_attention_kv(q, cache, cache[..., :rank], table, ctx, scale, splits, ws, None, None, 'b200',
                                        mla=True)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        go()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o, lse = go()
    for _ in range(3):
        ctx.copy_(torch.randint(0, 1000, (batch,), dtype=torch.int32, device=CUDA))
        ctx[0] = 0
        cache.copy_(torch.randn_like(cache))
        q.copy_(torch.randn_like(q))
        graph.replay()
        torch.cuda.synchronize()
        c = cache.float().cpu().numpy()
        o_ref, lse_ref = orc.history_attention_kv(q.float().cpu().numpy(), c, c[..., :rank], table.cpu().numpy(),
                                                  ctx.cpu().numpy(), scale)
        o_np, lse_np = o.float().cpu().numpy(), lse.cpu().numpy()
        np.testing.assert_allclose(o_np, o_ref, **O_TOL)
        keep = ctx.cpu().numpy() > 0
        np.testing.assert_allclose(lse_np[:, keep], lse_ref[:, keep], atol=LSE_ATOL, rtol=0)
        assert (o_np[0] == 0).all() and (lse_np[:, 0] == -np.inf).all()
