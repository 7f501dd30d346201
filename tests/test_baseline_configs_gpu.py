"""BASELINE configs 3 and 4 at their own sizes, against the oracle (GPU).

Config 3 - the latent writer of a prompt step: 8 prompts x 4096 tokens, hidden 2048, one layer's four
loops through PrefillWriter (the tcgen05 writer).  Every token's main and loop-1 row must sit exactly at
its vLLM slot and nothing else may be written (bit-exact placement, checked on the device over all
32768 tokens); sampled rows must equal the oracle's writer (register.py:45-79: GEMM, bf16 register add,
latent RoPE of the committed K half) within the bf16 GEMM tolerance.

Config 4 - one decode step (one layer, all four loops) of the 256-request mixed batch, contexts
log-uniform in [64, 32768] with 8 shorter than the window (bench.config_batch): spot rows - the
window-only requests, the longest, and a spread of others - against the oracle's composition of the
reference ops (window_attention_fa, history_attention, the B einsum, merge_states; s6_layer.py:87-115).
"""
import math

import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu
O_TOL = dict(atol=2e-2, rtol=1e-2)


def test_config3_writer_full_size_placement_and_sampled_rows():
    dec, pre = pkg('decode'), pkg('prefill')
    shape = dec.OuroShape(layers=1)
    m = pre.PrefillWriter(shape, 8, 4096, device='cuda', seed=13)
    assert m.T == 32768
    m.step()
    torch.cuda.synchronize()
    page = shape.page
    req = torch.arange(m.R, device='cuda').repeat_interleave(m.L)
    slots = m.block_table[req, m.positions // page].long() * page + m.positions % page
    for cache, width in ((m.l1[0], shape.rank1), (m.main[0], shape.rank)):
        flat = cache.view(-1, 2 * width)
        written = torch.isfinite(flat.float()).all(-1)
        expect = torch.zeros_like(written)
        expect[slots] = True
        assert torch.equal(written, expect)                      # every slot once, nothing else
        assert int(torch.isinf(flat[~expect].float()).all(-1).sum()) == int((~expect).sum())
    rng = np.random.default_rng(13)
    rows = np.sort(rng.choice(m.T, 384, replace=False))
    rows[:2] = [0, m.T - 1]
    pos = m.positions.cpu().numpy()[rows]
    sl = slots.cpu().numpy()[rows]
    h = [m.h[t][torch.from_numpy(rows).cuda()].float().cpu().numpy() for t in range(shape.loops)]
    lat = m.layers[0]
    E = [lat.writer(t).float().cpu().numpy() for t in range(shape.loops)]
    first = orc.write_update(h[0], E[0])
    reg = None
    for t in range(1, shape.loops):
        reg = orc.write_step(reg, orc.write_update(h[t], E[t]))
    for cache, row, width in ((m.l1[0], first, shape.rank1), (m.main[0], reg, shape.rank)):
        table = m.tables[width].float().cpu().numpy()
        want = orc.committed_row(row, width, pos, table)
        got = cache.view(-1, 2 * width)[torch.from_numpy(sl).cuda()].float().cpu().numpy()
        np.testing.assert_allclose(got, want, atol=3e-2, rtol=1e-2)


def _compact(cache, table, n_pages):
    """The pages rows' tables reference (first n_pages[i] columns of row i), copied to the host and renumbered."""
    used = sorted({int(b) for i, r in enumerate(table) for b in r[:n_pages[i]]} | {0})
    remap = {b: j for j, b in enumerate(used)}
    sub = cache[torch.tensor(used, device=cache.device).long()].float().cpu().numpy()
    out = np.zeros_like(table)
    for i, r in enumerate(table):
        out[i, :n_pages[i]] = [remap[int(b)] for b in r[:n_pages[i]]]
    return sub, out


def test_config4_mixed_batch_decode_step_spot_rows():
    import bench
    dec = pkg('decode')
    ctx = bench.config_batch(4, 0, 1, 0)[0]
    assert len(ctx) == 256 and sum(c < 32 for c in ctx) == 8 and max(ctx) <= 32768
    shape = dec.OuroShape(layers=1)
    m = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=4)
    stream = pkg('_lib').stream_of(m.out)
    order = np.argsort(ctx)
    rows = sorted(set(order[:8].tolist()) | {int(order[-1]), int(order[-2])} |
                  set(order[np.linspace(8, 255, 8).astype(int)].tolist()))
    c = np.asarray(ctx)[rows]
    scale = 1 / math.sqrt(shape.head_dim)
    page, W = shape.page, shape.window
    n = len(rows)
    for loop in range(shape.loops):
        m.layer_loop(0, loop, stream)
        torch.cuda.synchronize()
        A, Bm, width = m.layers[0].readers(loop)
        idx = torch.tensor(rows, device='cuda')
        q_lat = m.q_lat[idx, :, :width].float().cpu().numpy()
        q_rope = m.q_rope[idx].float().cpu().numpy()
        cache = m.l1[0] if loop == 0 else m.main[0]
        ctx_lat = np.maximum(c - W, 0)
        lat, ltab = _compact(cache, m.latent_table[idx].cpu().numpy(), -(-ctx_lat // page))
        ex, etab = _compact(m.exact_logical[0][loop], m.exact_table[idx].cpu().numpy(), -(-(c + 1) // page))
        ref = orc.attend_decode(q_lat, q_rope, lat, ltab, ctx_lat, ex, etab, np.arange(n + 1), c + 1, W,
                                Bm.float().cpu().numpy(), scale, np.zeros(n, dtype=bool))
        got = m.out[0, loop][idx].float().cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, ref, **O_TOL)
    assert torch.isfinite(m.out.float()).all()
