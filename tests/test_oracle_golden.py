"""Pin the CPU oracle to the reference: oracle outputs vs fixtures produced by the reference's
own torch code (tests/golden/gen_golden.py).  CPU only."""
import json
import math

import numpy as np
import pytest

import cases
from conftest import GOLDEN
from oracle import s6_oracle as orc

INF = float('inf')


def load(name, inputs):
    f = np.load(GOLDEN / f'{name}.npz')
    assert str(f['input_sha256']) == cases.digest(inputs), f'{name}: regenerated inputs differ from the fixture'
    return f


@pytest.mark.parametrize('name', sorted(cases.history_cases()))
def test_history_oracle_matches_reference(name):
    inp, scale = cases.history_cases()[name]
    g = load(name, inp)
    o, lse = orc.history_attention(inp['q'], inp['cache'], inp['block_table'], inp['ctx'], scale)
    assert np.isfinite(o).all() and not np.isnan(lse).any()
    np.testing.assert_allclose(o, g['o'], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(lse, g['lse'], rtol=1e-5, atol=2e-6)
    empty = inp['ctx'] == 0
    assert (o[empty] == 0).all() and (lse[:, empty] == -INF).all()


@pytest.mark.parametrize('name,kw', [('contig_512', dict(width=512)),
                                     ('contig_256', dict(seed=82, width=256, keys=37, batch=4))])
def test_contiguous_reader_oracle_matches_reference(name, kw):
    c = cases.contig_case(**kw)
    g = load(name, c)
    z, lse = orc.contiguous_history(c['q'], c['k'], c['v'], c['mask'].astype(bool), float(g['scale']))
    np.testing.assert_allclose(z, g['z'], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(lse, g['lse'], rtol=1e-5, atol=2e-6)
    assert (z[1] == 0).all() and (lse[1] == -INF).all()          # fully masked row


def test_export_oracle_matches_reference_known_answer():
    """The reference's own known answer (hla/tests/test_rollout_cache.py:36-37): fp32 caches
    arange(3*1*2*w) of widths 4 and 2, main blocks [2, 0], loop-1 blocks [1, 2], block size 2,
    three positions."""
    main = np.arange(3 * 1 * 2 * 4, dtype=np.float32).reshape(3, 1, 2, 4)
    l1 = np.arange(3 * 1 * 2 * 2, dtype=np.float32).reshape(3, 1, 2, 2)
    expected = np.concatenate([main[[2, 2, 0], 0, [0, 1, 0]], l1[[1, 1, 2], 0, [0, 1, 0]]], -1)[None]
    rows = orc.export_rows([main], [l1], [2, 0], [1, 2], 2, 3)
    assert len(rows) == 1
    np.testing.assert_array_equal(rows[0], expected)


def test_export_oracle_matches_reference_exporter():
    ec = cases.export_case()
    g = load('export', ec)
    rows = orc.export_rows(list(ec['main']), list(ec['l1']), ec['main_blocks'], ec['l1_blocks'],
                           int(ec['block_size']), int(ec['length']))
    np.testing.assert_array_equal(np.stack(rows), g['rows'])


@pytest.mark.parametrize('name,kw', [('heads_lla', dict()),
                                     ('heads_gqa', dict(seed=102, kv_heads=4, rank=64, d_rope=32, ctx=(40, 0, 16, 333)))])
def test_per_head_history_oracle_matches_reference(name, kw):
    hc = cases.heads_case(**kw)
    g = load(name, hc)
    r = int(hc['rank'])
    o, lse = orc.history_attention_kv(hc['q'], hc['cache'], hc['cache'][..., :r], hc['block_table'], hc['ctx'],
                                      float(g['scale']))
    assert np.isfinite(o).all()
    np.testing.assert_allclose(o, g['o'], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(lse, g['lse'], rtol=1e-5, atol=2e-6)


def test_window_decode_oracle_matches_reference():
    w = cases.window_case()
    g = load('window_decode', w)
    logical = w['cache_phys'].transpose(0, 2, 1, 3)
    T = w['q'].shape[0]
    _, valid = orc.token_requests(w['query_start_loc'], T)
    o, lse = orc.window_decode(w['q'], logical, w['block_table'], w['query_start_loc'], w['seq_lens'],
                               int(w['window']), float(g['scale']), ~valid)
    np.testing.assert_allclose(o, g['o'], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(lse, g['lse'], rtol=1e-5, atol=2e-6)


def test_merges_match_reference():
    m = cases.merge_case()
    g = load('merge', m)
    out = orc.merge_states(m['o_hist'], m['lse_hist'], m['o_chunk'], m['lse_chunk'], m['invalid'])
    np.testing.assert_allclose(out, g['merge_states'], rtol=1e-6, atol=1e-6)
    assert np.isfinite(out).all()
    l_c = np.where(m['lse_chunk'] == INF, -INF, m['lse_chunk'])
    o2, l2 = orc.merge_lse(m['o_hist'], m['lse_hist'], m['o_chunk'], l_c)
    np.testing.assert_allclose(o2, g['merge_lse_o'], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(l2, g['merge_lse_lse'], rtol=1e-6, atol=1e-6)


def test_latent_rope_tables_and_rotation_match_reference():
    r = cases.rope_case()
    g = load('rope', r)
    inv = orc.latent_inv_freq(int(r['head_dim']), float(r['theta']))
    # torch's vectorised pow and numpy's differ by at most one float32 ulp here
    np.testing.assert_allclose(inv, g['inv_freq'], rtol=3e-7, atol=0)
    pos = r['positions']
    rows = np.arange(pos.shape[0])
    for w in (512, 256):
        table = orc.latent_rope_table(int(r['max_pos']), inv, w)
        # a one-ulp inv_freq difference grows with the angle p * inv_freq (p < 4096 here)
        np.testing.assert_allclose(table[pos], g[f'table{w}_rows'], rtol=0, atol=5e-4)
        np.testing.assert_allclose(orc.bf16(table)[pos], g[f'table{w}_bf16_rows'], rtol=0, atol=8e-3)
        # rotation given the reference's own bf16 table rows: the torch bf16 operation order, bit-exact
        tb = g[f'table{w}_bf16_rows']
        out = orc.latent_rope(r[f'x{w}'], rows, tb, emulate_bf16=True)
        np.testing.assert_array_equal(out, g[f'rope{w}_bf16'])
        row = orc.latent_rope(r[f'row{w}'][:, :w], rows, tb, emulate_bf16=True)
        np.testing.assert_array_equal(row, g[f'rowrope{w}_bf16'])
        out32 = orc.latent_rope(r[f'x{w}'], rows, g[f'table{w}_rows'])
        np.testing.assert_allclose(out32, g[f'rope{w}_f32'], rtol=1e-5, atol=1e-5)


def test_writer_rows_match_reference_bit_exactly():
    wc = cases.writer_case()
    g = load('writer', wc)
    rank, rank1 = int(wc['rank']), int(wc['rank1'])
    inv = orc.latent_inv_freq(128, float(wc['theta']))
    tab = {w: orc.bf16(orc.latent_rope_table(int(wc['max_pos']), inv, w)) for w in (rank, rank1)}
    first = orc.write_update(wc['h'][0], wc['E1'])
    reg = None
    regs = []
    for loop in range(1, 4):
        reg = orc.write_step(reg, orc.write_update(wc['h'][loop], wc['E'][loop - 1]))
        regs.append(reg)
    # GEMM rounding may differ in the last bf16 bit between fp64-then-round and cuBLAS/CPU fp32
    # accumulation; everything after the GEMM is replayed bit-exactly below from the reference's values.
    np.testing.assert_allclose(first, g['first'], rtol=1e-2, atol=1e-2)
    for i, r_ in enumerate(regs):
        np.testing.assert_allclose(r_, g[f'reg{i + 1}'], rtol=2e-2, atol=2e-2)
    np.testing.assert_array_equal(orc.write_step(g['reg2'], orc.bf16(g['reg3'] - g['reg2'])) * 0 + g['reg3'], g['reg3'])
    row_l1 = orc.committed_row(g['first'], rank1, wc['positions'], tab[rank1])
    row_main = orc.committed_row(g['reg3'], rank, wc['positions'], tab[rank])
    np.testing.assert_array_equal(row_l1, g['row_l1'])
    np.testing.assert_array_equal(row_main, g['row_main'])
    packed = orc.pack(g['reg3'], g['first'], wc['positions'], tab[rank], tab[rank1], rank, rank1)
    np.testing.assert_array_equal(packed, g['packed'])


def test_integer_metadata_matches_reference():
    meta = json.loads((GOLDEN / 'meta.json').read_text())
    mc = cases.meta_cases()
    for (qsl, n), (req, valid) in zip(mc['token_requests'], meta['reference']['token_requests']):
        r, v = orc.token_requests(qsl, n)
        assert r.tolist() == req and v.tolist() == valid
    for (a, b), want in zip(mc['history_lengths'], meta['reference']['history_lengths']):
        assert orc.history_lengths(a, b).tolist() == want
    for c, want in zip(mc['num_kv_splits'], meta['reference']['num_kv_splits']):
        assert orc.num_kv_splits(*c) == want


def test_oracle_step_context_matches_reference():
    """The oracle's StepContext restatement against the reference's own fields (step_context.json)."""
    ref = json.loads((GOLDEN / 'step_context.json').read_text())
    assert len(ref) == len(cases.step_context_cases())
    for (qsl, seq_lens, T, window, table), want in zip(cases.step_context_cases(), ref):
        req, valid, ctx, ctx_lat = orc.step_context(qsl, seq_lens, T, window)
        assert req.tolist() == want['token_requests'] and valid.tolist() == want['valid']
        assert ctx.tolist() == want['ctx'] and ctx_lat.tolist() == want['ctx_latent']
        assert (ctx == 0).tolist() == want['empty'] and (ctx_lat == 0).tolist() == want['empty_latent']
        assert np.asarray(table, dtype=np.int32)[req].tolist() == want['block_table']


def test_oracle_decode_attend_equals_joint_softmax():
    """Independent check of the composed oracle (window + history + B + merge) against one
    joint softmax, as batched_engine.mixed_attention computes it."""
    rng = np.random.default_rng(7)
    H, d, W, page, window = 4, 16, 32, 4, 3
    seq_len = 12                                   # ctx 11: latent rows [0, 8), window [8, 11), current 11
    ctx = seq_len - 1
    ctx_lat = ctx - window
    lat = rng.standard_normal((4, 1, page, 2 * W))
    ex_phys = rng.standard_normal((4, page, H, 2 * d))
    ex = ex_phys.transpose(0, 2, 1, 3)
    bt = np.array([[2, 0, 3, 1]], dtype=np.int32)
    q_lat = rng.standard_normal((1, H, W))
    q_rope = rng.standard_normal((1, H, d))
    B = rng.standard_normal((H, W, d)) / math.sqrt(W)
    scale = 1 / math.sqrt(d)
    out = orc.attend_decode(q_lat, q_rope, lat, bt, np.array([ctx_lat]), ex, bt, np.array([0, 1]),
                            np.array([seq_len]), window, B, scale, np.array([False]))
    lat_rows = np.stack([lat[bt[0, j // page], 0, j % page] for j in range(ctx_lat)])
    ex_rows = np.stack([ex_phys[bt[0, j // page], j % page] for j in range(ctx_lat, seq_len)])
    joint = orc.joint_decode(q_lat[0], q_rope[0], lat_rows, ex_rows, B, scale)
    np.testing.assert_allclose(out[0], joint, rtol=1e-10, atol=1e-10)


def test_slot_mapping_and_scatter_skip_padding():
    bt = np.array([[5, 2, 7], [3, 1, 0]], dtype=np.int32)
    req = np.array([0, 0, 1, 1])
    pos = np.array([17, 33, 0, 5])
    valid = np.array([True, True, True, False])
    slots = orc.cache_slots(bt, req, pos, valid, 16)
    assert slots.tolist() == [2 * 16 + 1, 7 * 16 + 1, 3 * 16 + 0, -1]
    cache = np.full((8, 1, 16, 4), np.nan, dtype=np.float32)
    rows = np.arange(16, dtype=np.float32).reshape(4, 4)
    orc.scatter_rows(cache, rows, slots)
    flat = cache.reshape(-1, 4)
    written = {int(s) for s in slots if s >= 0}
    for s in range(flat.shape[0]):
        assert np.isnan(flat[s]).all() != (s in written)


def test_config1_decode_op_matches_reference():
    """BASELINE config 1 - one layer x 4 loops of the S6 decode op at context 2048 (2016 latent rows, W = 32
    window + the current token, identity page tables), the reference computing in fp32: the oracle's
    latent query (from q_pre and the absorb A, bf16 RoPE table) and its history + B + window + merge
    composition against the reference's outputs, loop by loop (loop 0 on the 256-wide loop-1 latent)."""
    c = cases.config1_case()
    g = load('config1', c)
    scale = float(g['scale'])
    inv = orc.latent_inv_freq(128, float(c['latent_theta']))
    ex_bt = c['table']
    for t in range(4):
        w = 256 if t == 0 else 512
        table = orc.bf16(orc.latent_rope_table(int(c['max_pos']), inv, w))
        # the reference runs the latent query in bf16: the einsum rounded once, then the torch bf16 RoPE order
        x = orc.bf16(np.einsum('thd,hdr->thr', c[f'q_pre{t}'].astype(np.float64), c[f'A{t}'].astype(np.float64)))
        q_lat = orc.latent_rope(x, c['positions'], table, emulate_bf16=True)
        same = q_lat == g[f'q_lat{t}']
        assert same.mean() > 0.99, f'loop {t}: {same.mean():.4f} of q_lat bit-exact'
        np.testing.assert_allclose(q_lat, g[f'q_lat{t}'], rtol=0, atol=1.6e-2)   # the rest: one bf16 ulp apart
        cache = c['lat_l1'] if t == 0 else c['lat_main']
        o, lse = orc.history_attention(g[f'q_lat{t}'], cache, c['table'], c['ctx_lat'], scale)
        np.testing.assert_allclose(lse, g[f'lse_hist{t}'], atol=1e-5, rtol=0)
        out = orc.attend_decode(g[f'q_lat{t}'], c[f'q_rope{t}'], cache, c['table'], c['ctx_lat'],
                                c[f'exact{t}'].transpose(0, 2, 1, 3), ex_bt, c['query_start_loc'], c['seq_lens'],
                                int(c['window']), c[f'B{t}'], scale, np.zeros(1, dtype=bool))
        np.testing.assert_allclose(out, g[f'out{t}'], rtol=1e-4, atol=1e-5)
        assert np.isfinite(out).all() and np.abs(out).max() > 1e-3
