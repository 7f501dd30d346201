"""Decode ops around the history reader vs the reference fixtures and the oracle (GPU).

Tolerances: bf16 outputs 2e-2 max-abs / 1e-2 relative, LSE 1e-3;
slot placement and committed-row values bit-exact (rows: given the same register values).
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
O_TOL = dict(atol=2e-2, rtol=1e-2)
LSE_ATOL = 1e-3
INF = float('inf')


def ops():
    return pkg('s6_ops')


def layer():
    return pkg('s6_layer')


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


def golden(name, inputs):
    g = np.load(GOLDEN / f'{name}.npz')
    assert str(g['input_sha256']) == cases.digest(inputs)
    return g


# ----------------------------------------------------------------------------- A5 window
def test_window_decode_matches_reference_fixture():
    w = cases.window_case()
    g = golden('window_decode', w)
    phys = dev(w['cache_phys'], BF16)
    logical = phys.transpose(1, 2)
    q = dev(w['q'], BF16)
    T = q.shape[0]
    qsl, seq_lens = dev(w['query_start_loc']), dev(w['seq_lens'])
    _, valid = ops().token_requests(qsl, T)
    o, lse = ops().window_attention_fa(q, logical, dev(w['block_table']), qsl, seq_lens, int(w['window']),
                                       float(g['scale']), 0, ~valid)
    o, lse = o.float().cpu().numpy(), lse.cpu().numpy()
    valid = valid.cpu().numpy()
    np.testing.assert_allclose(o[valid], g['o'][valid], **O_TOL)
    np.testing.assert_allclose(lse[:, valid], g['lse'][:, valid], atol=LSE_ATOL, rtol=0)
    assert (lse[:, ~valid] == -INF).all() and (o[~valid] == 0).all()


@pytest.mark.parametrize('window', [0, 1, 32, 100])
def test_window_matches_oracle_for_window_sizes(window):
    w = cases.window_case(seed=window + 3, window=window, seq_lens=(1, 7, 40, 129, 300, 17, 16, 33), padding=1)
    q = dev(w['q'], BF16)
    T = q.shape[0]
    qsl, seq_lens = dev(w['query_start_loc']), dev(w['seq_lens'])
    _, valid = ops().token_requests(qsl, T)
    o, lse = ops().window_attention_fa(q, dev(w['cache_phys'], BF16).transpose(1, 2), dev(w['block_table']), qsl,
                                       seq_lens, window, 1 / math.sqrt(128), 0, ~valid)
    o_ref, lse_ref = orc.window_decode(w['q'], w['cache_phys'].transpose(0, 2, 1, 3), w['block_table'],
                                       w['query_start_loc'], w['seq_lens'], window, 1 / math.sqrt(128),
                                       ~valid.cpu().numpy())
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, **O_TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=LSE_ATOL, rtol=0)


# ----------------------------------------------------------------------------- A7 merges
def test_merges_match_reference_fixture():
    m = cases.merge_case()
    g = golden('merge', m)
    o_h, o_c = dev(m['o_hist'], BF16), dev(m['o_chunk'], BF16)
    l_h, l_c = dev(m['lse_hist']), dev(m['lse_chunk'])
    out = ops().merge_states(o_h, l_h, o_c, l_c, dev(m['invalid']), 'b200')
    assert out.dtype == BF16 and torch.isfinite(out).all()
    np.testing.assert_allclose(out.float().cpu().numpy(), g['merge_states'], **O_TOL)
    assert (out[2] == 0).all() and (out[7] == 0).all()
    l_c2 = dev(np.where(m['lse_chunk'] == INF, -INF, m['lse_chunk']).astype(np.float32))
    o2, l2 = ops().merge_lse(o_h, l_h, o_c, l_c2)
    np.testing.assert_allclose(o2.float().cpu().numpy(), g['merge_lse_o'], **O_TOL)
    np.testing.assert_allclose(l2.cpu().numpy(), g['merge_lse_lse'], atol=LSE_ATOL, rtol=0)


def test_merge_lse_ignores_nan_scratch():
    o1 = torch.full((2, 16, 128), float('nan'), dtype=BF16, device=CUDA)
    o2 = torch.randn(2, 16, 128, dtype=BF16, device=CUDA)
    l1 = torch.full((16, 2), -INF, device=CUDA)
    l2 = torch.zeros(16, 2, device=CUDA)
    o, l = ops().merge_lse(o1, l1, o2, l2)
    assert torch.equal(o, o2) and torch.equal(l, l2)


# ----------------------------------------------------------------------------- A4 RoPE / query
@pytest.mark.parametrize('w', [512, 256])
def test_latent_rope_is_bit_exact_with_reference(w):
    r = cases.rope_case()
    g = golden('rope', r)
    T = r['positions'].shape[0]
    table = dev(g[f'table{w}_bf16_rows'], BF16)            # row t = the reference's table row at positions[t]
    pos = torch.arange(T, device=CUDA, dtype=torch.int64)
    x = dev(r[f'x{w}'], BF16).transpose(0, 1).contiguous().transpose(0, 1)   # einsum-shaped head stride
    y = ops().latent_rope(x, pos, table, 'b200')
    assert y is x
    np.testing.assert_array_equal(y.float().cpu().numpy(), g[f'rope{w}_bf16'])
    row = dev(r[f'row{w}'], BF16)
    v_before = row[:, w:].clone()
    ops().latent_rope(row[:, :w], pos, table, 'b200')
    np.testing.assert_array_equal(row[:, :w].float().cpu().numpy(), g[f'rowrope{w}_bf16'])
    assert torch.equal(row[:, w:], v_before)
    flat = dev(r[f'x{w}'], BF16).reshape(T, -1).contiguous()
    ops().latent_rope(flat, pos, table, 'b200')
    np.testing.assert_array_equal(flat.view(T, -1, w).float().cpu().numpy(), g[f'rope{w}_bf16'])
    # the LLA row / query tail: [T, H, 512 + w] rows whose last w columns are rotated in place (head stride
    # 512 + w, the fourth layout of the reference's test_s6_ops_gpu.py:221-240); the latent head stays untouched
    H = r[f'x{w}'].shape[1]
    lla = torch.randn(T, H, 512 + w, dtype=BF16, device=CUDA)
    lla[..., 512:] = dev(r[f'x{w}'], BF16)
    head_before = lla[..., :512].clone()
    y = ops().latent_rope(lla[..., 512:], pos, table, 'b200')
    assert y.stride() == lla[..., 512:].stride()
    np.testing.assert_array_equal(lla[..., 512:].float().cpu().numpy(), g[f'rope{w}_bf16'])
    assert torch.equal(lla[..., :512], head_before)


@pytest.mark.parametrize('w', [512, 256])
def test_latent_query_matches_oracle(w):
    rng = np.random.default_rng(w)
    T, H, d, max_pos = 37, 16, 128, 4096
    q = orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32))
    A = orc.bf16(rng.standard_normal((H, d, w), dtype=np.float32) / math.sqrt(128))
    pos = rng.integers(0, max_pos, T)
    inv = layer().latent_inv_freq(d, 1e6)
    table = layer().latent_rope_table(max_pos, inv, w, BF16)
    out = layer().latent_query(dev(q, BF16), dev(A, BF16), dev(pos), table.to(CUDA), 'b200')
    ref = orc.latent_query(q, A, pos, table.float().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, **O_TOL)
    # the fused kernel equals einsum->bf16 then the torch-order rotation, bit for bit
    x = orc.bf16(np.einsum('thd,hdr->thr', q.astype(np.float64), A.astype(np.float64)).astype(np.float32))
    rot = orc.latent_rope(x, pos, table.float().numpy(), emulate_bf16=True)
    mism = (out.float().cpu().numpy() != rot).mean()
    assert mism < 0.01   # only last-bit differences from fp32-vs-fp64 accumulation of the einsum


# ----------------------------------------------------------------------------- A10 exact append
def test_exact_append_places_rows_bit_exactly_and_ropes():
    rng = np.random.default_rng(5)
    H, d, page, max_pos = 16, 128, 16, 4096
    seq_lens = np.array([1, 17, 33, 200, 5], dtype=np.int32)
    R, T = len(seq_lens), len(seq_lens) + 2
    qsl = np.concatenate(([0], np.arange(1, R + 1))).astype(np.int32)
    need = -(-seq_lens // page)
    nb = int(need.sum()) + 3
    table = np.zeros((R, int(need.max()) + 1), dtype=np.int32)
    free = rng.permutation(np.arange(1, nb))
    k = 0
    for r in range(R):
        table[r, :need[r]] = free[k:k + need[r]]
        k += need[r]
    positions = np.concatenate((seq_lens - 1, [0, 0])).astype(np.int64)
    q, kk, v = (orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32)) for _ in range(3))
    inv = layer().latent_inv_freq(d, 1e6)
    ang = torch.arange(max_pos).float()[:, None] * inv[None]
    cos_sin = torch.cat((ang.cos(), ang.sin()), -1).to(CUDA)
    cache = torch.full((nb, page, H, 2 * d), float('nan'), dtype=BF16, device=CUDA)   # physical
    logical = cache.transpose(1, 2)
    qd, kd, vd = dev(q, BF16), dev(kk, BF16), dev(v, BF16)
    slots = torch.empty(T, dtype=torch.int64, device=CUDA)
    lib = pkg('_lib')
    pos_d, table_d, qsl_d = dev(positions), dev(table), dev(qsl)   # keep the buffers alive across the launch
    lib.call('hla_s6_exact_append', lib.ptr(qd), qd.stride(0), qd.stride(1), lib.ptr(kd), kd.stride(0), kd.stride(1),
             lib.ptr(vd), vd.stride(0), vd.stride(1), None, 0, 0, lib.ptr(pos_d), lib.ptr(cos_sin),
             cos_sin.stride(0), max_pos, lib.ptr(logical), nb, logical.stride(0), logical.stride(1),
             logical.stride(2), page, lib.ptr(table_d), table.shape[1], table.shape[1], lib.ptr(qsl_d), R, T, H,
             d, lib.ptr(slots), lib.stream_of(qd))
    req, valid = orc.token_requests(qsl, T)
    want = orc.cache_slots(table, req, positions, valid, page)
    assert slots.cpu().numpy().tolist() == want.tolist()
    k_ref = orc.neox_rope(kk, positions, d, 1e6)
    q_ref = orc.neox_rope(q, positions, d, 1e6)
    np.testing.assert_allclose(qd.float().cpu().numpy(), q_ref, **O_TOL)
    flat = cache.float().cpu().numpy().reshape(nb * page, H, 2 * d)
    written = set()
    for t in range(T):
        if want[t] < 0:
            continue
        written.add(int(want[t]))
        np.testing.assert_allclose(flat[want[t], :, :d], k_ref[t], **O_TOL)
        np.testing.assert_array_equal(flat[want[t], :, d:], v[t])
    untouched = [s for s in range(nb * page) if s not in written]
    assert np.isnan(flat[untouched]).all()


# ----------------------------------------------------------------------------- A9 writer + commit
def test_writer_and_committed_rows_match_reference_fixture():
    wc = cases.writer_case()
    g = golden('writer', wc)
    lat = pkg('latent').LatentLayer(wc['h'].shape[-1], 16, 128, 4, int(wc['rank']), int(wc['rank']),
                                    int(wc['rank1'])).to(CUDA, BF16)
    with torch.no_grad():
        for i in range(3):
            lat.cand_s[i].weight.copy_(dev(wc['E'][i], BF16))
        lat.cand1.weight.copy_(dev(wc['E1'], BF16))
    state = None
    regs = []
    for loop in range(4):
        state = layer().write_rows(lat, loop, dev(wc['h'][loop], BF16), state)
        regs.append(state.first if loop == 0 else state.reg)
    np.testing.assert_allclose(regs[0].float().cpu().numpy(), g['first'], **O_TOL)
    for i in range(1, 4):
        np.testing.assert_allclose(regs[i].float().cpu().numpy(), g[f'reg{i}'], atol=3e-2, rtol=1e-2)
    # commit kernels from the reference's register values: bit-exact rows and placement
    T = wc['positions'].shape[0]
    pos = dev(wc['positions'])
    inv = layer().latent_inv_freq(128, float(wc['theta']))
    lib = pkg('_lib')
    qsl = torch.arange(T + 1, dtype=I32, device=CUDA)
    for name, src, w in (('row_l1', g['first'], int(wc['rank1'])), ('row_main', g['reg3'], int(wc['rank']))):
        table = layer().latent_rope_table(int(wc['max_pos']), inv, w, BF16).to(CUDA)
        page, nb = 16, 40
        cache = torch.full((nb, 1, page, 2 * w), float('nan'), dtype=BF16, device=CUDA)
        bt = torch.randperm(nb - 1, device=CUDA).to(I32)[: T * 2].view(T, 2) + 1
        posm = pos % 32
        slots = torch.empty(T, dtype=torch.int64, device=CUDA)
        row = dev(src, BF16)
        lib.call('hla_s6_commit_rows', lib.ptr(row), row.stride(0), w, lib.ptr(posm), lib.ptr(table),
                 table.stride(0), table.shape[0], lib.ptr(cache), nb, cache.stride(0), cache.stride(2), page,
                 lib.ptr(bt), bt.stride(0), bt.shape[1], lib.ptr(qsl), T, T, lib.ptr(slots), lib.stream_of(row))
        want_slots = bt[torch.arange(T, device=CUDA), posm // page].long() * page + posm % page
        assert torch.equal(slots, want_slots)
        got = cache.view(-1, 2 * w)[slots]
        # the fixture rotated at the true positions; recompute the expected row at posm with the oracle
        expect = orc.committed_row(src, w, posm.cpu().numpy(), table.float().cpu().numpy())
        np.testing.assert_array_equal(got.float().cpu().numpy(), expect)
        mask = torch.ones(nb * page, dtype=torch.bool, device=CUDA)
        mask[slots] = False
        assert torch.isnan(cache.view(-1, 2 * w)[mask]).all()


def test_committed_row_in_place_matches_reference_fixture():
    wc = cases.writer_case()
    g = golden('writer', wc)
    inv = layer().latent_inv_freq(128, float(wc['theta']))
    rank, rank1 = int(wc['rank']), int(wc['rank1'])
    tables = {w: layer().latent_rope_table(int(wc['max_pos']), inv, w, BF16).to(CUDA) for w in (rank, rank1)}

    class Ctx:
        positions = dev(wc['positions'])
        backends = ops().B200_BACKENDS
    Ctx.tables = tables

    from types import SimpleNamespace
    SL = SimpleNamespace(loops=4, rank=rank, rank1=rank1)
    st = layer().WriterState(None, dev(g['first'], BF16))
    k, v = layer().committed_row(SL, 0, st, Ctx)
    np.testing.assert_array_equal(torch.cat((k, v), -1).float().cpu().numpy(), g['row_l1'])
    st = layer().WriterState(dev(g['reg3'], BF16), None)
    k, v = layer().committed_row(SL, 3, st, Ctx)
    np.testing.assert_array_equal(torch.cat((k, v), -1).float().cpu().numpy(), g['row_main'])
    assert layer().committed_row(SL, 1, st, Ctx) is None


# ----------------------------------------------------------------------------- fused entry points
# 37: mma.sync path; 200: single-CTA tcgen05 tiles (ragged tail); 300: CTA-pair tiles (ragged second
# pair tile); 20000: several pair tiles per persistent cluster
@pytest.mark.parametrize('T', [37, 200, 300, 20000])
@pytest.mark.parametrize('loop', [0, 3])
def test_writer_commit_equals_project_then_commit(loop, T):
    """The commit fused into the writer epilogue writes exactly the rows that the projection followed
    by the torch-order RoPE would (bit for bit), at exactly the vLLM slots; nothing else changes."""
    rng = np.random.default_rng(loop + 7 + T)
    K, page, max_pos = 256, 16, 4096
    w = 256 if loop == 0 else 512
    N = 2 * w
    h = dev(orc.bf16(rng.standard_normal((T, K), dtype=np.float32)), BF16)
    E = dev(orc.bf16(rng.standard_normal((N, K), dtype=np.float32) / 16), BF16)
    reg_in = None if loop == 0 else dev(orc.bf16(rng.standard_normal((T, N), dtype=np.float32)), BF16)
    lib = pkg('_lib')
    st = lib.stream_of(h)
    reg = torch.empty(T, N, dtype=BF16, device=CUDA)
    lib.call('hla_s6_writer_project', lib.ptr(h), h.stride(0), lib.ptr(E), E.stride(0), lib.ptr(reg_in),
             0 if reg_in is None else reg_in.stride(0), lib.ptr(reg), reg.stride(0), T, N, K, st)
    R = T - 3                                                   # three padding tokens
    qsl = torch.tensor(list(range(R + 1)), dtype=I32, device=CUDA)
    pos = torch.from_numpy(rng.integers(0, 2 * page, T)).to(CUDA)
    nb = 2 * R + 2
    bt = (torch.randperm(nb - 1, device=CUDA).to(I32)[:2 * R] + 1).view(R, 2)
    inv = layer().latent_inv_freq(128, 1e6)
    table = layer().latent_rope_table(max_pos, inv, w, BF16).to(CUDA)
    cache = torch.full((nb, 1, page, 2 * w), float('nan'), dtype=BF16, device=CUDA)
    lib.call('hla_s6_writer_commit', lib.ptr(h), h.stride(0), lib.ptr(E), E.stride(0), lib.ptr(reg_in),
             0 if reg_in is None else reg_in.stride(0), None, 0, T, N, K, lib.ptr(pos), lib.ptr(table),
             table.stride(0), table.shape[0], lib.ptr(cache), nb, cache.stride(0), cache.stride(2), page, lib.ptr(bt),
             bt.stride(0), bt.shape[1], lib.ptr(qsl), R, st)
    torch.cuda.synchronize()
    slots = (bt[torch.arange(R, device=CUDA), pos[:R] // page].long() * page + pos[:R] % page)
    expect = orc.committed_row(reg[:R].float().cpu().numpy(), w, pos[:R].cpu().numpy(), table.float().cpu().numpy())
    flat = cache.view(-1, 2 * w)
    np.testing.assert_array_equal(flat[slots].float().cpu().numpy(), expect)
    mask = torch.ones(flat.shape[0], dtype=torch.bool, device=CUDA)
    mask[slots] = False
    assert torch.isnan(flat[mask]).all()
    # the projection itself against the oracle (bf16 GEMM tolerance)
    upd = orc.write_update(h.float().cpu().numpy(), E.float().cpu().numpy())
    ref = upd if reg_in is None else orc.write_step(reg_in.float().cpu().numpy(), upd)
    np.testing.assert_allclose(reg.float().cpu().numpy(), ref, atol=3e-2, rtol=1e-2)


def test_decode_prepare_fuses_latent_query_and_exact_append():
    rng = np.random.default_rng(17)
    T, H, d, W, page, max_pos = 21, 16, 128, 512, 16, 4096
    R = T - 2
    q = orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32))
    k = orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32))
    v = orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32))
    A = orc.bf16(rng.standard_normal((H, d, W), dtype=np.float32) / math.sqrt(128))
    pos = rng.integers(0, 3 * page, T).astype(np.int64)
    nb = 3 * R + 1
    table_e = (np.arange(1, nb, dtype=np.int32)).reshape(R, 3)
    inv = layer().latent_inv_freq(d, 1e6)
    ltab = layer().latent_rope_table(max_pos, inv, W, BF16).to(CUDA)
    ang = torch.arange(max_pos).float()[:, None] * inv[None]
    cos_sin = torch.cat((ang.cos(), ang.sin()), -1).to(CUDA)
    qd, kd, vd, Ad = dev(q, BF16), dev(k, BF16), dev(v, BF16), dev(A, BF16)
    q_before = qd.clone()
    posd, btd = dev(pos), dev(table_e)
    qsl = torch.arange(R + 1, dtype=I32, device=CUDA)
    q_lat = torch.empty(T, H, W, dtype=BF16, device=CUDA)
    q_rope = torch.empty(T, H, d, dtype=BF16, device=CUDA)
    cache = torch.full((nb, page, H, 2 * d), float('nan'), dtype=BF16, device=CUDA)
    logical = cache.transpose(1, 2)
    slots = torch.empty(T, dtype=torch.int64, device=CUDA)
    lib = pkg('_lib')
    lib.call('hla_s6_decode_prepare', lib.ptr(qd), qd.stride(0), qd.stride(1), lib.ptr(Ad), Ad.stride(0),
             Ad.stride(1), lib.ptr(posd), lib.ptr(ltab), ltab.stride(0), ltab.shape[0], lib.ptr(q_lat),
             q_lat.stride(0), q_lat.stride(1), T, H, d, W, lib.ptr(q_rope), q_rope.stride(0), q_rope.stride(1),
             lib.ptr(kd), kd.stride(0), kd.stride(1), lib.ptr(vd), vd.stride(0), vd.stride(1), lib.ptr(cos_sin),
             cos_sin.stride(0), cos_sin.shape[0], lib.ptr(logical), nb, logical.stride(0), logical.stride(1),
             logical.stride(2), page, lib.ptr(btd), btd.stride(0), btd.shape[1], lib.ptr(qsl), R, lib.ptr(slots),
             lib.PREPARE_EARLY_LAUNCH, lib.stream_of(qd))   # staged early behind the torch ops above
    torch.cuda.synchronize()
    assert torch.equal(qd, q_before)   # q_pre is read only
    np.testing.assert_allclose(q_lat.float().cpu().numpy(), orc.latent_query(q, A, pos, ltab.float().cpu().numpy()),
                               **O_TOL)
    np.testing.assert_allclose(q_rope.float().cpu().numpy(), orc.neox_rope(q, pos, d, 1e6), **O_TOL)
    req, valid = orc.token_requests(qsl.cpu().numpy(), T)
    want = orc.cache_slots(table_e, req, pos, valid, page)
    assert slots.cpu().numpy().tolist() == want.tolist()
    flat = cache.float().cpu().numpy().reshape(nb * page, H, 2 * d)
    k_ref = orc.neox_rope(k, pos, d, 1e6)
    for t in range(T):
        if want[t] >= 0:
            np.testing.assert_allclose(flat[want[t], :, :d], k_ref[t], **O_TOL)
            np.testing.assert_array_equal(flat[want[t], :, d:], v[t])
    untouched = np.setdiff1d(np.arange(nb * page), want[want >= 0])
    assert np.isnan(flat[untouched]).all()
    # the same work as two launches on two streams - the latent query alone (k = NULL) and the exact part
    # alone (HLA_S6_PREPARE_EXACT_ONLY) - gives bit-identical q_lat, q_rope, cache rows and slots
    q_lat2, q_rope2 = torch.full_like(q_lat, float('nan')), torch.full_like(q_rope, float('nan'))
    cache2 = torch.full_like(cache, float('nan'))
    logical2 = cache2.transpose(1, 2)
    slots2 = torch.full_like(slots, -7)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    for kv, flags, strm in (((None, None), 0, lib.stream_of(qd)),
                            ((kd, vd), lib.PREPARE_EXACT_ONLY, lib.ctypes.c_void_p(side.cuda_stream))):
        lib.call('hla_s6_decode_prepare', lib.ptr(qd), qd.stride(0), qd.stride(1), lib.ptr(Ad), Ad.stride(0),
                 Ad.stride(1), lib.ptr(posd), lib.ptr(ltab), ltab.stride(0), ltab.shape[0], lib.ptr(q_lat2),
                 q_lat2.stride(0), q_lat2.stride(1), T, H, d, W, lib.ptr(q_rope2), q_rope2.stride(0),
                 q_rope2.stride(1), lib.ptr(kv[0]), kd.stride(0), kd.stride(1), lib.ptr(kv[1]), vd.stride(0),
                 vd.stride(1), lib.ptr(cos_sin), cos_sin.stride(0), cos_sin.shape[0], lib.ptr(logical2), nb,
                 logical2.stride(0), logical2.stride(1), logical2.stride(2), page, lib.ptr(btd), btd.stride(0),
                 btd.shape[1], lib.ptr(qsl), R, lib.ptr(slots2), flags, strm)
    torch.cuda.synchronize()
    assert torch.equal(q_lat2, q_lat) and torch.equal(q_rope2, q_rope) and torch.equal(slots2, slots)
    assert torch.equal(cache2.isnan(), cache.isnan())
    assert torch.equal(torch.nan_to_num(cache2), torch.nan_to_num(cache))
    with pytest.raises(ValueError, match='exact part alone needs k'):
        lib.call('hla_s6_decode_prepare', lib.ptr(qd), qd.stride(0), qd.stride(1), lib.ptr(Ad), Ad.stride(0),
                 Ad.stride(1), lib.ptr(posd), lib.ptr(ltab), ltab.stride(0), ltab.shape[0], lib.ptr(q_lat2),
                 q_lat2.stride(0), q_lat2.stride(1), T, H, d, W, lib.ptr(q_rope2), q_rope2.stride(0),
                 q_rope2.stride(1), None, 0, 0, None, 0, 0, lib.ptr(cos_sin), cos_sin.stride(0), cos_sin.shape[0],
                 lib.ptr(logical2), nb, logical2.stride(0), logical2.stride(1), logical2.stride(2), page,
                 lib.ptr(btd), btd.stride(0), btd.shape[1], lib.ptr(qsl), R, None, lib.PREPARE_EXACT_ONLY,
                 lib.stream_of(qd))


def test_probe_latent_rope_checks_the_b200_kernel():
    """The start-up probe the adapter runs (s6_ops.py:44-58, ouro_latent.py:203) answers for the B200
    kernel: the head stride is honoured (flat False) and the rotation is bit-exact with the torch formula."""
    lay = pkg('s6_layer')
    inv = lay.latent_inv_freq(128, 1e6)
    for w in (512, 256):
        table = lay.latent_rope_table(4096, inv, w, BF16).to(CUDA)
        assert ops().probe_latent_rope(table, 16) == (False, True)
        assert ops().probe_latent_rope(table) == (False, True)


@pytest.mark.parametrize('T', [200, 300])
def test_writer_epilogue_access_width_does_not_change_results(T):
    """Rows that are 32-byte aligned take the epilogue's 256-bit loads and stores; rows that are only
    16-byte aligned (here: every buffer offset by 8 elements, strides 8 elements past a multiple of
    16) take two 128-bit accesses.  Both write the same register and committed rows, bit for bit."""
    rng = np.random.default_rng(T + 101)
    K, page, max_pos, w = 256, 16, 4096, 512
    N = 2 * w
    lib = pkg('_lib')
    h = dev(orc.bf16(rng.standard_normal((T, K), dtype=np.float32)), BF16)
    E = dev(orc.bf16(rng.standard_normal((N, K), dtype=np.float32) / 16), BF16)
    reg_np = orc.bf16(rng.standard_normal((T, N), dtype=np.float32))
    R = T - 3
    qsl = torch.tensor(list(range(R + 1)), dtype=I32, device=CUDA)
    pos = torch.from_numpy(rng.integers(0, 2 * page, T)).to(CUDA)
    nb = 2 * R + 2
    bt = (torch.randperm(nb - 1, device=CUDA).to(I32)[:2 * R] + 1).view(R, 2)
    inv = layer().latent_inv_freq(128, 1e6)
    table = layer().latent_rope_table(max_pos, inv, w, BF16).to(CUDA)
    st = lib.stream_of(h)

    def run(pad):
        reg_in = torch.zeros(T, N + pad, dtype=BF16, device=CUDA)[:, pad:]
        reg_in.copy_(dev(reg_np, BF16))
        reg_out = torch.full((T, N + pad), float('nan'), dtype=BF16, device=CUDA)[:, pad:]
        cache = torch.full((nb, 1, page, N + pad), float('nan'), dtype=BF16, device=CUDA)[..., pad:]
        lib.call('hla_s6_writer_project', lib.ptr(h), h.stride(0), lib.ptr(E), E.stride(0), lib.ptr(reg_in),
                 reg_in.stride(0), lib.ptr(reg_out), reg_out.stride(0), T, N, K, st)
        lib.call('hla_s6_writer_commit', lib.ptr(h), h.stride(0), lib.ptr(E), E.stride(0), lib.ptr(reg_in),
                 reg_in.stride(0), None, 0, T, N, K, lib.ptr(pos), lib.ptr(table), table.stride(0), table.shape[0],
                 lib.ptr(cache), nb, cache.stride(0), cache.stride(2), page, lib.ptr(bt), bt.stride(0), bt.shape[1],
                 lib.ptr(qsl), R, st)
        torch.cuda.synchronize()
        return reg_out.float().cpu().numpy(), cache.float().cpu().numpy()

    reg32, cache32 = run(0)
    reg16, cache16 = run(8)
    assert not np.isnan(reg32).any()
    np.testing.assert_array_equal(reg16, reg32)
    np.testing.assert_array_equal(np.isnan(cache16), np.isnan(cache32))
    np.testing.assert_array_equal(np.nan_to_num(cache16), np.nan_to_num(cache32))
