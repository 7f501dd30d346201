"""Prefill / mixed steps (the non-fused branch of s6_layer.attend, reference s6_layer.py:101-115):
causal chunk attention, per-token window history, and the full attend against the oracle composed
from the reference's ops.  GPU."""
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
SCALE = 1 / math.sqrt(128)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


def golden(name, inputs):
    g = np.load(GOLDEN / f'{name}.npz')
    assert str(g['input_sha256']) == cases.digest(inputs)
    return g


def test_chunk_attention_matches_reference_fixture():
    c = cases.chunk_case()
    g = golden('chunk', c)
    ops = pkg('s6_ops')
    qsl = dev(c['query_start_loc'])
    T = int(c['num_tokens'])
    _, valid = ops.token_requests(qsl, T)
    o, lse = ops.chunk_attention(dev(c['q'], BF16), dev(c['k'], BF16), dev(c['v'], BF16), qsl, 41, ~valid, SCALE,
                                 'b200')
    o, lse, valid = o.float().cpu().numpy(), lse.cpu().numpy(), valid.cpu().numpy()
    np.testing.assert_allclose(o[valid], g['o'][valid], **O_TOL)
    np.testing.assert_allclose(lse[:, valid], g['lse'][:, valid], atol=LSE_ATOL, rtol=0)
    assert (o[~valid] == 0).all() and (lse[:, ~valid] == -np.inf).all()


@pytest.mark.parametrize('qsl', [(0, 300), (0, 64, 65, 200, 257, 257), (0, 1, 2, 3, 70, 130),
                                 tuple(range(34))])      # the last: uniform decode, one token per request
def test_chunk_attention_long_and_ragged_chunks(qsl):
    rng = np.random.default_rng(len(qsl))
    T = qsl[-1] + 5
    q, k, v = (orc.bf16(rng.standard_normal((T, 16, 128), dtype=np.float32)) for _ in range(3))
    invalid = np.arange(T) >= qsl[-1]
    ops = pkg('s6_ops')
    o, lse = ops.chunk_attention(dev(q, BF16), dev(k, BF16), dev(v, BF16), dev(np.asarray(qsl, np.int32)), 0,
                                 dev(invalid), SCALE, 'b200')
    o_ref, lse_ref = orc.chunk_attention(q, k, v, np.asarray(qsl), invalid, SCALE)
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, **O_TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=LSE_ATOL, rtol=0)


def test_window_history_matches_reference_fixture():
    wh = cases.window_history_case()
    g = golden('window_history', wh)
    ops = pkg('s6_ops')
    ctx = dev(wh['ctx'])
    o, lse = ops.window_history_fa(dev(wh['q'], BF16), dev(wh['cache_phys'], BF16).transpose(1, 2),
                                   dev(wh['block_table']), ctx, int(wh['window']), SCALE, 0, ctx == 0)
    np.testing.assert_allclose(o.float().cpu().numpy(), g['o'], **O_TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), g['lse'], atol=LSE_ATOL, rtol=0)


class _SL:
    def __init__(self, B, width):
        self.B, self.width = B, width

    def readers(self, loop):
        return None, self.B, self.width


def mixed_step(seed, width, requests, padding, window):
    """requests: (history length c, chunk length n).  Latent cache holds rows [0, c - window) of each
    request's history, the exact cache rows [0, c); the chunk's own k/v are passed directly."""
    rng = np.random.default_rng(seed)
    H, d, page = 16, 128, 16
    R = len(requests)
    starts = np.concatenate(([0], np.cumsum([n for _, n in requests])))
    T = int(starts[-1]) + padding
    qsl = starts.astype(np.int32)
    seq_lens = np.array([c + n for c, n in requests], dtype=np.int32)
    maxp = max(1, max(-(-(c + n) // page) for c, n in requests))
    nb = R * maxp + 1
    lat = orc.bf16(rng.standard_normal((nb, 1, page, 2 * width), dtype=np.float32))
    ex = orc.bf16(rng.standard_normal((nb, page, H, 2 * d), dtype=np.float32))
    lat[0] = np.inf
    ex[0] = np.inf
    table = np.zeros((R, maxp), dtype=np.int32)
    perm = rng.permutation(np.arange(1, nb))
    table[:] = perm[:R * maxp].reshape(R, maxp)
    q_lat = orc.bf16(rng.standard_normal((T, H, width), dtype=np.float32))
    q_rope, k_rope, v = (orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32)) for _ in range(3))
    B = orc.bf16(rng.standard_normal((H, width, d), dtype=np.float32) / math.sqrt(width))
    req, valid = orc.token_requests(qsl, T)
    hist = np.array([c for c, _ in requests])
    ctx = np.where(valid, hist[req], 0)
    ctx_lat = np.maximum(ctx - window, 0)
    tok_table = table[req]
    # oracle: the reference's non-fused branch
    o_c, lse_c = orc.chunk_attention(q_rope, k_rope, v, qsl, ~valid, SCALE)
    if window:
        o_w, lse_w = orc.window_attention(q_rope, ex.transpose(0, 2, 1, 3), tok_table, ctx, window, SCALE)
        o_c, lse_c = orc.merge_lse(o_c, lse_c, o_w, lse_w)
    o_h, lse_h = orc.history_attention(q_lat, lat, tok_table, ctx_lat, SCALE)
    o_h = np.einsum('thr,hrd->thd', o_h, B)
    ref = orc.merge_states(o_h, lse_h, o_c, lse_c, ~valid)
    return dict(T=T, qsl=qsl, seq_lens=seq_lens, lat=lat, ex=ex, table=table, q_lat=q_lat, q_rope=q_rope,
                k_rope=k_rope, v=v, B=B, ref=ref, valid=valid, maxq=max(n for _, n in requests), width=width)


@pytest.mark.parametrize('window', [32, 0])
@pytest.mark.parametrize('width', [512, 256])
def test_mixed_prefill_decode_attend_matches_oracle(window, width):
    s = mixed_step(window + width, width, [(0, 37), (100, 1), (50, 12), (0, 0), (300, 70), (5, 3)], 3, window)
    ops, lay = pkg('s6_ops'), pkg('s6_layer')
    T = s['T']
    ws = ops.S6Workspace(16, width, T * 4)
    ctx = lay.StepContext(torch.zeros(T, dtype=torch.int64, device=CUDA), dev(s['qsl']), dev(s['seq_lens']),
                          s['maxq'], T, {}, SCALE, ops.B200_BACKENDS, ws, 4, window=window)
    ex = dev(s['ex'], BF16).transpose(1, 2)
    win = (ex, dev(s['table'])) if window else None
    out = lay.attend(_SL(dev(s['B'], BF16), width), 1, dev(s['q_lat'], BF16), dev(s['q_rope'], BF16),
                     dev(s['k_rope'], BF16), dev(s['v'], BF16), dev(s['lat'], BF16), dev(s['table']), None, None,
                     ctx, win)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all() and (got[~s['valid']] == 0).all()
    np.testing.assert_allclose(got, s['ref'], **O_TOL)


def test_prompt_only_step_skips_history():
    s = mixed_step(5, 512, [(0, 20), (0, 9)], 1, 32)
    ops, lay = pkg('s6_ops'), pkg('s6_layer')
    T = s['T']
    ctx = lay.StepContext(torch.zeros(T, dtype=torch.int64, device=CUDA), dev(s['qsl']), dev(s['seq_lens']),
                          s['maxq'], T, {}, SCALE, ops.B200_BACKENDS, ops.S6Workspace(16, 512, T), 1, window=32)
    ctx.history_needed = False
    out = lay.attend(_SL(dev(s['B'], BF16), 512), 1, dev(s['q_lat'], BF16), dev(s['q_rope'], BF16),
                     dev(s['k_rope'], BF16), dev(s['v'], BF16), dev(s['lat'], BF16), dev(s['table']), None, None,
                     ctx, (dev(s['ex'], BF16).transpose(1, 2), dev(s['table'])))
    o_ref, _ = orc.chunk_attention(s['q_rope'], s['k_rope'], s['v'], s['qsl'], ~s['valid'], SCALE)
    np.testing.assert_allclose(out.float().cpu().numpy(), o_ref, **O_TOL)
