"""One (layer, loop) of the fused decode branch of s6_layer.attend (history split + fused combine)
vs the oracle's composition of the reference ops and an independent joint softmax (GPU)."""
import math

import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu
CUDA, BF16, I32 = 'cuda', torch.bfloat16, torch.int32
O_TOL = dict(atol=2e-2, rtol=1e-2)


def build_step(seed, width, ctxs, padding=2, H=16, d=128, page=16, window=32):
    rng = np.random.default_rng(seed)
    ctxs = np.asarray(ctxs, dtype=np.int64)
    R = len(ctxs)
    T = R + padding
    seq_lens = (ctxs + 1).astype(np.int32)
    qsl = np.concatenate(([0], np.arange(1, R + 1))).astype(np.int32)
    ctx_lat = np.maximum(ctxs - window, 0)
    # latent cache: pages for [0, ctx] (the current row would be committed after attend)
    lpages = -(-seq_lens // page)
    lnb = int(lpages.sum()) + 2
    lat = orc.bf16(rng.standard_normal((lnb, 1, page, 2 * width), dtype=np.float32))
    lat[0] = np.inf
    ltab = np.zeros((R, int(lpages.max()) + 1), dtype=np.int32)
    perm = rng.permutation(np.arange(1, lnb))
    k = 0
    for r in range(R):
        ltab[r, :lpages[r]] = perm[k:k + lpages[r]]
        k += lpages[r]
    # exact cache: only the pages of the window + current token exist (sliding window); others -> null 0
    enb = int(sum(-(-seq_lens[r] // page) for r in range(R))) + 2
    ex = orc.bf16(rng.standard_normal((enb, page, H, 2 * d), dtype=np.float32))
    ex[0] = np.inf
    etab = np.zeros((R, int(lpages.max()) + 1), dtype=np.int32)
    perm = rng.permutation(np.arange(1, enb))
    k = 0
    for r in range(R):
        first = max(0, int(seq_lens[r]) - 1 - window)
        for col in range(first // page, -(-int(seq_lens[r]) // page)):
            etab[r, col] = perm[k]
            k += 1
    q_lat = orc.bf16(rng.standard_normal((T, H, width), dtype=np.float32))
    q_rope = orc.bf16(rng.standard_normal((T, H, d), dtype=np.float32))
    B = orc.bf16(rng.standard_normal((H, width, d), dtype=np.float32) / math.sqrt(width))
    invalid = np.arange(T) >= R
    return dict(q_lat=q_lat, q_rope=q_rope, lat=lat, ltab=ltab, ctx_lat=ctx_lat, ex=ex, etab=etab, qsl=qsl,
                seq_lens=seq_lens, B=B, invalid=invalid, R=R, T=T, window=window, width=width)


def oracle(s, scale):
    T, R = s['T'], s['R']
    ltab_tok = np.zeros((T, s['ltab'].shape[1]), dtype=np.int32)
    ltab_tok[:R] = s['ltab']
    ctx_lat = np.zeros(T, dtype=np.int64)
    ctx_lat[:R] = s['ctx_lat']
    ex_logical = s['ex'].transpose(0, 2, 1, 3)
    return orc.attend_decode(s['q_lat'], s['q_rope'], s['lat'], ltab_tok, ctx_lat, ex_logical, s['etab'], s['qsl'],
                             s['seq_lens'], s['window'], s['B'], scale, s['invalid'])


class _SL:
    def __init__(self, B, width):
        self.B, self.width = B, width

    def readers(self, loop):
        return None, self.B, self.width


def run(s, splits, scale):
    ops, lay = pkg('s6_ops'), pkg('s6_layer')
    T, R, width = s['T'], s['R'], s['width']
    dv = lambda a, dt=None: (lambda t: t.to(dt) if dt else t)(torch.from_numpy(np.ascontiguousarray(a)).to(CUDA))
    positions = torch.zeros(T, dtype=torch.int64, device=CUDA)
    ws = ops.S6Workspace(16, width, T * splits)
    ctx = lay.StepContext(positions, dv(s['qsl']), dv(s['seq_lens']), 1, T, {}, scale, ops.B200_BACKENDS, ws,
                          splits, window=s['window'])
    assert ctx.ctx_latent.tolist()[:R] == s['ctx_lat'].tolist()
    ex = dv(s['ex'], BF16)
    out = lay.attend(_SL(dv(s['B'], BF16), width), 1, dv(s['q_lat'], BF16), dv(s['q_rope'], BF16), None, None,
                     dv(s['lat'], BF16), dv(s['ltab']), None, None, ctx, (ex.transpose(1, 2), dv(s['etab'])))
    return out


@pytest.mark.parametrize('width', [512, 256])
@pytest.mark.parametrize('splits', [1, 16])
def test_fused_decode_attend_matches_oracle(width, splits):
    scale = 1 / math.sqrt(128)
    s = build_step(width + splits, width, [0, 1, 31, 32, 33, 40, 100, 1000, 16, 48])
    out = run(s, splits, scale)
    ref = oracle(s, scale)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all() and (got[s['R']:] == 0).all()
    np.testing.assert_allclose(got, ref, **O_TOL)


def test_fused_decode_attend_equals_joint_softmax_for_one_token():
    scale = 1 / math.sqrt(128)
    s = build_step(99, 512, [300], padding=0)
    out = run(s, 4, scale).float().cpu().numpy()[0]
    page = 16
    ctx = 300
    lat_rows = np.stack([s['lat'][s['ltab'][0, j // page], 0, j % page] for j in range(ctx - 32)])
    ex_rows = np.stack([s['ex'][s['etab'][0, j // page], j % page] for j in range(ctx - 32, ctx + 1)])
    joint = orc.joint_decode(s['q_lat'][0], s['q_rope'][0], lat_rows, ex_rows, s['B'], scale)
    np.testing.assert_allclose(out, joint, **O_TOL)
