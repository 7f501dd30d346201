"""BASELINE config 1 on the B200 path: one layer x 4 loops of the S6 hybrid decode op for one sequence at
context 2048 (2016 latent rows, the W = 32 exact window and the current token, identity page tables)
against the reference's own fp32 outputs (tests/golden/config1.npz, from tests/golden/gen_golden.py):
the latent query, the history lse, and the fused decode attend (history split, then the combine's
reduce, B up-projection, exact window and merge).  Loop 0 reads the 256-wide loop-1 latent.  GPU."""
import numpy as np
import pytest
import torch

import cases
from conftest import GOLDEN, pkg

pytestmark = pytest.mark.gpu
CUDA, BF16 = 'cuda', torch.bfloat16
O_TOL = dict(atol=2e-2, rtol=1e-2)
LSE_ATOL = 1e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


class _Layer:
    def __init__(self, A, B, width):
        self.A, self.B, self.width = A, B, width

    def readers(self, loop):
        return self.A, self.B, self.width


@pytest.mark.parametrize('splits', [1, 16])
def test_config1_decode_op_matches_reference(splits):
    c = cases.config1_case()
    g = np.load(GOLDEN / 'config1.npz')
    assert str(g['input_sha256']) == cases.digest(c)
    ops, lay = pkg('s6_ops'), pkg('s6_layer')
    scale = float(g['scale'])
    inv = lay.latent_inv_freq(128, float(c['latent_theta']))
    tables = {w: lay.latent_rope_table(int(c['max_pos']), inv, w, BF16).to(CUDA) for w in (256, 512)}
    positions = dev(c['positions'])
    ws = ops.S6Workspace(16, 512, splits)
    ctx = lay.StepContext(positions, dev(c['query_start_loc']), dev(c['seq_lens']), 1, 1, tables, scale,
                          ops.B200_BACKENDS, ws, splits, window=int(c['window']))
    table = dev(c['table'])
    for t in range(4):
        w = 256 if t == 0 else 512
        A, B = dev(c[f'A{t}'], BF16), dev(c[f'B{t}'], BF16)
        q_lat = lay.latent_query(dev(c[f'q_pre{t}'], BF16), A, positions, tables[w], 'b200')
        np.testing.assert_allclose(q_lat.float().cpu().numpy(), g[f'q_lat{t}'], rtol=0, atol=1.6e-2)
        ql = dev(g[f'q_lat{t}'], BF16)   # the reference's q_lat (bf16 values) drives the rest
        cache = dev(c['lat_l1'] if t == 0 else c['lat_main'], BF16)
        _, lse = ops.history_attention(ql, cache, table, dev(c['ctx_lat']), scale, splits, ws, None, None, 'b200')
        np.testing.assert_allclose(lse.cpu().numpy(), g[f'lse_hist{t}'], atol=LSE_ATOL, rtol=0)
        ex = dev(c[f'exact{t}'], BF16)
        out = lay.attend(_Layer(A, B, w), t, ql, dev(c[f'q_rope{t}'], BF16), None, None, cache, table, None, None, ctx,
                         (ex.transpose(1, 2), table))
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, g[f'out{t}'], **O_TOL)
