"""Contiguous-layout reader of the HF engines (fused_history.history_attention, reference
hla/latent/fused_history.py:49-54 / history_kernels.py:11-33) on the B200 kernel: against the
reference's own outputs (golden fixtures) and the oracle at larger sizes.  GPU, except the
argument-contract tests."""
import math

import numpy as np
import pytest
import torch

import cases
from conftest import GOLDEN, pkg
from oracle import s6_oracle as orc

CUDA, BF16 = 'cuda', torch.bfloat16
O_TOL = dict(atol=2e-2, rtol=1e-2)
LSE_ATOL = 1e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


@pytest.mark.gpu
@pytest.mark.parametrize('name,kw', [('contig_512', dict(width=512)),
                                     ('contig_256', dict(seed=82, width=256, keys=37, batch=4))])
def test_matches_reference_fixture(name, kw):
    c = cases.contig_case(**kw)
    g = np.load(GOLDEN / f'{name}.npz')
    assert str(g['input_sha256']) == cases.digest(c)
    fh = pkg('fused_history')
    z, lse = fh.history_attention(dev(c['q'], BF16), dev(c['k'], BF16), dev(c['v'], BF16), dev(c['mask']).bool(),
                                  float(g['scale']))
    assert z.dtype == BF16 and z.shape == c['q'].shape and lse.shape == c['q'].shape[:2]
    z, lse = z.float().cpu().numpy(), lse.cpu().numpy()
    np.testing.assert_allclose(z, g['z'], **O_TOL)
    np.testing.assert_allclose(lse, g['lse'], atol=LSE_ATOL, rtol=0)
    assert (z[1] == 0).all() and (lse[1] == -np.inf).all()       # the fully masked row


@pytest.mark.gpu
@pytest.mark.parametrize('B,N,R,pattern', [(3, 1000, 512, 'random'), (2, 2050, 512, 'prefix'),
                                           (64, 300, 256, 'random'), (5, 17, 512, 'sparse'),
                                           (4, 4096, 1024, 'random')])
def test_matches_oracle(B, N, R, pattern):
    rng = np.random.default_rng(B * N + R)
    H = 16
    q = orc.bf16(rng.standard_normal((B, H, R), dtype=np.float32))
    k = orc.bf16(rng.standard_normal((B, N, R), dtype=np.float32))
    v = orc.bf16(rng.standard_normal((B, N, R), dtype=np.float32))
    if pattern == 'random':
        mask = rng.random((B, N)) < 0.7
    elif pattern == 'prefix':
        mask = np.arange(N)[None] < rng.integers(1, N + 1, (B, 1))
    else:
        mask = rng.random((B, N)) < 0.05
    mask[0, :] = False                                   # one empty row in every case
    scale = 1 / math.sqrt(128)
    z, lse, z32 = pkg('fused_history').forward(dev(q, BF16), dev(k, BF16), dev(v, BF16), dev(mask), scale)
    z_ref, lse_ref = orc.contiguous_history(q, k, v, mask, scale)
    np.testing.assert_allclose(z.float().cpu().numpy(), z_ref, **O_TOL)
    np.testing.assert_allclose(z32.cpu().numpy(), z_ref, **O_TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=LSE_ATOL, rtol=0)
    assert (z[0] == 0).all() and torch.isinf(lse[0]).all()


@pytest.mark.gpu
def test_all_rows_masked():
    B, N, H, R = 3, 40, 16, 512
    q = torch.randn(B, H, R, device=CUDA).to(BF16)
    k = torch.randn(B, N, R, device=CUDA).to(BF16)
    z, lse = pkg('fused_history').history_attention(q, k, k.clone(), torch.zeros(B, N, dtype=torch.bool,
                                                                                  device=CUDA), 0.1)
    assert (z == 0).all() and (lse == -float('inf')).all()


def test_argument_contract_follows_the_reference():
    fh = pkg('fused_history')
    q, k, m = torch.zeros(2, 16, 512), torch.zeros(2, 5, 512), torch.ones(2, 5, dtype=torch.bool)
    with pytest.raises(ValueError, match='Expected Q'):
        fh.history_attention(q, k, torch.zeros(2, 6, 512), m, 0.1)
    with pytest.raises(ValueError, match='Expected Q'):
        fh.history_attention(q, k, k, m[:, :4], 0.1)
    with pytest.raises(ValueError, match='storage row'):
        fh.forward(q, torch.zeros(2, 0, 512), torch.zeros(2, 0, 512), torch.ones(2, 0, dtype=torch.bool), 0.1)
    with pytest.raises(NotImplementedError):
        fh.history_attention(q.requires_grad_(), k, k, m, 0.1)
    with pytest.raises(RuntimeError, match='CUDA'):
        fh.forward(torch.zeros(2, 16, 512), k, k, m, 0.1)
