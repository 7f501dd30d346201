"""Rollout cache export (s6-rollout-cache-v1, reference hla/vllm_latent/cache_export.py:160-188) on the
B200 gather kernel: rows bit-identical to the reference exporter's (golden fixture) and to the oracle
at full model size; out-of-cache blocks and short block lists raise; the payload round-trips."""
import numpy as np
import pytest
import torch

import cases
from conftest import GOLDEN, pkg
from oracle import s6_oracle as orc

CUDA, BF16 = 'cuda', torch.bfloat16


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(CUDA)
    return t.to(dtype) if dtype is not None else t


@pytest.mark.gpu
def test_rows_equal_reference_exporter():
    ec = cases.export_case()
    g = np.load(GOLDEN / 'export.npz')
    assert str(g['input_sha256']) == cases.digest(ec)
    L = ec['main'].shape[0]
    rows = pkg('cache_export').export_rows([dev(ec['main'][i], BF16) for i in range(L)],
                                           [dev(ec['l1'][i], BF16) for i in range(L)], ec['main_blocks'],
                                           ec['l1_blocks'], int(ec['length']), int(ec['block_size']))
    assert len(rows) == L and rows[0].shape == (1, int(ec['length']), 1536) and rows[0].device.type == 'cpu'
    np.testing.assert_array_equal(np.stack([r.float().numpy() for r in rows]), g['rows'])


@pytest.mark.gpu
def test_full_model_request_matches_oracle():
    rng = np.random.default_rng(5)
    L, bs, length = 24, 16, 8192 + 5
    need = -(-length // bs)
    nb = need + 7
    main = [torch.randn(nb, 1, bs, 1024, device=CUDA).to(BF16) for _ in range(L)]
    l1 = [torch.randn(nb, 1, bs, 512, device=CUDA).to(BF16) for _ in range(L)]
    mb, lb = rng.permutation(nb)[:need], rng.permutation(nb)[:need]
    rows = pkg('cache_export').export_rows(main, l1, torch.from_numpy(mb), torch.from_numpy(lb), length, bs)
    ref = orc.export_rows([m.float().cpu().numpy() for m in main], [x.float().cpu().numpy() for x in l1], mb, lb, bs,
                          length)
    for got, want in zip(rows, ref):
        np.testing.assert_array_equal(got.float().numpy(), want)


@pytest.mark.gpu
def test_bad_blocks_raise():
    ce = pkg('cache_export')
    main = [torch.zeros(4, 1, 16, 1024, device=CUDA, dtype=BF16)]
    l1 = [torch.zeros(4, 1, 16, 512, device=CUDA, dtype=BF16)]
    with pytest.raises(IndexError):
        ce.export_rows(main, l1, [0, 9], [0, 1], 20, 16)          # block 9 is outside the cache
    with pytest.raises(IndexError):
        ce.export_rows(main, l1, [0], [0, 1], 20, 16)             # one block cannot hold 20 positions
    with pytest.raises(RuntimeError, match='TRITON_ATTN'):
        ce.export_rows([torch.zeros(4, 16, 1024, device=CUDA, dtype=BF16)], l1, [0, 1], [0, 1], 20, 16)


@pytest.mark.gpu
def test_snapshot_payload_round_trip(tmp_path):
    ce = pkg('cache_export')
    main = [torch.randn(3, 1, 16, 1024, device=CUDA).to(BF16) for _ in range(2)]
    l1 = [torch.randn(3, 1, 16, 512, device=CUDA).to(BF16) for _ in range(2)]
    rows = ce.export_rows(main, l1, [2, 0], [1, 2], 20, 16)
    rec = ce.write_snapshot(tmp_path, 0, 3, 'req', dict(num_layers=2), [1, 2, 3], 20, torch.zeros(1, 1, 8), rows)
    data = torch.load(rec['path'], map_location='cpu', weights_only=True)
    assert data['schema'] == 's6-rollout-cache-v1' and data['version'] == 3 and data['request_id'] == 'req'
    assert data['length'] == 20 and data['prompt_ids'] == [1, 2, 3] and data['first_response_logits'].shape == (1, 1, 8)
    assert len(data['rows']) == 2 and all(torch.equal(a, b) for a, b in zip(data['rows'], rows))
    assert rec['bytes'] > 0 and not (tmp_path / '0.tmp').exists()
