"""A3: the integer step metadata of StepContext on the GPU, bit-exact with the reference.

``tests/golden/step_context.json`` holds the reference's own StepContext fields (s6_layer.py:52-77:
token_requests, valid, invalid, ctx, ctx_latent, empty, empty_latent, and block_table(table)) for
decode, padded, prefill, mixed and window-0 steps; ``meta.json`` its token_requests /
history_lengths on the cases of its op tests (test_s6_ops.py:16-27, 51-53).  The b200 path computes
them with one metadata launch and one gather per table; every value must match exactly.
"""
import json

import pytest
import torch

import cases
from conftest import GOLDEN, pkg

pytestmark = pytest.mark.gpu
CUDA = 'cuda'


def test_step_context_fields_match_reference_exactly():
    lay, ops = pkg('s6_layer'), pkg('s6_ops')
    ref = json.loads((GOLDEN / 'step_context.json').read_text())
    for (qsl, seq_lens, T, window, table), want in zip(cases.step_context_cases(), ref):
        ctx = lay.StepContext(torch.zeros(T, dtype=torch.int64, device=CUDA),
                              torch.tensor(qsl, dtype=torch.int32, device=CUDA),
                              torch.tensor(seq_lens, dtype=torch.int32, device=CUDA), 1, T, {}, 1.0,
                              ops.B200_BACKENDS, window=window)
        got = dict(token_requests=ctx.token_requests, valid=ctx.valid, invalid=ctx.invalid, ctx=ctx.ctx,
                   ctx_latent=ctx.ctx_latent, empty=ctx.empty, empty_latent=ctx.empty_latent)
        for name, value in got.items():
            assert value.is_cuda and value.tolist() == want[name], (name, qsl, seq_lens, window)
        assert str(ctx.ctx.dtype) == want['ctx_dtype'] and str(ctx.ctx_latent.dtype) == want['ctx_latent_dtype']
        assert ctx.token_requests.dtype == torch.int64 and ctx.valid.dtype == torch.bool
        bt = ctx.block_table(torch.tensor(table, dtype=torch.int32, device=CUDA))
        assert bt.dtype == torch.int32 and bt.tolist() == want['block_table']
        # a strided (column-sliced) table gathers through the scalar path
        wide = torch.zeros(len(table), len(table[0]) + 3, dtype=torch.int32, device=CUDA)
        wide[:, :len(table[0])] = torch.tensor(table, dtype=torch.int32)
        assert ops.gather_block_table(wide[:, :len(table[0])], ctx.token_requests).tolist() == want['block_table']


def test_token_requests_and_history_lengths_match_reference():
    ops = pkg('s6_ops')
    meta = json.loads((GOLDEN / 'meta.json').read_text())
    mc = cases.meta_cases()
    for (qsl, n), (req, valid) in zip(mc['token_requests'], meta['reference']['token_requests']):
        r, v = ops.token_requests(torch.tensor(qsl, dtype=torch.int32, device=CUDA), n)
        assert r.dtype == torch.int64 and r.tolist() == req and v.tolist() == valid
    for (a, b), want in zip(mc['history_lengths'], meta['reference']['history_lengths']):
        got = ops.history_lengths(torch.tensor(a, dtype=torch.int32, device=CUDA),
                                  torch.tensor(b, dtype=torch.int32, device=CUDA))
        assert got.dtype == torch.int32 and got.tolist() == want


def test_metadata_survives_graph_replay_with_new_contents():
    """Captured once, replayed with new query_start_loc / seq_lens contents (FULL_DECODE_ONLY
    graphs keep the shapes and change the values)."""
    lay, ops = pkg('s6_layer'), pkg('s6_ops')
    ref = json.loads((GOLDEN / 'step_context.json').read_text())
    c = cases.step_context_cases()
    (qa, sa, T, wa, _), (qb, sb, Tb, wb, _) = c[0], c[5]
    assert len(qa) == len(qb) and T == 4 and Tb == 5 and wa == 32
    qsl = torch.tensor(qa, dtype=torch.int32, device=CUDA)
    sl = torch.tensor(sa, dtype=torch.int32, device=CUDA)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        lay.StepContext(torch.zeros(T, dtype=torch.int64, device=CUDA), qsl, sl, 1, T, {}, 1.0, ops.B200_BACKENDS,
                        window=32)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ctx = lay.StepContext(torch.zeros(T, dtype=torch.int64, device=CUDA), qsl, sl, 1, T, {}, 1.0,
                              ops.B200_BACKENDS, window=32)
    g.replay()
    torch.cuda.synchronize()
    assert ctx.ctx.tolist() == ref[0]['ctx'] and ctx.ctx_latent.tolist() == ref[0]['ctx_latent']
    # new contents, same shapes: [0, 2, 3, 3, 3] / [4, 7, 0, 0] over the first 4 tokens, window 32
    qsl.copy_(torch.tensor(qb, dtype=torch.int32))
    sl.copy_(torch.tensor(sb, dtype=torch.int32))
    g.replay()
    torch.cuda.synchronize()
    assert ctx.token_requests.tolist() == [0, 0, 1, 3]
    assert ctx.valid.tolist() == [True, True, True, False]
    assert ctx.ctx.tolist() == [2, 2, 6, 0] and ctx.ctx_latent.tolist() == [0, 0, 0, 0]


def test_one_row_table_with_any_stride():
    """A one-request table built from a broadcast numpy array can carry row stride 0 (torch keeps it for a
    size-1 dim): the gather must not care about the stride of a single row."""
    import numpy as np
    ops = pkg('s6_ops')
    row = np.arange(129, dtype=np.int32)
    table = torch.from_numpy(np.broadcast_to(row, (1, 129)).copy()).as_strided((1, 129), (0, 1)).to(CUDA)
    req = torch.zeros(3, dtype=torch.int64, device=CUDA)
    out = ops.gather_block_table(table, req)
    assert out.tolist() == [row.tolist()] * 3
