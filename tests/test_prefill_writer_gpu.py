"""The config-3 prompt-step writer (PrefillWriter, 4 loops per layer through the tcgen05 writer) against
the oracle: every token's committed main and loop-1 rows at its vLLM slot (reference s6_layer.py:124-147,
register.py:45-79), nothing else written.  GPU."""
import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('prompts,prompt_len', [(2, 300), (3, 1000)])
def test_prefill_writer_rows_match_oracle(prompts, prompt_len):
    dec, pre = pkg('decode'), pkg('prefill')
    shape = dec.OuroShape(layers=2, max_position=4096)
    m = pre.PrefillWriter(shape, prompts, prompt_len, device='cuda', seed=3)
    m.step()
    torch.cuda.synchronize()
    pos = m.positions.cpu().numpy()
    req = np.repeat(np.arange(prompts), prompt_len)
    bt = m.block_table.cpu().numpy()
    slots = bt[req, pos // shape.page].astype(np.int64) * shape.page + pos % shape.page
    h = [m.h[t].float().cpu().numpy() for t in range(shape.loops)]
    for layer in range(shape.layers):
        lat = m.layers[layer]
        E = [lat.writer(t).float().cpu().numpy() for t in range(shape.loops)]
        first = orc.write_update(h[0], E[0])
        reg = None
        for t in range(1, shape.loops):
            reg = orc.write_step(reg, orc.write_update(h[t], E[t]))
        for cache, row, width in ((m.l1[layer], first, shape.rank1), (m.main[layer], reg, shape.rank)):
            table = m.tables[width].float().cpu().numpy()
            expect = orc.committed_row(row, width, pos, table)
            flat = cache.view(-1, 2 * width).float().cpu().numpy()
            # bf16 GEMM tolerance (fp32 tensor-core accumulation vs one rounding of the exact product)
            np.testing.assert_allclose(flat[slots], expect, atol=3e-2, rtol=1e-2)
            rest = np.ones(flat.shape[0], dtype=bool)
            rest[slots] = False
            assert np.isinf(flat[rest]).all()


def test_prefill_writer_graph_replay_is_deterministic():
    dec, pre = pkg('decode'), pkg('prefill')
    m = pre.PrefillWriter(dec.OuroShape(layers=2, max_position=4096), 2, 512, device='cuda', seed=5)
    m.step()
    torch.cuda.synchronize()
    before = [c.clone() for c in (*m.main, *m.l1)]
    g = m.capture()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(before, (*m.main, *m.l1)):
        assert torch.equal(a, b)


def test_pipelined_host_io_step_matches_copy_step_copy():
    """PrefillWriter.step_io (each loop's hidden states copied in on a copy stream, the launches of a loop
    waiting only for their own copy, one cache read back at the end) gives exactly h <- host_in; step();
    host_out <- cache - eagerly and as a replayed graph with new host inputs."""
    dec, pre = pkg('decode'), pkg('prefill')
    shape = dec.OuroShape(layers=2, max_position=4096)
    piped = pre.PrefillWriter(shape, 2, 300, device='cuda', seed=4)
    plain = pre.PrefillWriter(shape, 2, 300, device='cuda', seed=4)
    g = torch.Generator().manual_seed(5)
    host_in = torch.empty(piped.h.shape, dtype=piped.h.dtype, pin_memory=True)
    host_out = torch.empty(piped.main[-1].shape, dtype=piped.main[-1].dtype, pin_memory=True)

    def check():
        plain.h.copy_(host_in)
        plain.step()
        torch.cuda.synchronize()
        assert torch.equal(host_out, plain.main[-1].cpu())
        assert torch.equal(piped.l1[0], plain.l1[0])

    host_in.copy_(torch.randn(host_in.shape, generator=g).to(host_in.dtype))
    piped.step_io(host_in, host_out, piped.main[-1])
    torch.cuda.synchronize()
    check()
    graph = piped.capture_io(host_in, host_out, piped.main[-1])
    for _ in range(2):
        host_in.copy_(torch.randn(host_in.shape, generator=g).to(host_in.dtype))
        host_out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        check()
