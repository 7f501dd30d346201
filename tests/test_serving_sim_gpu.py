"""The adapter's per-layer code path over a simulated paged cache, step after step (GPU).

``ouro_attention.LatentAttention.forward`` mirrors OuroLatentAttention.forward (hla/vllm_latent/
ouro_latent.py:106-131); this Sim plays vLLM's part, as the reference's own serving test does
(hla/tests/test_s6_serving.py:16-102): paged latent and exact-window caches with shuffled block ids
(block 0 never used), per-request block tables with stale columns, vLLM-style varlen metadata with
padded requests and padding tokens, and a sequence of steps - a full-prompt prefill, decodes over a
window-and-latent history, two prefills in one batch, a decode batch (the fused CUDA-graph branch), an
interleaved prefill/decode batch, decodes crossing pages.  Four loops per step with the writer commits.

A CPU oracle keeps its own history of every request - the exact rows from its own RoPE, the latent rows
as the GPU committed them once they matched its writer - and checks, per step and loop: the attention
output of every valid token (the reference ops composed: chunk + window history + merge_lse, latent
history + B + merge_states), zero output on padding tokens, the O projection, and the committed rows -
values within the bf16 GEMM tolerance of the oracle's writer, placement exact (each token's slot, no
other slot touched).
"""
import math

import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu
CUDA, BF16, I32 = 'cuda', torch.bfloat16, torch.int32
H, D, HIDDEN, RANK, RANK1, LOOPS, W, PAGE = 16, 128, 2048, 512, 256, 4, 32, 16
NB, MAXB, THETA, MAXPOS = 48, 8, 1e6, 4096
O_TOL = dict(atol=2e-2, rtol=1e-2)
ROW_TOL = dict(atol=3e-2, rtol=1e-2)


class Sim:
    def __init__(self, seed=0):
        lat_mod, lay, oa = pkg('latent'), pkg('s6_layer'), pkg('ouro_attention')
        g = torch.Generator(device=CUDA).manual_seed(seed)
        rnd = lambda *shape, std: (torch.randn(*shape, generator=g, device=CUDA) * std).to(BF16)
        sl = lat_mod.LatentLayer(HIDDEN, H, D, LOOPS, RANK, RANK, RANK1).to(CUDA, BF16).requires_grad_(False)
        with torch.no_grad():
            for p_ in (sl.q_absorb, sl.q_absorb1):
                p_.copy_(rnd(*p_.shape, std=D ** -0.5))
            sl.out_absorb.copy_(rnd(*sl.out_absorb.shape, std=RANK ** -0.5))
            sl.out_absorb1.copy_(rnd(*sl.out_absorb1.shape, std=RANK1 ** -0.5))
            for lin in (*sl.cand_s, sl.cand1):
                lin.weight.copy_(rnd(*lin.weight.shape, std=HIDDEN ** -0.5))
        self.sl = sl
        self.wqkv = rnd(3 * H * D, HIDDEN, std=HIDDEN ** -0.5)
        self.wo = rnd(HIDDEN, H * D, std=(H * D) ** -0.5)
        inv = lay.latent_inv_freq(D, THETA)
        self.tables = {w: lay.latent_rope_table(MAXPOS, inv, w, BF16).to(CUDA) for w in (RANK, RANK1)}
        ang = torch.arange(MAXPOS).float()[:, None] * inv[None]
        cos_sin = torch.cat((ang.cos(), ang.sin()), -1).to(CUDA)
        self.attn = oa.LatentAttention(sl, self.wqkv, self.wo, cos_sin, W)
        nan = float('nan')
        self.caches = oa.PagedCaches(
            main=torch.full((NB, 1, PAGE, 2 * RANK), nan, dtype=BF16, device=CUDA),
            l1=torch.full((NB, 1, PAGE, 2 * RANK1), nan, dtype=BF16, device=CUDA),
            latent_table=None,
            exact=[torch.full((NB, PAGE, H, 2 * D), nan, dtype=BF16, device=CUDA) for _ in range(LOOPS)],
            exact_table=None)
        rng = np.random.default_rng(seed)
        self.rng = rng
        self.free_lat = (rng.permutation(NB - 1) + 1).tolist()
        self.free_ex = (rng.permutation(NB - 1) + 1).tolist()
        self.blocks_lat, self.blocks_ex = {}, {}
        # the oracle's history per request: committed latent rows, and exact rows per loop
        self.hist_main, self.hist_l1, self.hist_ex = {}, {}, {}
        self.tab_np = {w: self.tables[w].float().cpu().numpy() for w in (RANK, RANK1)}
        self.E = [sl.writer(t).float().cpu().numpy() for t in range(LOOPS)]
        self.A = [sl.readers(t)[0].float().cpu().numpy() for t in range(LOOPS)]
        self.B = [sl.readers(t)[1].float().cpu().numpy() for t in range(LOOPS)]
        self.written = {name: set() for name in ('main', 'l1')}
        self.steps = 0

    def run_step(self, requests, padded_requests=0, padding_tokens=0):
        ops, lay = pkg('s6_ops'), pkg('s6_layer')
        lengths = [(rid, n, len(self.hist_main.get(rid, []))) for rid, n in requests]
        real = sum(n for _, n, _ in lengths)
        T, R = real + padding_tokens, len(requests) + padded_requests
        starts = np.concatenate(([0], np.cumsum([n for _, n, _ in lengths]))).astype(np.int64)
        qsl = np.concatenate((starts, [real] * padded_requests)).astype(np.int32)
        seq_lens = np.array([c + n for _, n, c in lengths] + [0] * padded_requests, dtype=np.int32)
        positions = np.concatenate([np.arange(c, c + n) for _, n, c in lengths] +
                                   [np.ones(padding_tokens, dtype=np.int64)]).astype(np.int64)
        # per-request tables; stale columns point at live blocks (only ceil(len / page) columns are read)
        tl = self.rng.integers(1, NB, (R, MAXB)).astype(np.int32)
        te = self.rng.integers(1, NB, (R, MAXB)).astype(np.int32)
        tl[len(requests):] = 0
        te[len(requests):] = 0
        for r, (rid, n, c) in enumerate(lengths):
            for blocks, free, tab in ((self.blocks_lat, self.free_lat, tl), (self.blocks_ex, self.free_ex, te)):
                b = blocks.setdefault(rid, [])
                while len(b) * PAGE < c + n:
                    b.append(free.pop())
                tab[r, :len(b)] = b
        self.caches.latent_table = torch.from_numpy(tl).to(CUDA)
        self.caches.exact_table = torch.from_numpy(te).to(CUDA)
        max_q = max(n for _, n, _ in lengths)
        splits = 4
        ws = ops.S6Workspace(H, RANK, max(T, 1) * splits)
        ctx = lay.StepContext(torch.from_numpy(positions).to(CUDA), torch.from_numpy(qsl).to(CUDA),
                              torch.from_numpy(seq_lens).to(CUDA), max_q, T, self.tables, D ** -0.5,
                              ops.B200_BACKENDS, ws, splits, window=W)
        req, valid = orc.token_requests(qsl, T)
        hist = np.array([c for _, _, c in lengths] + [0] * padded_requests)
        ctx_np = np.where(valid, hist[req], 0)
        assert ctx.ctx.tolist() == ctx_np.tolist() and ctx.valid.tolist() == valid.tolist()
        lat_slots = np.where(valid, tl[req, positions // PAGE].astype(np.int64) * PAGE + positions % PAGE, -1)
        state = None
        reg, first = None, None
        new_ex = [[] for _ in range(LOOPS)]
        for loop in range(LOOPS):
            gen = torch.Generator(device=CUDA).manual_seed(100 * self.steps + loop)
            hidden = torch.randn(T, HIDDEN, generator=gen, device=CUDA).to(BF16)
            qkv = torch.nn.functional.linear(hidden, self.wqkv)          # the same cuBLAS product forward makes
            q_pre, k_pre, v = (x.view(T, H, D).float().cpu().numpy() for x in qkv.split(H * D, -1))
            out_dev, state, attn = self.attn.forward(ctx.positions, hidden, loop, state, ctx, self.caches,
                                                     return_attention=True)
            torch.cuda.synchronize()
            h = hidden.float().cpu().numpy()
            # ---- oracle: writer, exact RoPE, latent query, attention over its own history
            if loop == 0:
                first = orc.write_update(h, self.E[0])
            else:
                reg = orc.write_step(reg, orc.write_update(h, self.E[loop]))
            width = RANK1 if loop == 0 else RANK
            q_rope = orc.bf16(orc.neox_rope(q_pre, positions, D, THETA).astype(np.float32))
            k_rope = orc.bf16(orc.neox_rope(k_pre, positions, D, THETA).astype(np.float32))
            # the reference's bf16 model: einsum rounded to bf16, then latent RoPE in the torch bf16 order
            absorbed = orc.bf16(np.einsum('thd,hdr->thr', q_pre, self.A[loop]).astype(np.float32))
            q_lat = orc.latent_rope(absorbed, positions, self.tab_np[width], emulate_bf16=True)
            ref = self._oracle_attention(loop, width, lengths, starts, qsl, T, valid, ctx_np, q_lat, q_rope, k_rope, v)
            got = attn.float().cpu().numpy()
            assert np.isfinite(got).all() and (got[~valid] == 0).all()
            np.testing.assert_allclose(got[valid], ref[valid], **O_TOL)
            out_ref = attn.reshape(T, H * D).float() @ self.wo.float().t()
            torch.testing.assert_close(out_dev.float(), out_ref, atol=3e-2, rtol=2e-2)
            for r, (rid, n, c) in enumerate(lengths):
                s = int(starts[r])
                rows = np.concatenate((k_rope[s:s + n], v[s:s + n]), -1)      # [n, H, 2d]
                new_ex[loop].append((rid, rows))
            # ---- commits at loops 0 and 3: placement exact, values within the writer tolerance
            if loop in (0, LOOPS - 1):
                name = 'l1' if loop == 0 else 'main'
                row = orc.committed_row(first if loop == 0 else reg, width, positions, self.tab_np[width])
                cache = self.caches.l1 if loop == 0 else self.caches.main
                flat = cache.view(-1, 2 * width).float().cpu().numpy()
                sl_valid = lat_slots[valid]
                np.testing.assert_allclose(flat[sl_valid], row[valid], **ROW_TOL)
                self.written[name] |= set(sl_valid.tolist())
                untouched = np.ones(flat.shape[0], dtype=bool)
                untouched[list(self.written[name])] = False
                assert np.isnan(flat[untouched]).all()
                for r, (rid, n, c) in enumerate(lengths):
                    s = int(starts[r])
                    hist_rows = flat[lat_slots[s:s + n]]            # the rows the GPU committed feed later steps
                    store = self.hist_l1 if loop == 0 else self.hist_main
                    store.setdefault(rid, []).extend(list(hist_rows))
        for loop in range(LOOPS):
            for rid, rows in new_ex[loop]:
                self.hist_ex.setdefault((rid, loop), []).extend(list(rows))
        self.steps += 1
        return ctx

    def _oracle_attention(self, loop, width, lengths, starts, qsl, T, valid, ctx_np, q_lat, q_rope, k_rope, v):
        """chunk + window history (merge_lse), latent history + B, merge_states (s6_layer.py:87-115)."""
        scale = D ** -0.5
        o_c, lse_c = orc.chunk_attention(q_rope, k_rope, v, qsl, ~valid, scale)
        # paged views of the oracle's own history: one page run per request, identity tables
        R = len(lengths)
        pages = max(1, max(-(-c // PAGE) for _, _, c in lengths))
        lat = np.zeros((1 + R * pages, 1, PAGE, 2 * width), dtype=np.float64)
        ex = np.zeros((1 + R * pages, H, PAGE, 2 * D), dtype=np.float64)
        tab = np.zeros((T, pages), dtype=np.int32)
        for r, (rid, n, c) in enumerate(lengths):
            ids = 1 + r * pages + np.arange(pages)
            if c:
                rows = np.stack((self.hist_l1 if loop == 0 else self.hist_main)[rid][:c])
                ex_rows = np.stack(self.hist_ex[(rid, loop)][:c])
                for j in range(c):
                    lat[ids[j // PAGE], 0, j % PAGE] = rows[j]
                    ex[ids[j // PAGE], :, j % PAGE] = ex_rows[j]
            s = int(starts[r])
            tab[s:s + n] = ids
        o_w, lse_w = orc.window_attention(q_rope, ex, tab, ctx_np, W, scale)
        o_c, lse_c = orc.merge_lse(o_c, lse_c, o_w, lse_w)
        o_h, lse_h = orc.history_attention(q_lat, lat, tab, np.maximum(ctx_np - W, 0), scale)
        # bf16 tensors between the reference's ops: history output, B einsum output, exact part
        o_h = orc.bf16(np.einsum('thr,hrd->thd', orc.bf16(o_h.astype(np.float32)), self.B[loop]).astype(np.float32))
        return orc.merge_states(o_h, lse_h, orc.bf16(o_c.astype(np.float32)), lse_c, ~valid)


def test_prefill_decode_page_crossing_mixed_and_padding_match_oracle():
    sim = Sim(3)
    sim.run_step([(0, 40)])                                  # full-prompt prefill, empty history
    sim.run_step([(0, 1)])                                   # decode over 40 rows: window 32 + 8 latent rows
    sim.run_step([(1, 33), (2, 50)])                         # two prefills in one batch
    ctx = sim.run_step([(0, 1), (1, 1), (2, 1)], padded_requests=1, padding_tokens=2)   # fused decode branch
    assert ctx.max_query_len == 1 and ctx.valid.tolist() == [True] * 3 + [False] * 2
    sim.run_step([(1, 17), (3, 5), (0, 1)])                  # interleaved prefill / decode
    ctx = sim.run_step([(3, 1), (2, 1), (0, 1)], padding_tokens=1)   # decodes, pages crossed
    assert ctx.ctx.tolist() == [5, 51, 43, 0]
    assert {rid: len(rows) for rid, rows in sim.hist_main.items()} == {0: 44, 1: 51, 2: 52, 3: 6}
