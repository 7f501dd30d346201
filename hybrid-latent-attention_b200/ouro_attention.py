"""One layer's attention of the S6 serving adapter on the B200 kernels, without vLLM.

The reference's ``OuroLatentAttention.forward`` (hla/vllm_latent/ouro_latent.py:106-131) is the per-layer
code path vLLM runs once per loop: the writer accumulation, the fused QKV projection, the latent query
(before the exact RoPE), the exact RoPE and the exact-window cache append, ``s6_layer.attend``, the commit
of the latent row at loops 0 and T-1, and the O projection.  vLLM supplies the paged caches, block tables
and metadata through its forward context (``get_attention_context``); here the caller passes them in a
``PagedCaches`` record, so the same per-layer sequence runs in tests over a simulated paged cache, and in
any host that owns its KV memory.

Per (layer, loop) the launches are this package's kernels except the two dense projections (cuBLAS via
torch, as vLLM's ``QKVParallelLinear`` / ``RowParallelLinear``):

  writer            s6_layer.write_rows                         (ouro_latent.py:108)
  qkv               F.linear                                    (:109-110)
  latent query      StepContext.latent_query                    (:111, before the in-place exact RoPE)
  exact RoPE + append  hla_s6_exact_append: q rotated in place, k rotated, k|v stored at the exact
                    cache's slots (rotary_emb :112 + unified_kv_cache_update :121-123)
                    - in a decode batch with a window both run as one launch (hla_s6_decode_prepare:
                    q_lat, and the exact RoPE of q into a separate q_rope), and the history split
                    is its programmatic dependent
  attend            s6_layer.attend                              (:124-125)
  commit            hla_s6_commit_rows: the K half latent-RoPE'd and the row stored at the latent
                    cache's slots (committed_row + unified_kv_cache_update, :126-129)
  o_proj            F.linear                                    (:130)

Padding tokens (``t >= query_start_loc[-1]``) get zero output and write no cache row.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib, s6_layer


@dataclass
class PagedCaches:
    """The paged caches one layer reads and writes, and their per-request block tables (int32).

    ``main`` ``[nb, 1, page, 2 * rank]`` and ``l1`` ``[nb, 1, page, 2 * rank1]`` share ``latent_table``
    (one cache group geometry, as the reference's serving test uses); ``exact[t]`` is loop t's exact
    cache in vLLM's TRITON_ATTN physical layout ``[nb, page, H, 2 * head_dim]`` with ``exact_table``
    (a sliding window of W + 1 rows needs only the pages it touches).  ``exact`` may be empty when the
    model has no window (W = 0)."""
    main: torch.Tensor
    l1: torch.Tensor
    latent_table: torch.Tensor
    exact: list
    exact_table: torch.Tensor | None


class LatentAttention:
    """The S6 attention of one Ouro layer: frozen ``qkv_weight [3 H d, hidden]`` / ``o_weight [hidden, H d]``,
    the layer's ``LatentLayer`` student, the exact RoPE table ``cos_sin [max_position, d]`` (``[cos | sin]``
    fp32, neox pairs ``(i, i + d/2)``) and the window W."""

    def __init__(self, latent, qkv_weight, o_weight, cos_sin, window):
        self.latent, self.qkv_weight, self.o_weight = latent, qkv_weight, o_weight
        self.cos_sin, self.window = cos_sin, int(window)
        self.heads, self.head_dim = latent.heads, latent.head_dim

    def forward(self, positions, hidden_states, current_ut, state, ctx, caches, return_attention=False):
        """One loop of one layer: ``(output [T, hidden], writer state)`` (plus the attention output
        ``[T, H, d]`` before the O projection when ``return_attention``); commits the loop-1 row at loop 0
        and the main row at the last loop (reference ouro_latent.py:106-131)."""
        T, sl = hidden_states.shape[0], self.latent
        H, d = self.heads, self.head_dim
        state = s6_layer.write_rows(sl, current_ut, hidden_states, state)
        qkv = F.linear(hidden_states, self.qkv_weight)
        q, k, v = (x.view(T, H, d) for x in qkv.split(H * d, -1))
        cache = caches.l1 if current_ut == 0 else caches.main
        md = ctx.md_present
        if self.window and md and ctx.max_query_len == 1:
            # decode batch: latent query, exact RoPE and exact-cache append in one launch, and the history
            # split as its programmatic dependent (the same values as the separate ops below)
            cache_e = caches.exact[current_ut].transpose(1, 2)  # logical [nb, H, page, 2d]
            # the per-token block table the split reads is gathered now, so that no launch comes between the
            # prepare and the split (whose producer reads the table before it waits for the prepare)
            ctx.block_table(caches.latent_table)
            q_lat, q_rope = self._prepare(current_ut, q, k, v, positions, cache_e, caches.exact_table, ctx)
            ctx.history_after_query = True
            try:
                out = s6_layer.attend(sl, current_ut, q_lat, q_rope, None, v, cache, caches.latent_table, None,
                                      None, ctx, (cache_e, caches.exact_table))
            finally:
                ctx.history_after_query = False
            if current_ut == 0 or current_ut == sl.loops - 1:
                self._commit(current_ut, state, positions, cache, caches.latent_table, ctx)
            output = F.linear(out.reshape(T, H * d), self.o_weight)
            return (output, state, out) if return_attention else (output, state)
        q_lat = ctx.latent_query(sl, current_ut, q)            # before the in-place exact RoPE
        k_rope = torch.empty(T, H, d, dtype=k.dtype, device=k.device)
        window = None
        if self.window and md:
            cache_e = caches.exact[current_ut].transpose(1, 2)  # logical [nb, H, page, 2d]
            self._exact_append(q, k, v, k_rope, positions, cache_e, caches.exact_table, ctx)
            window = (cache_e, caches.exact_table)
        else:
            self._exact_append(q, k, v, k_rope, positions, None, None, ctx)
        out = s6_layer.attend(sl, current_ut, q_lat, q, k_rope, v, cache if md else None,
                              caches.latent_table if md else None, None, None, ctx, window)
        if md and (current_ut == 0 or current_ut == sl.loops - 1):
            self._commit(current_ut, state, positions, cache, caches.latent_table, ctx)
        output = F.linear(out.reshape(T, H * d), self.o_weight)
        return (output, state, out) if return_attention else (output, state)

    def _prepare(self, loop, q, k, v, positions, cache, table, ctx):
        """hla_s6_decode_prepare: ``q_lat`` = latent RoPE of ``q . A`` (ctx.latent_query), ``q_rope`` = exact
        RoPE of q (a separate output), RoPE(k) | v stored at each token's exact-cache slot - one launch."""
        sl = self.latent
        T, H, d = q.shape
        A, _, width = sl.readers(loop)
        tab = ctx.tables[width]
        q_lat = torch.empty(T, H, width, dtype=q.dtype, device=q.device)
        q_rope = torch.empty(T, H, d, dtype=q.dtype, device=q.device)
        pos = positions if positions.dtype == torch.int64 else positions.long()
        qsl = ctx.query_start_loc
        nb, _, page, _ = cache.shape
        sb, sh, sr, _ = cache.stride()
        _lib.call('hla_s6_decode_prepare', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(A), A.stride(0),
                  A.stride(1), _lib.ptr(pos), _lib.ptr(tab), tab.stride(0), tab.shape[0], _lib.ptr(q_lat),
                  q_lat.stride(0), q_lat.stride(1), T, H, d, width, _lib.ptr(q_rope), q_rope.stride(0),
                  q_rope.stride(1), _lib.ptr(k), k.stride(0), k.stride(1), _lib.ptr(v), v.stride(0), v.stride(1),
                  _lib.ptr(self.cos_sin), self.cos_sin.stride(0), self.cos_sin.shape[0], _lib.ptr(cache), nb, sb, sh,
                  sr, page, _lib.ptr(table), table.stride(0), table.shape[1], _lib.ptr(qsl), qsl.shape[0] - 1, None,
                  0, _lib.stream_of(q))
        return q_lat, q_rope

    def _exact_append(self, q, k, v, k_rope, positions, cache, table, ctx):
        """Exact neox RoPE of q (in place) and k (into ``k_rope``), and - with a cache - k_rope | v stored at
        slot ``table[req, pos // page] * page + pos % page`` (padding tokens skipped)."""
        T, H, d = q.shape
        if cache is None:                                      # RoPE only: no slot (max_blocks 0) is written
            nb = sb = sh = sr = 0
            page, bt_stride, max_blocks = 1, 0, 0
        else:
            nb, _, page, _ = cache.shape
            sb, sh, sr, _ = cache.stride()
            bt_stride, max_blocks = table.stride(0), table.shape[1]
        qsl = ctx.query_start_loc
        pos = positions if positions.dtype == torch.int64 else positions.long()
        _lib.call('hla_s6_exact_append', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(k), k.stride(0), k.stride(1),
                  _lib.ptr(v), v.stride(0), v.stride(1), _lib.ptr(k_rope), k_rope.stride(0), k_rope.stride(1),
                  _lib.ptr(pos), _lib.ptr(self.cos_sin), self.cos_sin.stride(0), self.cos_sin.shape[0],
                  _lib.ptr(cache), nb, sb, sh, sr, page, _lib.ptr(table), bt_stride, max_blocks, _lib.ptr(qsl),
                  qsl.shape[0] - 1, T, H, d, None, _lib.stream_of(q))

    def _commit(self, loop, state, positions, cache, table, ctx):
        """The committed latent row of ``loop`` (loop-1 row at loop 0, main row at the last loop): K half
        latent-RoPE'd in the torch bf16 order of LatentLayer.pack and the row stored at the token's slot -
        committed_row + unified_kv_cache_update in one launch."""
        sl = self.latent
        row, width = (state.first, sl.rank1) if loop == 0 else (state.reg, sl.rank)
        tab = ctx.tables[width]
        pos = positions if positions.dtype == torch.int64 else positions.long()
        qsl = ctx.query_start_loc
        _lib.call('hla_s6_commit_rows', _lib.ptr(row), row.stride(0), width, _lib.ptr(pos), _lib.ptr(tab),
                  tab.stride(0), tab.shape[0], _lib.ptr(cache), cache.shape[0], cache.stride(0), cache.stride(2),
                  cache.shape[2], _lib.ptr(table), table.stride(0), table.shape[1], _lib.ptr(qsl), qsl.shape[0] - 1,
                  row.shape[0], None, _lib.stream_of(row))
