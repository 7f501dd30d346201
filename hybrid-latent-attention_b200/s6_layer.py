"""Per (layer, loop) S6 math on B200: the ``hla/vllm_latent/s6_layer.py`` API over libhla_s6.

Same names, signatures and contracts as the reference module: ``StepContext`` once per step,
then per layer and loop ``latent_query`` (before the exact RoPE), ``attend``, ``write_rows`` and
``committed_row``.  Sync-free, no per-request loops, graph-capturable.

The decode branch of ``attend`` (``max_query_len == 1`` with an exact window) is two launches:
the stream-K history kernel and the fused combine (split reduce, B up-projection, exact window,
LSE merge), where the reference issues FA2, the Triton history stages, a cuBLAS einsum and the
merge kernel.  Prefill / mixed steps add the causal chunk attention and the window history.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, s6_ops


def latent_inv_freq(head_dim, theta):
    """The teacher's ``head_dim/2`` RoPE frequencies (reference s6_layer.py:16-18)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))


def latent_rope_table(max_position, inv_freq, width, dtype):
    """``[max_position, width]`` = ``[cos | sin]`` of the latent angles, teacher frequencies round-robin over
    the ``width/2`` pairs (reference s6_layer.py:21-29); built once per model."""
    idx = torch.arange(width // 2, device=inv_freq.device) % inv_freq.shape[0]
    angle = torch.arange(max_position, device=inv_freq.device).float()[:, None] * inv_freq[idx][None, :]
    return torch.cat((angle.cos(), angle.sin()), -1).to(dtype)


def latent_query(q_pre_rope, A, positions, table, backend, flat=False):
    """``[T,H,d]`` pre-RoPE query -> latent-rotated ``[T,H,w]`` (reference s6_layer.py:32-40): absorb and
    latent RoPE fused in one kernel.  ``flat`` is accepted for signature compatibility (the kernel honours
    any head stride)."""
    s6_ops._require(backend, 'rope')
    T, H, d = q_pre_rope.shape
    w = A.shape[-1]
    if A.dtype != torch.bfloat16 or q_pre_rope.dtype != torch.bfloat16 or A.stride(-1) != 1 or q_pre_rope.stride(-1) != 1:
        raise ValueError('latent_query takes bf16 q [T,H,d] and A [H,d,w] with unit last strides')
    out = torch.empty(T, H, w, dtype=q_pre_rope.dtype, device=q_pre_rope.device)
    pos = positions if positions.dtype == torch.int64 else positions.long()
    _lib.call('hla_s6_latent_query', _lib.ptr(q_pre_rope), q_pre_rope.stride(0), q_pre_rope.stride(1), _lib.ptr(A),
              A.stride(0), A.stride(1), _lib.ptr(pos), _lib.ptr(table), table.stride(0), table.shape[0],
              _lib.ptr(out), out.stride(0), out.stride(1), T, H, d, w, _lib.stream_of(q_pre_rope))
    return out


class StepContext:
    """Per-step tensors shared by every layer and loop (reference s6_layer.py:43-84).

    The integer fields (``token_requests``, ``valid``, ``invalid``, ``ctx``, ``ctx_latent``, ``empty``,
    ``empty_latent``) come from one metadata kernel and the per-token block tables from one gather each,
    bit-exact with the reference's torch ops; ``ctx`` / ``ctx_latent`` are int32, the masks bool.

    ``query_start_loc=None`` means a metadata-less (profiling) step: one request spanning all tokens,
    no history and no cache writes.  ``tables`` maps a latent width to its ``[max_position, w]`` RoPE
    table.  All shapes depend only on ``num_tokens`` and CPU ints; nothing here syncs with the host.
    """

    def __init__(self, positions, query_start_loc, seq_lens, max_query_len, num_tokens, tables, scale, backends,
                 workspace=None, num_kv_splits=1, rope_flat=False, window=0, max_seqlen_k=0):
        device = positions.device
        self.window, self.max_seqlen_k = window, max_seqlen_k
        self.positions, self.tables, self.scale, self.backends = positions, tables, scale, backends
        self.workspace, self.num_kv_splits, self.rope_flat = workspace, num_kv_splits, rope_flat
        self.history_needed = True
        self.md_present = query_start_loc is not None
        if not self.md_present:
            query_start_loc = torch.tensor([0, num_tokens], dtype=torch.int32, device=device)
            seq_lens, max_query_len = query_start_loc[1:], num_tokens
        self.query_start_loc, self.seq_lens, self.max_query_len = query_start_loc, seq_lens, max_query_len
        # every integer field in one launch, bit-exact with the reference's torch chain
        (self.token_requests, self.valid, self.invalid, self.ctx, self.ctx_latent, self.empty,
         self.empty_latent) = s6_ops.step_metadata(query_start_loc, seq_lens, num_tokens, window)
        self._block_tables = {}
        if workspace is not None:
            workspace.ensure(device)

    def block_table(self, table):
        """Per-token gather of a per-request block table, once per distinct tensor per step (one launch)."""
        key = table.data_ptr()
        if key not in self._block_tables:
            self._block_tables[key] = s6_ops.gather_block_table(table, self.token_requests)
        return self._block_tables[key]

    def latent_query(self, sl, loop, q_pre_rope):
        A, _, width = sl.readers(loop)
        return latent_query(q_pre_rope, A, self.positions, self.tables[width], self.backends.rope, self.rope_flat)


def attend(sl, loop, q_lat, q_rope, k_rope, v, cache, block_table, k_scale, v_scale, ctx, window=None):
    """One softmax over the paged latent history and the exact part (reference s6_layer.py:87-115).

    ``window = (exact_cache, per-request block table)`` or None; returns ``[T,H,d]`` with ``~valid``
    rows zeroed.  Decode steps with a window (the ones CUDA graphs capture): the stream-K history split
    then one fused combine (split reduce, B up-projection, window over the exact cache incl. the
    current token, merge).  Other steps: causal chunk attention, merged with the window history when
    there is a window, then history split + combine taking that exact part.
    """
    s6_ops._require(ctx.backends.history, 'history')
    T, H, d = q_rope.shape
    stream = _lib.stream_of(q_rope)
    qsl, seq_lens = ctx.query_start_loc, ctx.seq_lens
    fused = window is not None and ctx.md_present and ctx.max_query_len == 1
    chunk_o = chunk_lse = None
    if not fused:
        chunk_o, chunk_lse = s6_ops.chunk_attention(q_rope, k_rope, v, qsl, ctx.max_query_len, ctx.invalid, ctx.scale,
                                                    ctx.backends.chunk)
        if cache is None or not ctx.md_present or not ctx.history_needed:
            return chunk_o.masked_fill_(ctx.invalid[:, None, None], 0)
        if window is not None:
            o_win, lse_win = s6_ops.window_history_fa(q_rope, window[0], ctx.block_table(window[1]), ctx.ctx,
                                                      ctx.window, ctx.scale, ctx.max_seqlen_k, ctx.empty)
            chunk_o, chunk_lse = s6_ops.merge_lse(chunk_o, chunk_lse, o_win, lse_win)
    A, B, width = sl.readers(loop)
    out = torch.empty(T, H, d, dtype=q_rope.dtype, device=q_rope.device)
    use_history = cache is not None and ctx.md_present and ctx.history_needed
    ws_ptr, ws_floats, splits, lpage = None, 0, ctx.num_kv_splits, 16
    if use_history:
        nb, lpage, sb, sr = s6_ops._latent_cache_geometry(cache, width)
        ws = ctx.workspace.attn_logits(T, H, splits, width, q_lat.device)
        ws_ptr, ws_floats = ctx.workspace.buffer, ws.numel()
        bt = ctx.block_table(block_table)
        # a caller whose last launch wrote q_lat (ouro_attention's fused prepare) sets history_after_query:
        # the split then streams pages while that launch runs
        after_query = _lib.PARTIALS_AFTER_QUERY if getattr(ctx, 'history_after_query', False) else 0
        _lib.call('hla_s6_history_partials', _lib.ptr(q_lat), q_lat.stride(0), q_lat.stride(1), _lib.ptr(cache), nb,
                  sb, sr, _lib.ptr(bt), bt.stride(0), bt.shape[1], _lib.ptr(ctx.ctx_latent), T, H, width, lpage,
                  float(ctx.scale), int(splits), _lib.ptr(ws_ptr), ws_floats, None, after_query, stream)
        z_in = lse_in = None
        empty = ctx.empty_latent
    else:
        # no history: one reduced part with lse = -inf stands in for the partials
        z_in = torch.zeros(T, H, width, dtype=torch.float32, device=q_rope.device)
        lse_in = torch.full((H, T), float('-inf'), dtype=torch.float32, device=q_rope.device)
        empty = None
    if fused:
        exact, exact_table = window
        (enb, _, epage, _), (esb, esh, esr, _) = s6_ops._exact_cache_geometry(exact)
        win_args = (_lib.ptr(q_rope), q_rope.stride(0), q_rope.stride(1), _lib.ptr(exact), enb, esb, esh, esr, epage,
                    _lib.ptr(exact_table), exact_table.stride(0), exact_table.shape[1])
        chunk_args = (None, 0, 0, None)
    else:
        win_args = (None, 0, 0, None, 0, 0, 0, 0, 1, None, 0, 0)
        chunk_args = (_lib.ptr(chunk_o), chunk_o.stride(0), chunk_o.stride(1), _lib.ptr(chunk_lse))
    flags = _lib.COMBINE_AFTER_PARTIALS if (use_history and fused) else 0
    _lib.call('hla_s6_decode_combine', T, H, width, lpage, int(splits), _lib.ptr(ws_ptr), ws_floats, _lib.ptr(z_in),
              _lib.ptr(lse_in), 1, 0, None, None, _lib.ptr(empty), _lib.ptr(B), B.stride(0), B.stride(1), *win_args,
              _lib.ptr(qsl), qsl.shape[0] - 1, _lib.ptr(seq_lens), int(ctx.window), float(ctx.scale), *chunk_args,
              _lib.ptr(out), out.stride(0), out.stride(1), None, flags, None, stream)
    return out


@dataclass
class WriterState:
    reg: torch.Tensor | None = None
    first: torch.Tensor | None = None


def write_rows(sl, loop, h, state=None):
    """Writer accumulation on the attention input ``h[T, hidden]`` (reference s6_layer.py:124-132):
    loop 0 gives ``first = E_1' h``; later loops ``reg = reg + E_t h`` with a bf16 add."""
    weight = sl.writer(loop) if hasattr(sl, 'writer') else (sl.cand1.weight if loop == 0 else sl.cand_s[loop - 1].weight)
    T, K = h.shape
    N = weight.shape[0]
    out = torch.empty(T, N, dtype=h.dtype, device=h.device)
    reg_in = None if loop == 0 or state is None else state.reg
    _lib.call('hla_s6_writer_project', _lib.ptr(h), h.stride(0), _lib.ptr(weight), weight.stride(0),
              _lib.ptr(reg_in), 0 if reg_in is None else reg_in.stride(0), _lib.ptr(out), out.stride(0), T, N, K,
              _lib.stream_of(h))
    if loop == 0:
        return WriterState(None, out)
    return WriterState(out, None)


def committed_row(sl, loop, state, ctx):
    """``(key[T,w], value[T,w])`` to store after this loop: loop-1 row at loop 0, main row at the last
    loop, else None (reference s6_layer.py:135-147).  The K half is rotated in place."""
    if loop == 0:
        row, width = state.first, sl.rank1
    elif loop == sl.loops - 1:
        row, width = state.reg, sl.rank
    else:
        return None
    return s6_ops.latent_rope(row[:, :width], ctx.positions, ctx.tables[width], ctx.backends.rope), row[:, width:]
