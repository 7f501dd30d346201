"""S6 serving ops on B200: the ``hla/vllm_latent/s6_ops.py`` API, backed by libhla_s6 (sm_100a).

Same function names, argument order and meaning, output layouts and error behaviour as the
reference module, so ``s6_layer.attend`` and the vLLM adapter call them unchanged; the
backend string of every op is ``'b200'`` (``select_backends()`` returns it).  There is no
torch or CPU backend here: any other backend string raises ``ValueError`` exactly as an
unknown backend does in the reference, and a missing ``libhla_s6.so`` raises on first use.

Contracts shared by all ops (reference s6_ops.py:1-10): outputs are normalised attention
outputs; ``lse`` is a contiguous fp32 ``[H, T]`` natural-log LSE over already-scaled scores;
empty rows give ``lse = -inf`` and ``o = 0``; no NaN leaves a merge.  No op synchronises with
the host, loops over requests, or allocates beyond its outputs, so every op can be captured
in a CUDA graph and replayed with new contents of q, ctx, block tables and caches.
"""
from __future__ import annotations

from collections import namedtuple

import torch

from . import _lib

INF = float('inf')
BACKEND = 'b200'
Backends = namedtuple('Backends', 'history chunk merge rope')
B200_BACKENDS = Backends(BACKEND, BACKEND, BACKEND, BACKEND)


def _require(backend, kind):
    if backend != BACKEND:
        raise ValueError(f'Unknown {kind} backend {backend!r}')


def _check_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError('S6 b200 ops take CUDA tensors (no CPU path exists)')


# ----------------------------------------------------------------------------- step metadata
def _int32(x):
    return x if x.dtype == torch.int32 else x.int()


def token_requests(query_start_loc, num_tokens):
    """Request index per token (long, clamped into range) and ``valid = arange(T) < query_start_loc[-1]``.

    Same contract as reference s6_ops.py:61-68; one sync-free launch (``hla_s6_step_metadata``).
    Padding tokens are ``~valid``.
    """
    _check_cuda(query_start_loc)
    qsl = _int32(query_start_loc).contiguous()
    device = qsl.device
    req = torch.empty(num_tokens, dtype=torch.int64, device=device)
    valid = torch.empty(num_tokens, dtype=torch.bool, device=device)
    _lib.call('hla_s6_step_metadata', _lib.ptr(qsl), qsl.shape[0] - 1, None, num_tokens, 0, _lib.ptr(req),
              _lib.ptr(valid), None, None, None, None, None, None, _lib.stream_of(qsl))
    return req, valid


def history_lengths(seq_lens, query_start_loc):
    """Per-request history length ``seq_len - query_len``, clamped at 0 (reference s6_ops.py:71-73); one
    launch.  The result has ``seq_lens``' dtype, as the reference's torch arithmetic gives."""
    _check_cuda(seq_lens, query_start_loc)
    qsl = _int32(query_start_loc).contiguous()
    sl = _int32(seq_lens).contiguous()
    hist = torch.empty(sl.shape[0], dtype=torch.int32, device=sl.device)
    _lib.call('hla_s6_step_metadata', _lib.ptr(qsl), qsl.shape[0] - 1, _lib.ptr(sl), 0, 0, None, None, None,
              _lib.ptr(hist), None, None, None, None, _lib.stream_of(sl))
    return hist if seq_lens.dtype == torch.int32 else hist.to(seq_lens.dtype)


def step_metadata(query_start_loc, seq_lens, num_tokens, window=0):
    """Every integer field of ``StepContext`` in one launch: ``(token_requests int64, valid, invalid,
    ctx int32, ctx_latent int32, empty, empty_latent)`` (the masks bool), as s6_layer.py:52-70 derives
    them with torch ops (bit-exact)."""
    _check_cuda(query_start_loc, seq_lens)
    qsl = _int32(query_start_loc).contiguous()
    sl = _int32(seq_lens).contiguous()
    device = qsl.device
    req = torch.empty(num_tokens, dtype=torch.int64, device=device)
    masks = torch.empty(4, num_tokens, dtype=torch.bool, device=device)
    ints = torch.empty(2, num_tokens, dtype=torch.int32, device=device)
    valid, invalid, empty, empty_latent = masks.unbind(0)
    ctx, ctx_latent = ints.unbind(0)
    _lib.call('hla_s6_step_metadata', _lib.ptr(qsl), qsl.shape[0] - 1, _lib.ptr(sl), num_tokens, int(window),
              _lib.ptr(req), _lib.ptr(valid), _lib.ptr(invalid), None, _lib.ptr(ctx), _lib.ptr(ctx_latent),
              _lib.ptr(empty), _lib.ptr(empty_latent), _lib.stream_of(qsl))
    return req, valid, invalid, ctx, ctx_latent, empty, empty_latent


def gather_block_table(table, token_requests):
    """``table[token_requests]`` for a per-request int32 block table (one launch)."""
    _check_cuda(table, token_requests)
    if table.dtype != torch.int32 or table.dim() != 2 or table.stride(-1) != 1:
        raise ValueError('block table must be int32 [num_reqs, max_blocks] with a unit last-dim stride')
    T = token_requests.shape[0]
    out = torch.empty(T, table.shape[1], dtype=torch.int32, device=table.device)
    _lib.call('hla_s6_gather_block_table', _lib.ptr(table), table.stride(0), table.shape[1], table.shape[0],
              _lib.ptr(token_requests), T, _lib.ptr(out), out.stride(0), _lib.stream_of(table))
    return out


def num_kv_splits(max_seq_len, num_tokens, split_max_tokens, sm_count, head_blocks=1):
    """Split budget of the paged-history kernel for a step of ``num_tokens`` rows (reference
    s6_ops.py:76-89, same formula).  On B200 it bounds the partial slots the stream-K history
    kernel may use (``T * splits`` per call); the kernel balances pages across SMs itself."""
    if num_tokens > split_max_tokens:
        return 1
    ideal = 1 << (max(1, max_seq_len // 512) - 1).bit_length()
    fill = -(-2 * sm_count // (num_tokens * head_blocks))
    return max(1, min(max(ideal, fill), 2 * sm_count, -(-max_seq_len // 32)))


class S6Workspace:
    """Persistent fp32 workspace of the history kernel (reference s6_ops.py:92-114).

    Sized for ``rows_x_splits`` (the largest ``num_tokens * num_kv_splits`` a step can request),
    allocated once on first use and never grown: an oversized request raises.
    """

    def __init__(self, heads, width_max, rows_x_splits):
        self.floats = rows_x_splits * heads * (width_max + 1)
        self.buffer = None

    def ensure(self, device):
        if self.buffer is None:
            self.buffer = torch.empty(self.floats, dtype=torch.float32, device=device)
        return self.buffer

    def attn_logits(self, tokens, heads, splits, width, device=None):
        need = tokens * heads * splits * (width + 1)
        buffer = self.ensure(device)
        if need > buffer.numel():
            raise RuntimeError(f'S6 workspace overflow: need {need} floats, have {buffer.numel()}')
        return buffer[:need].view(tokens, heads, splits, width + 1)


# ----------------------------------------------------------------------------- A1 history reader
def _latent_cache_geometry(cache, W):
    if cache.dim() != 4 or cache.shape[1] != 1 or cache.shape[-1] != 2 * W:
        raise ValueError(f'latent cache must be [num_blocks, 1, block, {2 * W}], got {tuple(cache.shape)}')
    if cache.dtype != torch.bfloat16 or cache.stride(-1) != 1:
        raise ValueError('latent cache must be bf16 with a unit last-dim stride')
    return cache.shape[0], cache.shape[2], cache.stride(0), cache.stride(2)


def history_attention(q_lat, cache, block_table, ctx, scale, num_kv_splits, workspace, k_scale, v_scale, backend,
                      empty=None):
    """Fully visible attention of ``q_lat[T,H,W]`` over the first ``ctx[t]`` paged latent rows of an MQA S6 cache.

    ``cache`` is the logical vLLM layout ``[num_blocks, 1, block, 2W]`` (K then V on the last dim);
    ``block_table[T, max_blocks]`` int32 per token (only columns ``< ceil(ctx[t]/block)`` are read);
    ``ctx[T]`` int32.  Returns ``(o[T,H,W] bf16, lse[H,T] fp32)``; empty rows give ``o = 0``,
    ``lse = -inf`` (reference s6_ops.py:117-161).  ``k_scale``/``v_scale`` are accepted for
    signature compatibility; like the reference adapter, quantized caches are not supported.
    """
    _require(backend, 'history')
    _check_cuda(q_lat, cache, block_table, ctx)
    if q_lat.dim() != 3 or q_lat.stride(-1) != 1:
        raise ValueError('q_lat must be [T, H, W] with a unit last-dim stride')
    if q_lat.dtype != torch.bfloat16:
        raise ValueError('q_lat must be bf16')
    T, H, W = q_lat.shape
    nb, page, sb, sr = _latent_cache_geometry(cache, W)
    if block_table.dtype != torch.int32 or ctx.dtype != torch.int32:
        raise ValueError('block_table and ctx must be int32')
    if block_table.stride(-1) != 1:
        raise ValueError('block_table needs a unit last-dim stride')
    o = torch.empty(T, H, W, dtype=q_lat.dtype, device=q_lat.device)
    lse = torch.empty(H, T, dtype=torch.float32, device=q_lat.device)
    ws = workspace.attn_logits(T, H, num_kv_splits, W, q_lat.device)
    buffer = workspace.buffer
    emp = None
    if empty is not None:
        emp = empty.to(torch.uint8) if empty.dtype != torch.bool else empty
    ctx_c = ctx.contiguous()
    _lib.call('hla_s6_history_attention', _lib.ptr(q_lat), q_lat.stride(0), q_lat.stride(1), _lib.ptr(cache), nb, sb,
              sr, _lib.ptr(block_table), block_table.stride(0), block_table.shape[1], _lib.ptr(ctx_c), _lib.ptr(emp), T, H, W, page,
              float(scale), int(num_kv_splits), _lib.ptr(buffer), ws.numel(), _lib.ptr(o), o.stride(0), o.stride(1),
              _lib.ptr(lse), None, _lib.stream_of(q_lat))
    return o, lse


def history_attention_kv(q, k, v, block_table, ctx, scale, num_kv_splits, workspace, k_scale, v_scale, backend,
                         empty=None, mla=False):
    """Paged attention of ``q[T,H,Lk]`` over the first ``ctx[t]`` rows of ``k[num_blocks,kvH,block,Lk]`` /
    ``v[...,Lv]`` (reference s6_ops.py:128-161), ``H`` a multiple of ``kvH``.  Two layouts run on B200:

    * the S6 MQA cache: ``kvH == 1`` with ``k`` and ``v`` the two halves of one ``[num_blocks, 1,
      block, 2W]`` cache (``Lk == Lv``) -> the paged MQA reader (``history_attention``);
    * a per-head cache read MLA-style (``mla=True``, LLA: ``k = cache[..., :r + d_rope]``,
      ``v = cache[..., :r]``): ``v`` must be the first ``Lv`` columns of ``k``'s rows -> the per-head
      reader, which reads each row once.

    Returns ``(o[T,H,Lv] bf16, lse[H,T] fp32)``; empty rows give ``o = 0``, ``lse = -inf``.  Other
    layouts raise ``ValueError``."""
    _require(backend, 'history')
    prefix_view = (v.data_ptr() == k.data_ptr() and v.stride() == k.stride() and v.shape[:3] == k.shape[:3]
                   and v.shape[-1] <= k.shape[-1])
    if mla or k.shape[1] != 1:
        if not prefix_view:
            raise ValueError('b200 per-head history reads the MLA row layout: v must be the first Lv columns of k')
        return _history_heads(q, k, v.shape[-1], block_table, ctx, scale, num_kv_splits, workspace, empty)
    W = q.shape[-1]
    if v.shape[-1] != W or k.shape[-1] != W:
        raise ValueError('b200 MQA history needs Lk == Lv == q width')
    if k.stride() != v.stride() or v.data_ptr() != k.data_ptr() + W * k.element_size():
        raise ValueError('b200 history kernel needs k and v to be the K/V halves of one latent cache')
    cache = torch.as_strided(k, (k.shape[0], 1, k.shape[2], 2 * W), k.stride())
    return history_attention(q, cache, block_table, ctx, scale, num_kv_splits, workspace, k_scale, v_scale,
                             backend, empty)


def _history_heads(q, k, Lv, block_table, ctx, scale, num_kv_splits, workspace, empty):
    _check_cuda(q, k, block_table, ctx)
    if q.dim() != 3 or q.stride(-1) != 1 or q.dtype != torch.bfloat16:
        raise ValueError('q must be bf16 [T, H, Lk] with a unit last-dim stride')
    if k.dim() != 4 or k.dtype != torch.bfloat16 or k.stride(-1) != 1:
        raise ValueError('the per-head cache must be a bf16 [num_blocks, kvH, block, Lk] view with unit last stride')
    if block_table.dtype != torch.int32 or ctx.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise ValueError('block_table and ctx must be int32 (table with a unit last-dim stride)')
    T, H, Lk = q.shape
    nb, kvh, page, _ = k.shape
    if k.shape[-1] != Lk or H % kvh:
        raise ValueError(f'q [T, H, {Lk}] does not match the cache rows ({k.shape[-1]}) / {kvh} KV heads')
    o = torch.empty(T, H, Lv, dtype=q.dtype, device=q.device)
    lse = torch.empty(H, T, dtype=torch.float32, device=q.device)
    ws = workspace.attn_logits(T, H, num_kv_splits, Lv, q.device)
    emp = None
    if empty is not None:
        emp = empty.to(torch.uint8) if empty.dtype != torch.bool else empty
    ctx_c = ctx.contiguous()
    _lib.call('hla_s6_history_attention_heads', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(k), nb, k.stride(0),
              k.stride(1), k.stride(2), kvh, Lk, Lv, page, _lib.ptr(block_table), block_table.stride(0),
              block_table.shape[1], _lib.ptr(ctx_c), T, H, float(scale), int(num_kv_splits), _lib.ptr(workspace.buffer),
              ws.numel(), _lib.ptr(emp), _lib.ptr(o), o.stride(0), o.stride(1), _lib.ptr(lse), None,
              _lib.stream_of(q))
    return o, lse


def _bool_ptr(mask):
    if mask is None:
        return None
    return mask if mask.dtype in (torch.bool, torch.uint8) else mask.to(torch.uint8)


# ----------------------------------------------------------------------------- A5 exact window
def _exact_cache_geometry(cache):
    """Logical TRITON_ATTN view [num_blocks, H, block, 2d] -> (nb, H, block, 2d, strides)."""
    if cache.dim() != 4 or cache.dtype != torch.bfloat16 or cache.stride(-1) != 1:
        raise ValueError('exact cache must be a bf16 [num_blocks, H, block, 2*head_dim] view with unit last stride')
    return cache.shape, cache.stride()


def window_attention_fa(q, cache, block_table, query_start_loc, seq_lens, window, scale, max_seqlen_k, invalid):
    """Decode-only exact window over keys ``[seq_len - 1 - window, seq_len - 1]`` (the window history
    plus the current token, already written) of the exact cache ``[nb, H, block, 2d]``.

    Per-request ``block_table`` / ``seq_lens``; every request has query length 1.  Returns
    ``(o[T,H,d] bf16, lse[H,T] fp32)``; ``invalid`` rows get ``o = 0``, ``lse = -inf``
    (reference s6_ops.py:317-331; ``max_seqlen_k`` is accepted for signature compatibility).
    """
    _check_cuda(q, cache, block_table, query_start_loc, seq_lens)
    T, H, d = q.shape
    (nb, Hc, block, two_d), (sb, sh, sr, _) = _exact_cache_geometry(cache)
    if Hc != H or two_d != 2 * d or q.stride(-1) != 1 or q.dtype != torch.bfloat16:
        raise ValueError('window attention: q [T,H,d] bf16 must match the exact cache [nb, H, block, 2d]')
    o = torch.empty(T, H, d, dtype=q.dtype, device=q.device)
    lse = torch.empty(H, T, dtype=torch.float32, device=q.device)
    _lib.call('hla_s6_window_attention', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(cache), nb, sb, sh, sr,
              block, _lib.ptr(block_table), block_table.stride(0), block_table.shape[1],
              _lib.ptr(query_start_loc), query_start_loc.shape[0] - 1, _lib.ptr(seq_lens), int(window), float(scale),
              T, H, d, _lib.ptr(o), o.stride(0), o.stride(1), _lib.ptr(lse), _lib.stream_of(q))
    return o, lse


def window_history_fa(q, cache, token_block_table, ctx, window, scale, max_seqlen_k, empty):
    """Exact window over history rows only (non-decode steps): token ``t`` reads rows ``[ctx[t] - window,
    ctx[t])`` of the exact cache ``[nb, H, block, 2d]`` through row ``t`` of a per-token block table.
    Rows without history give ``o = 0``, ``lse = -inf`` (reference s6_ops.py:334-350; ``max_seqlen_k``
    and ``empty`` are accepted for signature compatibility - ``ctx == 0`` is the empty condition)."""
    _check_cuda(q, cache, token_block_table, ctx)
    T, H, d = q.shape
    (nb, Hc, block, two_d), (sb, sh, sr, _) = _exact_cache_geometry(cache)
    if Hc != H or two_d != 2 * d or q.stride(-1) != 1 or q.dtype != torch.bfloat16:
        raise ValueError('window history: q [T,H,d] bf16 must match the exact cache [nb, H, block, 2d]')
    if ctx.dtype != torch.int32 or token_block_table.dtype != torch.int32:
        raise ValueError('window history: ctx and the block table must be int32')
    o = torch.empty(T, H, d, dtype=q.dtype, device=q.device)
    lse = torch.empty(H, T, dtype=torch.float32, device=q.device)
    ctx_c = ctx.contiguous()
    _lib.call('hla_s6_window_history', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(cache), nb, sb, sh, sr, block,
              _lib.ptr(token_block_table), token_block_table.stride(0), token_block_table.shape[1], _lib.ptr(ctx_c),
              int(window), float(scale), T, H, d, _lib.ptr(o), o.stride(0), o.stride(1), _lib.ptr(lse),
              _lib.stream_of(q))
    return o, lse


# ----------------------------------------------------------------------------- causal chunk
def chunk_attention(q, k, v, query_start_loc, max_query_len, invalid, scale, backend):
    """Causal attention within each request's current chunk (``q, k, v`` are ``[T,H,d]``).

    Returns ``(o[T,H,d] bf16, lse[H,T] fp32)``; padding tokens (``t >= query_start_loc[-1]``) give
    ``o = 0`` and ``lse = -inf`` (reference s6_ops.py:234-259; ``max_query_len`` and ``invalid`` are
    accepted for signature compatibility - validity follows ``query_start_loc``)."""
    _require(backend, 'chunk')
    _check_cuda(q, k, v, query_start_loc)
    T, H, d = q.shape
    for x in (q, k, v):
        if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            raise ValueError('chunk_attention takes bf16 q/k/v with a unit last-dim stride')
    o = torch.empty(T, H, d, dtype=q.dtype, device=q.device)
    lse = torch.empty(H, T, dtype=torch.float32, device=q.device)
    _lib.call('hla_s6_chunk_attention', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(k), k.stride(0), k.stride(1),
              _lib.ptr(v), v.stride(0), v.stride(1), _lib.ptr(query_start_loc), query_start_loc.shape[0] - 1, T, H, d,
              float(scale), _lib.ptr(o), o.stride(0), o.stride(1), _lib.ptr(lse), _lib.stream_of(q))
    return o, lse


# ----------------------------------------------------------------------------- A7 merges
def merge_states(o_hist, lse_hist, o_chunk, lse_chunk, invalid, backend):
    """LSE merge of two partial softmaxes; ``[T,H,D]`` outputs, ``[H,T]`` fp32 lse; ``invalid`` rows are
    zeroed; ``+inf`` lse counts as empty; both empty give 0 (reference s6_ops.py:262-284)."""
    _require(backend, 'merge')
    _check_cuda(o_hist, o_chunk, lse_hist, lse_chunk)
    T, H, D = o_chunk.shape
    for x in (o_hist, o_chunk):
        if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            raise ValueError('merge_states takes bf16 outputs with a unit last-dim stride')
    out = torch.empty(T, H, D, dtype=o_chunk.dtype, device=o_chunk.device)
    lh, lc = lse_hist.contiguous(), lse_chunk.contiguous()
    inv = _bool_ptr(invalid)   # held in a local: the buffer must outlive the launch's argument list
    _lib.call('hla_s6_merge_states', _lib.ptr(o_hist), o_hist.stride(0), o_hist.stride(1), _lib.ptr(lh),
              _lib.ptr(o_chunk), o_chunk.stride(0), o_chunk.stride(1), _lib.ptr(lc), _lib.ptr(inv),
              _lib.ptr(out), out.stride(0), out.stride(1), T, H, D, _lib.stream_of(o_chunk))
    return out


def merge_lse(o1, lse1, o2, lse2):
    """LSE merge that also returns the merged lse (``[T,H,d]`` outputs, ``[H,T]`` lse); both empty give
    ``0, -inf``; NaN in either output (FA scratch rows) is ignored (reference s6_ops.py:353-361)."""
    _check_cuda(o1, o2, lse1, lse2)
    T, H, D = o1.shape
    out = torch.empty(T, H, D, dtype=o1.dtype, device=o1.device)
    lse = torch.empty(H, T, dtype=torch.float32, device=o1.device)
    l1, l2 = lse1.contiguous(), lse2.contiguous()
    _lib.call('hla_s6_merge_lse', _lib.ptr(o1), o1.stride(0), o1.stride(1), _lib.ptr(l1), _lib.ptr(o2), o2.stride(0),
              o2.stride(1), _lib.ptr(l2), _lib.ptr(out), out.stride(0), out.stride(1), _lib.ptr(lse), T, H, D,
              _lib.stream_of(o1))
    return out, lse


# ----------------------------------------------------------------------------- A4 latent RoPE
def latent_rope(x, positions, table, backend):
    """Neox RoPE of ``x`` by ``table[positions]`` IN PLACE; ``table[max_position, w]`` holds ``[cos | sin]``.

    ``x`` is ``[T, w]``, ``[T, H, w]`` (any head stride, unit last stride) or ``[T, H*w]``;
    ``positions`` int64 ``[T]``.  Per element the torch bf16 order of ``LatentLayer.pack``
    (register.py:73-79): bit-identical to the reference's training formula.  Returns ``x``
    (reference s6_ops.py:23-41, vLLM backend semantics: in place).
    """
    _require(backend, 'rope')
    _check_cuda(x, positions, table)
    w = table.shape[1]
    if x.dtype != torch.bfloat16 or table.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise ValueError('latent_rope takes bf16 x (unit last stride) and a bf16 table')
    T = x.shape[0]
    if x.dim() == 3:
        H, st, sh = x.shape[1], x.stride(0), x.stride(1)
    elif x.shape[-1] == w:
        H, st, sh = 1, x.stride(0), w
    else:
        H, st, sh = x.shape[-1] // w, x.stride(0), w
    pos = positions if positions.dtype == torch.int64 else positions.long()
    _lib.call('hla_s6_latent_rope', _lib.ptr(x), st, sh, T, H, w, _lib.ptr(pos), _lib.ptr(table), table.stride(0),
              table.shape[0], _lib.stream_of(x))
    return x


def probe_latent_rope(table, heads=2, tokens=3):
    """[RUNTIME CHECK] the B200 latent-RoPE kernel against the torch formula on an einsum-shaped ``[T,H,w]``
    input (head stride ``T*w``), as the reference probes its vLLM rotary kernel at model start-up
    (s6_ops.py:44-58, called at ouro_latent.py:203).

    Returns ``(flat, exact)``: ``flat`` is always False here - the kernel honours any head stride, so callers
    never need a contiguous ``[T, H*w]`` copy - and ``exact`` is bit-equality with the torch formula
    ``x*cos + rotate_half(x)*sin`` in the bf16 operation order of ``LatentLayer.pack`` (register.py:73-79).
    Raises ``RuntimeError`` when the kernel disagrees with the formula beyond bf16 rounding."""
    _check_cuda(table)
    w = table.shape[1]
    gen = torch.Generator(device=table.device).manual_seed(0)   # own generator: the model's RNG stays untouched
    x = torch.randn(heads, tokens, w, dtype=table.dtype, device=table.device, generator=gen).transpose(0, 1)
    pos = torch.randint(0, table.shape[0], (tokens,), device=table.device, generator=gen)
    cos, sin = (t.repeat(1, 1, 2) for t in table[pos].view(-1, 1, 2, w // 2).unbind(2))
    half = w // 2
    ref = (x * cos + torch.cat((-x[..., half:], x[..., :half]), -1) * sin).float()
    out = latent_rope(x.clone(), pos, table, BACKEND).float()
    if not torch.allclose(out, ref, atol=1e-2, rtol=1e-2):
        raise RuntimeError('b200 latent_rope disagrees with the latent RoPE reference')
    return False, bool(torch.equal(out, ref))


def select_backends(head_size=128):
    """The B200 kernel backends for every op; raises when CUDA or libhla_s6 is unavailable
    (reference s6_ops.py:364-372)."""
    if not torch.cuda.is_available():
        raise RuntimeError('S6 b200 ops require CUDA')
    _lib.load()
    if head_size != 128:
        raise RuntimeError(f'b200 window kernel is built for head size 128, got {head_size}')
    return B200_BACKENDS
