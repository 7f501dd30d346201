"""CPU oracle of the S6 hybrid decode path: a numpy restatement of the reference's torch path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import this module, and only as the checker / the timed CPU reference.
The product path (``hybrid-latent-attention_b200``) never imports it and has no CPU fallback.

Every function restates one reference function (cited as ``file:line`` within the reference
project, Ch1nyzzz/hybrid-latent-attention) with the same argument meaning, the same masking
and empty-row conventions and the same output layouts.  Floating-point work runs in the
dtype given by ``dt`` (float64 for checking, float32 when timed as the CPU baseline, matching
the reference's ``.float()``).  Integer/index work (token->request mapping, history lengths,
split counts, block-table gathers, cache slots) is exact.

bf16 behaviour is emulated where the reference's *values* depend on bf16 rounding (the
writer's bf16 add and the latent RoPE of committed rows, register.py:45-79): ``bf16()`` is
round-to-nearest-even on the fp32 bit pattern, as torch's CPU bf16 cast.

Pinned by ``tests/test_oracle_golden.py`` against fixtures generated from the reference
itself (``tests/golden/gen_golden.py``).
"""
from __future__ import annotations

import math

import numpy as np

INF = float('inf')


# ----------------------------------------------------------------------------- bf16 helpers
def bf16(x):
    """Round float32 values to the nearest bf16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def bf16_bits(x):
    """bf16 bit patterns (uint16) of bf16-representable float32 values."""
    a = bf16(x)
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits):
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- step metadata
def token_requests(query_start_loc, num_tokens):
    """Request index per token and validity.  hla/vllm_latent/s6_ops.py:61-68."""
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    idx = np.arange(num_tokens, dtype=np.int64)
    req = np.searchsorted(qsl[1:], idx, side='right')
    req = np.minimum(req, qsl.shape[0] - 2)
    return req.astype(np.int64), idx < qsl[-1]


def history_lengths(seq_lens, query_start_loc):
    """``seq_len - query_len`` clamped at 0.  s6_ops.py:71-73."""
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    return np.maximum(np.asarray(seq_lens, dtype=np.int64) - (qsl[1:] - qsl[:-1]), 0)


def step_context(query_start_loc, seq_lens, num_tokens, window=0):
    """Per-token (request, valid, ctx, ctx_latent) of s6_layer.StepContext (s6_layer.py:52-70)."""
    req, valid = token_requests(query_start_loc, num_tokens)
    hist = history_lengths(seq_lens, query_start_loc)
    ctx = np.where(valid, hist[req], 0)
    ctx_latent = np.maximum(ctx - window, 0) if window else ctx.copy()
    return req, valid, ctx, ctx_latent


def num_kv_splits(max_seq_len, num_tokens, split_max_tokens, sm_count, head_blocks=1):
    """Split count of the paged-history kernel.  s6_ops.py:76-89."""
    if num_tokens > split_max_tokens:
        return 1
    ideal = 1 << (max(1, max_seq_len // 512) - 1).bit_length()
    fill = -(-2 * sm_count // (num_tokens * head_blocks))
    return max(1, min(max(ideal, fill), 2 * sm_count, -(-max_seq_len // 32)))


def workspace_floats(heads, width_max, rows_x_splits):
    """Float count of S6Workspace.  s6_ops.py:100-101."""
    return rows_x_splits * heads * (width_max + 1)


def cache_slots(block_table, req, positions, valid, page):
    """vLLM slot mapping used by unified_kv_cache_update (ouro_latent.py:123,129):
    ``block_table[req, pos // page] * page + pos % page``; padding tokens get -1 (skipped)."""
    bt = np.asarray(block_table, dtype=np.int64)
    pos = np.asarray(positions, dtype=np.int64)
    slots = bt[req, pos // page] * page + pos % page
    return np.where(valid, slots, -1)


# ----------------------------------------------------------------------------- A1 history reader
def history_attention(q, cache, block_table, ctx, scale, dt=np.float64):
    """Paged MQA latent history attention.  s6_ops.py:117-125 -> _history_reference :204-222.

    q [T,H,W]; cache [nb, 1, page, 2W] (K | V); block_table [T, max_blocks] per token;
    ctx [T].  Returns o [T,H,W] and lse [H,T]; empty rows give 0 / -inf.  Only block-table
    columns < ceil(ctx/page) are read (stale columns may point anywhere).
    """
    q = np.asarray(q, dtype=dt)
    cache = np.asarray(cache)
    T, H, W = q.shape
    page = cache.shape[2]
    ctx = np.asarray(ctx, dtype=np.int64)
    o = np.zeros((T, H, W), dtype=dt)
    lse = np.full((H, T), -INF, dtype=dt)
    for t in range(T):
        n = int(ctx[t])
        if n <= 0:
            continue
        pages = -(-n // page)
        ids = np.asarray(block_table[t, :pages], dtype=np.int64)
        if pages > 1 and ids[0] >= 0 and np.array_equal(ids, ids[0] + np.arange(pages)):
            block = cache[ids[0]:ids[0] + pages, 0]               # consecutive blocks: a view, no gather copy
        else:
            block = np.take(cache[:, 0], ids, axis=0)
        rows = block.reshape(pages * page, 2 * W)[:n].astype(dt, copy=False)
        s = (q[t] @ rows[:, :W].T) * dt(scale)                    # [H, n]
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        l = e.sum(-1, keepdims=True)
        o[t] = (e / l) @ rows[:, W:]
        lse[:, t] = (m + np.log(l))[:, 0]
    return o, lse


def history_attention_kv(q, k, v, block_table, ctx, scale, dt=np.float64):
    """Per-head (or MQA) paged attention with separate K/V buffers.  s6_ops.py:128-141, 204-222.

    k [nb, kvH, page, Lk], v [nb, kvH, page, Lv]; H a multiple of kvH.
    """
    q = np.asarray(q, dtype=dt)
    T, H, Lk = q.shape
    kvh, page, Lv = k.shape[1], k.shape[2], v.shape[-1]
    grp = H // kvh
    ctx = np.asarray(ctx, dtype=np.int64)
    o = np.zeros((T, H, Lv), dtype=dt)
    lse = np.full((H, T), -INF, dtype=dt)
    for t in range(T):
        n = int(ctx[t])
        if n <= 0:
            continue
        pages = -(-n // page)
        ids = np.asarray(block_table[t, :pages], dtype=np.int64)
        for g in range(kvh):
            kk = k[ids, g].reshape(pages * page, Lk)[:n].astype(dt)
            vv = v[ids, g].reshape(pages * page, Lv)[:n].astype(dt)
            qs = q[t, g * grp:(g + 1) * grp]
            s = (qs @ kk.T) * dt(scale)
            m = s.max(-1, keepdims=True)
            e = np.exp(s - m)
            l = e.sum(-1, keepdims=True)
            o[t, g * grp:(g + 1) * grp] = (e / l) @ vv
            lse[g * grp:(g + 1) * grp, t] = (m + np.log(l))[:, 0]
    return o, lse


def contiguous_history(q, k, v, mask, scale, dt=np.float64):
    """Contiguous-layout reader of the HF engines.  hla/latent/fused_history.py:11-20.

    q [B,H,R], k/v [B,N,R], mask [B,N] -> z [B,H,R], lse [B,H]; rows without a visible key give 0 / -inf.
    """
    q, k, v = (np.asarray(x, dtype=dt) for x in (q, k, v))
    mask = np.asarray(mask, dtype=bool)
    B, H, R = q.shape
    z = np.zeros((B, H, R), dtype=dt)
    lse = np.full((B, H), -INF, dtype=dt)
    for b in range(B):
        vis = mask[b]
        if not vis.any():
            continue
        s = (q[b] @ k[b][vis].T) * dt(scale)
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        l = e.sum(-1, keepdims=True)
        z[b] = (e / l) @ v[b][vis]
        lse[b] = (m + np.log(l))[:, 0]
    return z, lse


# ----------------------------------------------------------------------------- A5 exact window
def window_attention(q, cache, block_table, ctx, window, scale, dt=np.float64):
    """Exact attention over history rows [ctx - window, ctx).  s6_ops.py:290-314.

    cache is the logical [nb, H, page, 2d] (K | V) view; block_table per token.
    Rows without window history give 0 / -inf.
    """
    q = np.asarray(q, dtype=dt)
    T, H, d = q.shape
    page = cache.shape[2]
    o = np.zeros((T, H, d), dtype=dt)
    lse = np.full((H, T), -INF, dtype=dt)
    for t in range(T):
        pos = [int(ctx[t]) - window + j for j in range(window)]
        pos = [p for p in pos if p >= 0]
        if not pos:
            continue
        rows = np.stack([cache[int(block_table[t, p // page]), :, p % page] for p in pos]).astype(dt)  # [n,H,2d]
        s = np.einsum('hd,nhd->hn', q[t], rows[..., :d]) * dt(scale)
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        l = e.sum(-1, keepdims=True)
        o[t] = np.einsum('hn,nhd->hd', e / l, rows[..., d:])
        lse[:, t] = (m + np.log(l))[:, 0]
    return o, lse


def window_decode(q, cache, block_table, query_start_loc, seq_lens, window, scale, invalid, dt=np.float64):
    """Decode exact window plus the current token: keys [seq_len-1-window, seq_len-1] of each
    request's exact cache (the current token already written).  s6_ops.py:317-331
    (window_attention_fa: FA2 varlen, window_size=[window, 0], seqused_k = seq_lens).

    block_table is per request; each request has query length 1.  Invalid tokens give lse -inf
    and o 0 (the reference leaves FA scratch there; merge_states zeroes it).
    """
    q = np.asarray(q, dtype=dt)
    T, H, d = q.shape
    page = cache.shape[2]
    req, _ = token_requests(query_start_loc, T)
    o = np.zeros((T, H, d), dtype=dt)
    lse = np.full((H, T), -INF, dtype=dt)
    for t in range(T):
        if invalid[t]:
            continue
        r = int(req[t])
        last = int(seq_lens[r]) - 1
        pos = [p for p in range(last - window, last + 1) if p >= 0]
        if not pos:
            continue
        rows = np.stack([cache[int(block_table[r, p // page]), :, p % page] for p in pos]).astype(dt)
        s = np.einsum('hd,nhd->hn', q[t], rows[..., :d]) * dt(scale)
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        l = e.sum(-1, keepdims=True)
        o[t] = np.einsum('hn,nhd->hd', e / l, rows[..., d:])
        lse[:, t] = (m + np.log(l))[:, 0]
    return o, lse


def chunk_attention(q, k, v, query_start_loc, invalid, scale, dt=np.float64):
    """Causal attention inside each request's current chunk.  s6_ops.py:234-259 (_chunk_reference)."""
    q, k, v = (np.asarray(x, dtype=dt) for x in (q, k, v))
    T, H, d = q.shape
    req, _ = token_requests(query_start_loc, T)
    idx = np.arange(T)
    allowed = (req[:, None] == req[None, :]) & (idx[None, :] <= idx[:, None])
    s = np.einsum('ihd,jhd->hij', q, k) * dt(scale)
    s = np.where(allowed[None], s, -INF)
    m = s.max(-1, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(-1, keepdims=True)
    out = np.einsum('hij,jhd->ihd', e / l, v)
    lse = (m + np.log(l))[..., 0]
    lse = np.where(np.asarray(invalid)[None, :], -INF, lse)
    out[np.asarray(invalid)] = 0
    return out, lse


# ----------------------------------------------------------------------------- A7 merges
def merge_states(o_hist, lse_hist, o_chunk, lse_chunk, invalid, dt=np.float64):
    """LSE merge; +inf lse counts as empty, both empty -> 0, invalid rows zeroed.
    s6_ops.py:262-284 (merge_states / _merge_reference)."""
    lh = np.asarray(lse_hist, dtype=dt)
    lc = np.asarray(lse_chunk, dtype=dt)
    lh = np.where(lh == INF, -INF, lh)
    lc = np.where(lc == INF, -INF, lc)
    peak = np.maximum(lh, lc)
    peak = np.where(np.isinf(peak), 0.0, peak)
    with np.errstate(invalid='ignore'):
        wh, wc = np.exp(lh - peak), np.exp(lc - peak)
    total = wh + wc
    with np.errstate(invalid='ignore', divide='ignore'):
        wh = np.where(total > 0, wh / total, 0.0)
        wc = np.where(total > 0, wc / total, 0.0)
    out = np.asarray(o_hist, dtype=dt) * wh.T[..., None] + np.asarray(o_chunk, dtype=dt) * wc.T[..., None]
    out[np.asarray(invalid, dtype=bool)] = 0
    return out


def merge_lse(o1, lse1, o2, lse2, dt=np.float64):
    """LSE merge returning the merged lse; both empty -> 0, -inf.  s6_ops.py:353-361."""
    l1 = np.asarray(lse1, dtype=dt)
    l2 = np.asarray(lse2, dtype=dt)
    peak = np.maximum(l1, l2)
    peak = np.where(np.isinf(peak), 0.0, peak)
    w1, w2 = np.exp(l1 - peak), np.exp(l2 - peak)
    total = w1 + w2
    with np.errstate(invalid='ignore', divide='ignore'):
        a = np.where(total > 0, w1 / total, 0.0).T[..., None]
        b = np.where(total > 0, w2 / total, 0.0).T[..., None]
        out = np.nan_to_num(np.asarray(o1, dtype=dt)) * a + np.nan_to_num(np.asarray(o2, dtype=dt)) * b
        lse = peak + np.log(total)
    return out, lse


# ----------------------------------------------------------------------------- A4 latent query / RoPE
def latent_inv_freq(head_dim, theta):
    """Teacher RoPE frequencies.  s6_layer.py:16-18 (fp32 as torch)."""
    return (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32)
                                          / np.float32(head_dim)))).astype(np.float32)


def latent_rope_table(max_position, inv_freq, width):
    """``[max_position, width]`` = ``[cos | sin]`` of pair angles p * inv_freq[i mod len].
    s6_layer.py:21-29.  fp32; cast to bf16 with ``bf16()`` for a bf16 model."""
    idx = np.arange(width // 2) % inv_freq.shape[0]
    angle = np.arange(max_position, dtype=np.float32)[:, None] * inv_freq[idx][None, :]
    return np.concatenate((np.cos(angle), np.sin(angle)), -1).astype(np.float32)


def rotate_half(x):
    """register.py:14-16."""
    h = x.shape[-1] // 2
    return np.concatenate((-x[..., h:], x[..., :h]), -1)


def latent_rope(x, positions, table, emulate_bf16=False, dt=np.float64):
    """Neox rotate-half RoPE by ``table[positions]``.  s6_ops.py:23-36 (torch backend).

    x [T, ..., w]; with ``emulate_bf16`` the torch bf16 operation order of LatentLayer.pack
    (register.py:73-79) is replayed: bf16(x*cos), bf16(rotate_half(x)*sin), bf16(sum).
    """
    w = table.shape[1]
    tab = table[np.asarray(positions, dtype=np.int64)]
    cos = np.concatenate((tab[:, :w // 2], tab[:, :w // 2]), -1)
    sin = np.concatenate((tab[:, w // 2:], tab[:, w // 2:]), -1)
    shape = (x.shape[0],) + (1,) * (x.ndim - 2) + (w,)
    cos, sin = cos.reshape(shape), sin.reshape(shape)
    if emulate_bf16:
        xf = np.asarray(x, dtype=np.float32)
        a = bf16(xf * cos.astype(np.float32))
        b = bf16(rotate_half(xf) * sin.astype(np.float32))
        return bf16(a + b)
    xd = np.asarray(x, dtype=dt)
    return xd * cos + rotate_half(xd) * sin


def latent_query(q_pre, A, positions, table, dt=np.float64):
    """``RoPE_lat(einsum('thd,hdr->thr', q_pre, A))``.  s6_layer.py:32-40."""
    x = np.einsum('thd,hdr->thr', np.asarray(q_pre, dtype=dt), np.asarray(A, dtype=dt))
    return latent_rope(x, positions, table, dt=dt)


def neox_rope(x, positions, head_dim, theta, dt=np.float64):
    """Exact-path RoPE of q/k per head (HF/vLLM neox, fp32 angles): the model's rotary_emb
    applied at ouro_latent.py:113 before the window cache write."""
    inv = latent_inv_freq(head_dim, theta)
    ang = np.asarray(positions, dtype=np.float32)[:, None] * inv[None, :]
    cos = np.concatenate((np.cos(ang), np.cos(ang)), -1)[:, None, :]
    sin = np.concatenate((np.sin(ang), np.sin(ang)), -1)[:, None, :]
    xd = np.asarray(x, dtype=dt)
    return xd * cos + rotate_half(xd) * sin


# ----------------------------------------------------------------------------- A9 writer
def write_update(h, E):
    """One writer projection ``nn.Linear(hidden, out, bias=False)`` (register.py:47,61):
    fp64 product rounded once to bf16 (cuBLAS accumulates in fp32; differences are held to a
    bf16 tolerance in the tests)."""
    return bf16(np.asarray(h, dtype=np.float64) @ np.asarray(E, dtype=np.float64).T)


def write_step(reg, update):
    """``previous + update`` in bf16 (register.py:45-49, s6_layer.py:124-132)."""
    return update if reg is None else bf16(np.asarray(reg, np.float32) + np.asarray(update, np.float32))


def committed_row(row, width, positions, table_bf16):
    """Rotated K half + untouched V half (s6_layer.py:135-147 with the torch RoPE order of
    register.py:73-79): returns the [T, 2*width] row that is written to the cache."""
    key = latent_rope(row[:, :width], positions, table_bf16, emulate_bf16=True)
    return np.concatenate((key, np.asarray(row[:, width:], np.float32)), -1)


def pack(reg, first, positions, table_main_bf16, table_l1_bf16, rank, rank1):
    """HF row layout ``[rotK rank | V rank | rotK1 rank1 | V1 rank1]``.  register.py:73-79."""
    return np.concatenate((committed_row(reg, rank, positions, table_main_bf16),
                           committed_row(first, rank1, positions, table_l1_bf16)), -1)


def scatter_rows(cache, rows, slots):
    """Write rows into a paged cache [nb, 1, page, 2w] at flat slots; negative slots are skipped
    (vLLM reshape_and_cache semantics used at ouro_latent.py:129)."""
    flat = cache.reshape(-1, cache.shape[-1])
    for i, s in enumerate(np.asarray(slots, dtype=np.int64)):
        if s >= 0:
            flat[s] = rows[i]
    return cache


# ----------------------------------------------------------------------------- rollout cache export
ROLLOUT_SCHEMA = 's6-rollout-cache-v1'      # cache_export.py:10


def export_rows(main_caches, l1_caches, main_blocks, l1_blocks, block_size, length):
    """Rows of one finished request as RolloutCacheExporter.export gathers them (cache_export.py:
    160-174): per layer, positions 0 .. length-1 of the main cache [nb, 1, bs, 2 rank] and of the
    loop-1 cache [nb, 1, bs, 2 rank1], each through its own kv group's physical block list
    (``blocks[pos // bs]``, row ``pos % bs``), concatenated main | l1 -> [1, length, 2 rank + 2 rank1]."""
    pos = np.arange(int(length))
    rows = []
    for main, l1 in zip(main_caches, l1_caches):
        parts = []
        for cache, blocks in ((main, main_blocks), (l1, l1_blocks)):
            phys = np.asarray(blocks, dtype=np.int64)[pos // block_size]
            parts.append(np.asarray(cache)[phys, 0, pos % block_size, :])
        rows.append(np.concatenate(parts, -1)[None])
    return tuple(rows)


# ----------------------------------------------------------------------------- A8 decode attend
def attend_decode(q_lat, q_rope, latent_cache, latent_bt, ctx_latent, exact_cache, exact_bt, query_start_loc,
                  seq_lens, window, B, scale, invalid, dt=np.float64):
    """One (layer, loop) of the fused decode branch of s6_layer.attend (s6_layer.py:87-115):
    window_attention_fa -> history_attention -> einsum B -> merge_states."""
    o_chunk, lse_chunk = window_decode(q_rope, exact_cache, exact_bt, query_start_loc, seq_lens, window, scale,
                                       invalid, dt=dt)
    o_hist, lse_hist = history_attention(q_lat, latent_cache, latent_bt, ctx_latent, scale, dt=dt)
    o_hist = np.einsum('thr,hrd->thd', o_hist, np.asarray(B, dtype=dt))
    return merge_states(o_hist, lse_hist, o_chunk, lse_chunk, invalid, dt=dt)


def joint_decode(q_lat, q_rope, latent_rows, exact_rows, B, scale, dt=np.float64):
    """Independent single-softmax check for one token (batched_engine.mixed_attention,
    batched_engine.py:154-182, and window_diagnostic.window_attention :26-48): one softmax
    over latent scores and exact (window + current) scores, history output ``B (P c^V)``.

    q_lat [H,W], q_rope [H,d], latent_rows [n,2W], exact_rows [m,H,2d], B [H,W,d] -> [H,d].
    """
    W = q_lat.shape[-1]
    d = q_rope.shape[-1]
    q_lat, q_rope = np.asarray(q_lat, dtype=dt), np.asarray(q_rope, dtype=dt)
    lat = np.asarray(latent_rows, dtype=dt)
    ex = np.asarray(exact_rows, dtype=dt)
    s_lat = (q_lat @ lat[:, :W].T) * dt(scale) if lat.shape[0] else np.zeros((q_lat.shape[0], 0), dt)
    s_ex = np.einsum('hd,mhd->hm', q_rope, ex[..., :d]) * dt(scale)
    s = np.concatenate((s_lat, s_ex), -1)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(-1, keepdims=True)
    n = lat.shape[0]
    z = p[:, :n] @ lat[:, W:] if n else np.zeros_like(q_lat)
    out = np.einsum('hr,hrd->hd', z, np.asarray(B, dtype=dt))
    out += np.einsum('hm,mhd->hd', p[:, n:], ex[..., d:])
    return out


def lse_scale_log2(scale):
    return scale * math.log2(math.e)
