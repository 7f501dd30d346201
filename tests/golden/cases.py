"""Deterministic inputs of the golden cases (numpy PCG64, fixed seeds).

The fixtures under tests/golden/*.npz hold the reference's OUTPUTS for these inputs plus a
sha256 of the inputs, so the tests rebuild the inputs here and check the hash before using
the stored outputs.  Values that feed bf16 kernels are bf16-representable float32.
"""
from __future__ import annotations

import hashlib

import numpy as np

INF = float('inf')


def _bf16(x):
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32).copy()


def digest(arrays: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(arrays):
        a = np.ascontiguousarray(arrays[k])
        h.update(k.encode())
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def paged_case(seed, heads, width, page, num_blocks, ctx, max_blocks=None, bf16=True, poison=True):
    """q [T,H,W], cache [nb,1,page,2W] (block 0 = +inf null block), per-token shuffled block
    tables whose stale columns point at the null block (the reference fixture of
    test_s6_ops.py:73-90)."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int32)
    T = ctx.shape[0]
    need = -(-ctx // page)
    mb = max_blocks or max(int(need.max()), 1) + 2
    cache = rng.standard_normal((num_blocks, 1, page, 2 * width), dtype=np.float32)
    q = rng.standard_normal((T, heads, width), dtype=np.float32)
    if bf16:
        cache, q = _bf16(cache), _bf16(q)
    if poison:
        cache[0] = INF
    table = np.zeros((T, mb), dtype=np.int32)
    for t in range(T):
        ids = rng.permutation(np.arange(1, num_blocks))[:mb].astype(np.int32)
        table[t] = ids
        table[t, need[t]:] = 0
    return dict(q=q, cache=cache, block_table=table, ctx=ctx)


def history_cases():
    return {
        'hist_h2_w8_p4': (paged_case(11, 2, 8, 4, 64, [0, 1, 17, 40, 5, 0], max_blocks=12, bf16=False), 1 / np.sqrt(8)),
        'hist_h2_w8_p8': (paged_case(12, 2, 8, 8, 64, [0, 1, 17, 40, 5, 0], max_blocks=12, bf16=False), 1 / np.sqrt(8)),
        'hist_h16_w512_p16': (paged_case(13, 16, 512, 16, 24, [0, 1, 17, 100, 255, 33, 16, 300]), 1 / np.sqrt(128)),
        'hist_h16_w256_p16': (paged_case(14, 16, 256, 16, 24, [0, 1, 17, 100, 255, 33, 16, 300]), 1 / np.sqrt(128)),
        'hist_h16_w512_p32': (paged_case(15, 16, 512, 32, 14, [0, 1, 17, 100, 255, 33, 32, 300]), 1 / np.sqrt(128)),
    }


def window_case(seed=21, heads=16, d=128, page=16, window=32, seq_lens=(1, 2, 33, 34, 70, 5), padding=2):
    """Decode step over per-request exact caches: logical [nb, H, page, 2d] (physical
    (nb, page, H, 2d)), per-request block tables, the current token already written."""
    rng = np.random.default_rng(seed)
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    R = seq_lens.shape[0]
    T = R + padding
    qsl = np.concatenate(([0], np.arange(1, R + 1))).astype(np.int32)
    need = -(-seq_lens // page)
    mb = int(need.max()) + 1
    nb = int(need.sum()) + 4
    phys = _bf16(rng.standard_normal((nb, page, heads, 2 * d), dtype=np.float32))
    phys[0] = INF
    free = rng.permutation(np.arange(1, nb)).astype(np.int32)
    table = np.zeros((R, mb), dtype=np.int32)
    k = 0
    for r in range(R):
        table[r, :need[r]] = free[k:k + need[r]]
        k += need[r]
    q = _bf16(rng.standard_normal((T, heads, d), dtype=np.float32))
    return dict(q=q, cache_phys=phys, block_table=table, query_start_loc=qsl, seq_lens=seq_lens,
                window=np.int32(window))


def merge_case(seed=31, tokens=8, heads=16, dim=128):
    rng = np.random.default_rng(seed)
    o_h = _bf16(rng.standard_normal((tokens, heads, dim), dtype=np.float32))
    o_c = _bf16(rng.standard_normal((tokens, heads, dim), dtype=np.float32))
    l_h = (rng.standard_normal((heads, tokens)) * 3).astype(np.float32)
    l_c = (rng.standard_normal((heads, tokens)) * 3).astype(np.float32)
    l_h[:, 0] = -INF
    l_c[:, 1] = INF
    l_h[:, 2] = -INF
    l_c[:, 2] = -INF
    l_c[:, 3] = -INF
    invalid = np.zeros(tokens, dtype=bool)
    invalid[2] = True
    invalid[7] = True
    return dict(o_hist=o_h, lse_hist=l_h, o_chunk=o_c, lse_chunk=l_c, invalid=invalid)


def rope_case(seed=41, tokens=9, heads=3, widths=(512, 256), max_pos=4096, head_dim=128, theta=1e6):
    rng = np.random.default_rng(seed)
    pos = rng.integers(0, max_pos, tokens).astype(np.int64)
    out = dict(positions=pos, max_pos=np.int64(max_pos), head_dim=np.int64(head_dim), theta=np.float64(theta))
    for w in widths:
        out[f'x{w}'] = _bf16(rng.standard_normal((heads, tokens, w), dtype=np.float32)).transpose(1, 0, 2).copy()
        out[f'row{w}'] = _bf16(rng.standard_normal((tokens, 2 * w), dtype=np.float32))
    return out


def writer_case(seed=51, tokens=7, hidden=256, rank=512, rank1=256, loops=4, max_pos=4096, theta=1e6):
    """Writer inputs: per-loop attention inputs h, bf16 writer weights (LatentLayer.cand_s /
    cand1 shapes), positions, and a paged cache placement (page 16, shuffled blocks)."""
    rng = np.random.default_rng(seed)
    h = _bf16(rng.standard_normal((loops, tokens, hidden), dtype=np.float32))
    E = _bf16(rng.standard_normal((loops - 1, 2 * rank, hidden), dtype=np.float32) / np.sqrt(hidden))
    E1 = _bf16(rng.standard_normal((2 * rank1, hidden), dtype=np.float32) / np.sqrt(hidden))
    pos = rng.integers(0, max_pos, tokens).astype(np.int64)
    return dict(h=h, E=E, E1=E1, positions=pos, max_pos=np.int64(max_pos), theta=np.float64(theta),
                head_dim=np.int64(128), rank=np.int64(rank), rank1=np.int64(rank1))


def chunk_case(seed=61, heads=16, d=128, qsl=(0, 37, 38, 50, 50, 91), num_tokens=94):
    """Varlen causal chunk attention inputs (prefill 37, decode 1, prefill 12, a padded request,
    prefill 41, three padding tokens) - the shape of test_s6_ops.py:105-120 at model widths."""
    rng = np.random.default_rng(seed)
    q, k, v = (_bf16(rng.standard_normal((num_tokens, heads, d), dtype=np.float32)) for _ in range(3))
    return dict(q=q, k=k, v=v, query_start_loc=np.asarray(qsl, dtype=np.int32), num_tokens=np.int64(num_tokens))


def window_history_case(seed=71, heads=16, d=128, page=16, window=32, ctx=(0, 5, 32, 33, 100, 0, 47)):
    """Per-token exact window over history rows [ctx - W, ctx) (s6_ops.py:334-350 semantics)."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int32)
    T = ctx.shape[0]
    need = -(-np.maximum(ctx, 1) // page)
    mb = int(need.max()) + 1
    nb = int(need.sum()) + 2
    phys = _bf16(rng.standard_normal((nb, page, heads, 2 * d), dtype=np.float32))
    phys[0] = INF
    table = np.zeros((T, mb), dtype=np.int32)
    free = rng.permutation(np.arange(1, nb)).astype(np.int32)
    k = 0
    for t in range(T):
        table[t, :need[t]] = free[k:k + need[t]]
        k += need[t]
    q = _bf16(rng.standard_normal((T, heads, d), dtype=np.float32))
    return dict(q=q, cache_phys=phys, block_table=table, ctx=ctx, window=np.int32(window))


def contig_case(seed=81, batch=6, heads=16, width=512, keys=100):
    """Contiguous-layout reader (hla/latent/fused_history.py:11-20): q [B,H,R], K/V [B,N,R], mask [B,N].
    Rows: random masks, a fully masked row, a row whose only visible key is the last one, a fully
    visible row; K at masked keys is poisoned with +inf (the mask must win before the softmax)."""
    rng = np.random.default_rng(seed)
    q = _bf16(rng.standard_normal((batch, heads, width), dtype=np.float32))
    k = _bf16(rng.standard_normal((batch, keys, width), dtype=np.float32))
    v = _bf16(rng.standard_normal((batch, keys, width), dtype=np.float32))
    mask = rng.random((batch, keys)) < 0.6
    mask[1] = False
    mask[2] = False
    mask[2, keys - 1] = True
    mask[3] = True
    k[~mask] = INF
    return dict(q=q, k=k, v=v, mask=mask.astype(np.uint8))


def export_case(seed=91, layers=2, blocks=6, block_size=16, main_w=1024, l1_w=512, length=37):
    """One finished request's rows (cache_export.py:160-174): per-layer bf16 caches, shuffled physical
    block lists per kv group (main and loop-1 use different blocks), a length that ends mid-block."""
    rng = np.random.default_rng(seed)
    main = _bf16(rng.standard_normal((layers, blocks, 1, block_size, main_w), dtype=np.float32))
    l1 = _bf16(rng.standard_normal((layers, blocks, 1, block_size, l1_w), dtype=np.float32))
    need = -(-length // block_size)
    main_blocks = rng.permutation(blocks)[:need].astype(np.int64)
    l1_blocks = rng.permutation(blocks)[:need].astype(np.int64)
    return dict(main=main, l1=l1, main_blocks=main_blocks, l1_blocks=l1_blocks, block_size=np.int64(block_size),
                length=np.int64(length))


def heads_case(seed=101, heads=16, kv_heads=16, rank=128, d_rope=32, page=16, ctx=(0, 1, 17, 100, 250)):
    """Per-head cache read MLA-style (lla_layer.py:67-74 -> s6_ops.py:128-161, mla=True): q [T,H,r+d_rope],
    cache [nb, kvH, page, r + d_rope], v = the first r columns of each row.  Block 0 (+inf) sits under the
    stale table columns and the rows past ctx are +inf, so only visible rows may be read."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int32)
    T, Lk = ctx.shape[0], rank + d_rope
    need = -(-np.maximum(ctx, 1) // page)
    mb = int(need.max()) + 2
    nb = int(need.sum()) + 1
    cache = _bf16(rng.standard_normal((nb, kv_heads, page, Lk), dtype=np.float32))
    cache[0] = INF
    table = np.zeros((T, mb), dtype=np.int32)
    free = rng.permutation(np.arange(1, nb)).astype(np.int32)
    k = 0
    for t in range(T):
        table[t, :need[t]] = free[k:k + need[t]]
        if ctx[t] % page:
            cache[table[t, need[t] - 1], :, ctx[t] % page:] = INF      # rows past ctx in the last page
        k += need[t]
    q = _bf16(rng.standard_normal((T, heads, Lk), dtype=np.float32))
    return dict(q=q, cache=cache, block_table=table, ctx=ctx, rank=np.int32(rank))


def meta_cases():
    """Integer metadata cases (test_s6_ops.py:16-27, 51-70)."""
    return dict(
        token_requests=[((0, 1, 2, 3), 3), ((0, 5), 5), ((0, 3, 4, 6), 6), ((0, 2, 3, 3, 3), 3),
                        ((0, 2, 3, 3, 3), 5), ((0, 2, 3), 5)],
        history_lengths=[((4, 7, 0, 0), (0, 2, 3, 3, 3)), ((1, 1), (0, 2, 4))],
        num_kv_splits=[(8448, 1, 512, 108), (8448, 32, 512, 108), (8448, 512, 512, 108), (384, 1, 512, 108),
                       (100, 8, 512, 108), (8448, 513, 512, 108), (1 << 20, 1, 512, 4), (8192, 64, 512, 148),
                       (8192, 1, 512, 148), (32768, 256, 512, 148), (131072, 4, 512, 148)],
    )


def step_context_cases():
    """vLLM-style step metadata for s6_layer.StepContext (s6_layer.py:52-77): (query_start_loc,
    seq_lens, num_tokens, window, block_table [R, max_blocks]).  Decode batches (one token per request,
    contexts below, at and above the window), padded tokens without and with padded requests (the
    repeated last query_start_loc entry), prefill and mixed prefill/decode chunks, window 0, and a
    64-request decode step at context 8192 (BASELINE config 2's metadata)."""
    rng = np.random.default_rng(88)
    out = []

    def add(qsl, seq_lens, T, window, max_blocks=6):
        R = len(qsl) - 1
        table = rng.integers(0, 1000, (R, max_blocks)).astype(np.int32)
        out.append((list(qsl), list(seq_lens), T, window, table.tolist()))

    add([0, 1, 2, 3, 4], [5, 40, 33, 1], 4, 32)
    add([0, 1, 2, 3, 3, 3], [100, 2, 1, 0, 0], 6, 32)
    add([0, 1, 2], [9, 70], 5, 32)
    add([0, 3, 4, 6], [3, 10, 50], 8, 32)
    add([0, 3, 4, 6], [3, 10, 50], 8, 0)
    add([0, 2, 3, 3, 3], [4, 7, 0, 0], 5, 16)
    add([0, 5], [5], 5, 32)
    add(list(range(65)), [8193] * 64, 64, 32, max_blocks=513)
    return out


def _neox_rope(x, positions, base=10000.0):
    """Rotate-half RoPE over the last dim (head_dim 128) at integer positions, float64."""
    d = x.shape[-1]
    inv = base ** (-np.arange(0, d, 2, dtype=np.float64) / d)
    ang = np.asarray(positions, dtype=np.float64)[..., None] * inv
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., :d // 2].astype(np.float64), x[..., d // 2:].astype(np.float64)
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def config1_case(seed=2048, heads=16, head_dim=128, ctx=2048, window=32, page=16, rank=512, rank1=256, loops=4,
                 latent_theta=10000.0, max_pos=4096):
    """one layer of the S6 hybrid decode op (4 loops; loop 0 reads the loop-1 latent of
    width rank1, loops 1-3 the main latent of width rank) for batch 1 at context 2048 - 2016 latent rows
    and a W = 32 exact window plus the current token (position 2048).  Values N(0, 1); absorb A_t
    [H, d, w] ~ N(0, 1/sqrt(d)) and up-projection B_t [H, w, d] ~ N(0, 1/sqrt(w)); window K and the
    query rotated with RoPE base 10000; page 16 with identity page tables (block j holds page j).
    Every value is bf16-representable."""
    rng = np.random.default_rng(seed)
    H, d = heads, head_dim
    ctx_lat = ctx - window
    pages = -(-(ctx + 1) // page)                        # pages of positions 0 .. ctx
    table = np.arange(pages, dtype=np.int32)[None, :]    # identity: block j = page j
    out = dict(table=table, ctx=np.array([ctx], dtype=np.int32), ctx_lat=np.array([ctx_lat], dtype=np.int32),
               positions=np.array([ctx], dtype=np.int64), seq_lens=np.array([ctx + 1], dtype=np.int32),
               query_start_loc=np.array([0, 1], dtype=np.int32), window=np.int32(window),
               latent_theta=np.float64(latent_theta), max_pos=np.int32(max_pos))
    out['lat_main'] = _bf16(rng.standard_normal((pages, 1, page, 2 * rank), dtype=np.float32))
    out['lat_l1'] = _bf16(rng.standard_normal((pages, 1, page, 2 * rank1), dtype=np.float32))
    pos_rows = (np.arange(pages)[:, None] * page + np.arange(page)[None, :])          # [pages, page]
    for t in range(loops):
        w = rank1 if t == 0 else rank
        out[f'q_pre{t}'] = _bf16(rng.standard_normal((1, H, d), dtype=np.float32))
        out[f'A{t}'] = _bf16(rng.standard_normal((H, d, w), dtype=np.float32) / np.sqrt(d))
        out[f'B{t}'] = _bf16(rng.standard_normal((H, w, d), dtype=np.float32) / np.sqrt(w))
        out[f'q_rope{t}'] = _bf16(_neox_rope(rng.standard_normal((1, H, d)), [[ctx]]))
        k = rng.standard_normal((pages, page, H, d))
        k = _neox_rope(k, pos_rows[:, :, None])
        v = rng.standard_normal((pages, page, H, d))
        out[f'exact{t}'] = _bf16(np.concatenate([k, v], axis=-1))                       # physical [nb, page, H, 2d]
    return out
