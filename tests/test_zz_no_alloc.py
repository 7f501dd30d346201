"""hla_s6_history_attention_static: the history attention for callers that cannot allocate device
memory (a foreign-language binding handed only input/output pointers, or a serving process whose
GPU memory is reserved up front).  It takes no workspace - the scratch is a fixed device array
inside the library - and must give the same results as hla_s6_history_attention with a caller
workspace, call after call (the shared scratch keeps the previous call's contents).

This file is collected last so that, if it fails, a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import s6_oracle as orc

pytestmark = pytest.mark.gpu
CUDA, BF16, I32 = 'cuda', torch.bfloat16, torch.int32
O_TOL = dict(atol=2e-2, rtol=1e-2)
LSE_ATOL = 1e-3
P, I64, I32_, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float


def static_entry():
    lib = pkg('_lib').load()
    fn = lib.hla_s6_history_attention_static
    fn.argtypes = [P, I64, I64, P, I64, I64, I64, P, I64, I32_, P, P, I32_, I32_, I32_, I32_, F32, I32_, P, I64, I64,
                   P, P, P]
    fn.restype = ctypes.c_int32
    return fn


def case(seed, T, W, ctx_values, num_blocks=256, page=16):
    g = torch.Generator(device=CUDA).manual_seed(seed)
    cache = torch.randn(num_blocks, 1, page, 2 * W, dtype=BF16, device=CUDA, generator=g)
    ctx = torch.tensor((list(ctx_values) * T)[:T], dtype=I32, device=CUDA)
    maxb = -(-int(ctx.max()) // page) + 1
    table = torch.randint(0, num_blocks, (T, maxb), dtype=I32, device=CUDA, generator=g)
    q = torch.randn(T, 16, W, dtype=BF16, device=CUDA, generator=g)
    return q, cache, table, ctx


def run_static(fn, q, cache, table, ctx, splits, scale):
    T, H, W = q.shape
    o = torch.empty(T, H, W, dtype=BF16, device=CUDA)
    lse = torch.empty(H, T, dtype=torch.float32, device=CUDA)
    lib = pkg('_lib')
    rc = fn(lib.ptr(q), q.stride(0), q.stride(1), lib.ptr(cache), cache.shape[0], cache.stride(0), cache.stride(2),
            lib.ptr(table), table.stride(0), table.shape[1], lib.ptr(ctx), None, T, H, W, cache.shape[2], scale,
            splits, lib.ptr(o), o.stride(0), o.stride(1), lib.ptr(lse), None, lib.stream_of(q))
    lib.check(rc, 'hla_s6_history_attention_static')
    return o, lse


def test_static_scratch_matches_workspace_entry_point_on_consecutive_calls():
    ops = pkg('s6_ops')
    fn = static_entry()
    scale = 1 / math.sqrt(128)
    for i, (T, W, ctx_values, splits) in enumerate([(8, 512, [3000, 0, 17, 1, 255, 1000], 16),
                                                     (33, 256, [700, 5, 0, 64, 2000], 4)]):
        q, cache, table, ctx = case(i + 1, T, W, ctx_values)
        ws = ops.S6Workspace(16, W, T * splits)
        o_ref, lse_ref = ops.history_attention(q, cache, table, ctx, scale, splits, ws, None, None, 'b200')
        o, lse = run_static(fn, q, cache, table, ctx, splits, scale)
        torch.cuda.synchronize()
        torch.testing.assert_close(o.float(), o_ref.float(), **O_TOL)
        empty = ctx == 0
        assert (lse[:, empty] == -math.inf).all() and (o[empty] == 0).all()
        torch.testing.assert_close(lse[:, ~empty], lse_ref[:, ~empty], atol=LSE_ATOL, rtol=0)
        # and the CPU oracle of the reference's history attention (s6_ops.py:204-222)
        o_orc, lse_orc = orc.history_attention(q.float().cpu().numpy(), cache.float().cpu().numpy(),
                                               table.cpu().numpy(), ctx.cpu().numpy(), scale)
        np.testing.assert_allclose(o.float().cpu().numpy(), o_orc, **O_TOL)
        keep = ~empty.cpu().numpy()
        np.testing.assert_allclose(lse.cpu().numpy()[:, keep], lse_orc[:, keep], atol=LSE_ATOL, rtol=0)


def test_static_scratch_one_split_per_row():
    """num_kv_splits = 1: one CTA per row instead of the stream-K page split."""
    ops = pkg('s6_ops')
    fn = static_entry()
    scale = 1 / math.sqrt(128)
    q, cache, table, ctx = case(5, 40, 512, [1500, 0, 33, 16, 1])
    ws = ops.S6Workspace(16, 512, 40)
    o_ref, lse_ref = ops.history_attention(q, cache, table, ctx, scale, 1, ws, None, None, 'b200')
    for _ in range(2):
        o, lse = run_static(fn, q, cache, table, ctx, 1, scale)
        torch.cuda.synchronize()
        torch.testing.assert_close(o.float(), o_ref.float(), **O_TOL)
        empty = ctx == 0
        torch.testing.assert_close(lse[:, ~empty], lse_ref[:, ~empty], atol=LSE_ATOL, rtol=0)
        assert (lse[:, empty] == -math.inf).all()


def test_static_calls_back_to_back_on_one_stream():
    """Two calls enqueued on the same stream before one synchronize: stream order keeps the second
    call's split from overwriting the scratch before the first call's reduce has read it."""
    ops = pkg('s6_ops')
    fn = static_entry()
    scale = 1 / math.sqrt(128)
    a = case(11, 16, 512, [4000, 200, 0, 31])
    b = case(12, 24, 256, [900, 1, 77, 5000])
    refs = []
    for (q, cache, table, ctx), W, splits in ((a, 512, 8), (b, 256, 16)):
        ws = ops.S6Workspace(16, W, q.shape[0] * splits)
        refs.append(ops.history_attention(q, cache, table, ctx, scale, splits, ws, None, None, 'b200'))
    torch.cuda.synchronize()
    out_a = run_static(fn, *a, 8, scale)
    out_b = run_static(fn, *b, 16, scale)
    torch.cuda.synchronize()
    for (o, lse), (o_ref, lse_ref), (_, _, _, ctx) in zip((out_a, out_b), refs, (a, b)):
        torch.testing.assert_close(o.float(), o_ref.float(), **O_TOL)
        empty = ctx == 0
        torch.testing.assert_close(lse[:, ~empty], lse_ref[:, ~empty], atol=LSE_ATOL, rtol=0)


def test_static_scratch_rejects_calls_beyond_its_size():
    fn = static_entry()
    lib = pkg('_lib')
    T, H, W, splits = 64, 16, 512, 16          # 64 * 16 * 16 * 513 floats > 2 Mi
    rc = fn(None, 0, 0, None, 1, 0, 0, None, 0, 0, None, None, T, H, W, 16, 1.0, splits, None, 0, 0, None, None,
            None)
    assert rc == lib.EOVERFLOW
    assert b'static scratch' in lib.load().hla_s6_last_error()
