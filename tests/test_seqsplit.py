"""Sequence split of the latent history across ranks.

CPU: two gloo ranks each attend over their page slice with the oracle, all-gather (z, lse) and
LSE-merge; the result equals the oracle over the whole history, and the slices tile it exactly.
GPU (two or more devices): two ranks run the kernel path - history split on the local slice, fp32
reduce, exchange of the packed parts (peer stores of tagged exchange words, or an NCCL all-gather), N-part
combine -
and match the single-GPU path over the whole history, over two steps.
"""
import math
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import pkg
from oracle import s6_oracle as orc

PAGE = 16


def _run_ranks(fn, world, init, out, limit_s, *extra):
    """Spawn ``world`` ranks and wait at most ``limit_s`` seconds; stragglers are terminated."""
    ctx = mp.spawn(fn, args=(world, init, out, *extra), nprocs=world, join=False)
    import time
    deadline = time.time() + limit_s
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.terminate()
            raise TimeoutError(f'ranks did not finish within {limit_s} s')


def _global_case(seed, T=3, W=64, H=4, ctx=(300, 17, 100)):
    rng = np.random.default_rng(seed)
    pages = [-(-c // PAGE) for c in ctx]
    nb = sum(pages) + 1
    cache = rng.standard_normal((nb, 1, PAGE, 2 * W)).astype(np.float32)
    table = np.zeros((T, max(pages)), dtype=np.int32)
    k = 1
    for t, p in enumerate(pages):
        table[t, :p] = np.arange(k, k + p)
        k += p
    q = rng.standard_normal((T, H, W)).astype(np.float32)
    return q, cache, table, np.asarray(ctx)


def test_split_rows_tile_the_history():
    dec = pkg('decode')
    for rows in ([131040], [0, 1, 15, 16, 17, 1000], [5000, 33]):
        for world in (1, 2, 3, 8):
            parts = [dec.seq_split_rows(rows, PAGE, r, world) for r in range(world)]
            for i, n in enumerate(rows):
                assert sum(p[i][1] for p in parts) == n
                starts = [p[i][0] for p in parts]
                assert starts == sorted(starts)


def _cpu_rank(rank, world, init, out):
    dist.init_process_group('gloo', init_method=init, rank=rank, world_size=world)
    try:
        dec = pkg('decode')
        q, cache, table, ctx = _global_case(1)
        scale = 1 / math.sqrt(128)
        split = dec.seq_split_rows(ctx.tolist(), PAGE, rank, world)
        local_table = np.zeros_like(table)
        rows = np.zeros_like(ctx)
        for t, (p0, n) in enumerate(split):
            npg = -(-n // PAGE)
            local_table[t, :npg] = table[t, p0:p0 + npg]
            rows[t] = n
        z, lse = orc.history_attention(q, cache, local_table, rows, scale)
        zt = torch.from_numpy(z.astype(np.float64))
        lt = torch.from_numpy(lse.astype(np.float64))
        zs = [torch.empty_like(zt) for _ in range(world)]
        ls = [torch.empty_like(lt) for _ in range(world)]
        dist.all_gather(zs, zt)
        dist.all_gather(ls, lt)
        if rank == 0:
            L = torch.stack(ls)                     # [world, H, T]
            m = L.max(0).values
            safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
            w = torch.exp(L - safe)                 # [world, H, T]
            tot = w.sum(0)
            Z = torch.stack(zs)                     # [world, T, H, W]
            merged = (Z * w.permute(0, 2, 1)[..., None]).sum(0) / tot.t()[..., None].clamp_min(1e-300)
            merged_lse = safe + torch.log(tot)
            ref, ref_lse = orc.history_attention(q, cache, table, ctx, scale)
            np.testing.assert_allclose(merged.numpy(), ref, rtol=1e-9, atol=1e-9)
            np.testing.assert_allclose(merged_lse.numpy(), ref_lse, rtol=1e-9, atol=1e-9)
            with open(out, 'w') as f:
                f.write('ok')
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 4])
def test_gloo_ranks_merge_to_the_full_history(world):
    with tempfile.TemporaryDirectory() as d:
        init, out = f'file://{os.path.join(d, "rdv")}', os.path.join(d, 'result')
        _run_ranks(_cpu_rank, world, init, out, 180)
        assert open(out).read() == 'ok'


# ----------------------------------------------------------------------------- GPU, NCCL
def _gpu_rank(rank, world, init, out, mode):
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', init_method=init, rank=rank, world_size=world,
                            device_id=torch.device('cuda', rank), timeout=datetime.timedelta(seconds=60))
    part = None
    try:
        dec = pkg('decode')
        lib = pkg('_lib')
        shape = dec.OuroShape(layers=1)
        ctx = [4096, 1000, 40, 2000]
        full = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=7)
        split = dec.seq_split_rows([max(c - 32, 0) for c in ctx], PAGE, rank, world)
        part = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=7,
                                 latent_rows=[n for _, n in split], exchange=(rank, world, dist.group.WORLD),
                                 exchange_mode=mode)
        # the split model attends over the same latent rows: give it this rank's pages of the full model
        for t, (p0, n) in enumerate(split):
            npg = -(-n // PAGE)
            part.latent_table[t].zero_()
            part.latent_table[t, :npg] = full.latent_table[t, p0:p0 + npg]
        for name in ('main', 'l1'):
            for layer in range(shape.layers):
                getattr(part, name)[layer] = getattr(full, name)[layer]
        part.acts.copy_(full.acts)
        part.exact = full.exact
        part.exact_logical = full.exact_logical
        for a, b in zip(part.layers, full.layers):
            a.load_state_dict(b.state_dict())
        stream = lib.stream_of(full.out)
        acts0 = full.acts.clone()
        # two steps: every exchange slot (and, in peer mode, its epoch and CTA counter) is used twice
        for step in range(2):
            for loop in range(shape.loops):
                full.acts[0, loop].copy_(acts0[0, loop])
                part.acts[0, loop].copy_(acts0[0, loop])
                full.layer_loop(0, loop, stream)
                part.layer_loop(0, loop, stream)
            torch.cuda.synchronize()
            torch.testing.assert_close(part.out.float(), full.out.float(), atol=2e-2, rtol=1e-2)
            part.out.zero_()
        if mode == 'peer':
            counters = part.x_counters.view(-1, 2).cpu()
            assert (counters[:, 0] == 2).all()                 # every slot's epoch advanced once per step
            assert (counters[:, 1] == 0).all()                 # CTA counters left zeroed for the next use
        if rank == 0:
            with open(out, 'w') as f:
                f.write('ok')
    finally:
        if part is not None:
            part.close_exchange()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('mode', ['peer', 'nccl'])
def test_two_ranks_match_the_whole_history_path(mode):
    """peer: the reduce stores each part into both GPUs' memory as exchange words that the combine
    polls (one GPU per rank, so the polls never wait on a launch of the same GPU); nccl: all_gather
    of the parts."""
    with tempfile.TemporaryDirectory() as d:
        init, out = f'file://{os.path.join(d, "rdv")}', os.path.join(d, 'result')
        _run_ranks(_gpu_rank, 2, init, out, 300, mode)
        assert open(out).read() == 'ok'
