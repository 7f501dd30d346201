"""Run eager S6 decode steps of an Ouro-shaped model - a small, self-contained workload for profilers.

    python hybrid-latent-attention_b200/profile_step.py [--layers 2] [--batch 64] [--ctx 8192] [--steps 2]
    python hybrid-latent-attention_b200/profile_step.py --prefill [--layers 1] [--prompts 8] [--steps 1]
    python hybrid-latent-attention_b200/profile_step.py --seq-split 2 [--layers 2] [--batch 4] [--ctx 131072]
    python hybrid-latent-attention_b200/profile_step.py --reader contig|heads|export [--batch 64] [--ctx 8192]

Every step issues the four launches per (layer, loop) of ``decode.S6DecodeModel.step`` in order
(writer, prepare, history split, combine; loop 0 reads the 256-wide latent, loops 1-3 the 512-wide
one), so ``ncu -k regex:history_split -s 1 -c 2`` selects one launch of each width.  With the
defaults the device holds about 3 GB.

``--seq-split N`` runs rank 0's share of an N-way sequence split (config 5: ``--batch 4 --ctx 131072``) as a
one-rank job (``--time`` also times it as a graph): the latent rows of the first of N page slices, the reduce with its peer-store exchange
(to this GPU only) and the N = 1 flag wait in the combine; the kernel sequence and sizes per GPU are
those of the N-GPU step, without the other ranks.

``--reader`` runs two calls of one of the other readers at the config-2 shape (B = 64 rows, ctx 8192):
``contig`` the HF engines' contiguous reader (K/V [64, 8160, 512], 1.07 GB), ``heads`` the per-head
LLA reader (16 KV heads, rows 128 + 32, 2.7 GB), ``export`` the rollout cache export of one request
(24 layers x 8192 positions, 0.6 GB).

``--prefill`` runs eager steps of the config-3 prompt-step writer instead (prefill.PrefillWriter: four
writer launches per layer, N = 512 at loop 0 and 1024 at loops 1-3, 4096 tokens per prompt); with one
layer and 8 prompts the device holds about 1 GB, the hidden states of a loop (128 MiB) exceed L2.
"""
import argparse
import importlib
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def _graph_ms(torch, graph, reps):
    """Device time per replay of a captured graph (CUDA events, after three warm-up replays)."""
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--layers', type=int, default=2)
    ap.add_argument('--batch', type=int, default=64)
    ap.add_argument('--ctx', type=int, default=8192)
    ap.add_argument('--steps', type=int, default=2)
    ap.add_argument('--prefill', action='store_true')
    ap.add_argument('--prompts', type=int, default=8)
    ap.add_argument('--seq-split', type=int, default=0)
    ap.add_argument('--reader', choices=['contig', 'heads', 'export'])
    ap.add_argument('--time', action='store_true',
                    help='with --seq-split: capture the step as a CUDA graph and report its device time and that of '
                         'its history launches alone (CUDA events)')
    args = ap.parse_args()
    import torch
    dec = importlib.import_module('hybrid-latent-attention_b200.decode')
    if args.reader:
        run_reader(args)
        return
    if args.seq_split:
        import torch.distributed as dist
        dist.init_process_group('gloo', init_method='tcp://127.0.0.1:29531', rank=0, world_size=1)
        shape = dec.OuroShape(layers=args.layers, max_position=args.ctx + 128)
        ctx = [args.ctx] * args.batch
        split = dec.seq_split_rows([c - shape.window for c in ctx], shape.page, 0, args.seq_split)
        model = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=0,
                                  latent_rows=[n for _, n in split], exchange=(0, 1, dist.group.WORLD))
        for _ in range(args.steps):
            model.step(overlap_writer=False)
        torch.cuda.synchronize()
        if args.time:
            ms, ms_hist = _graph_ms(torch, model.capture(), 20), _graph_ms(torch, model.capture_history(), 20)
            loops = shape.layers * shape.loops
            print(f'1/{args.seq_split} slice: step {ms:.3f} ms, history launches alone {ms_hist:.3f} ms, the rest '
                  f'{(ms - ms_hist) / loops * 1e3:.1f} us per (layer, loop)')
            model.graph = model.history_graph = None
        model.close_exchange()
        dist.destroy_process_group()
        print(f'ok: {args.steps} steps of a 1/{args.seq_split} sequence-split slice, '
              f'{model.launches_per_step()} launches each')
        return
    if args.prefill:
        pre = importlib.import_module('hybrid-latent-attention_b200.prefill')
        model = pre.PrefillWriter(dec.OuroShape(layers=args.layers), args.prompts, 4096, device='cuda', seed=0)
        for _ in range(args.steps):
            model.step()
        torch.cuda.synchronize()
        print(f'ok: {args.steps} prefill steps, {model.launches_per_step()} launches each')
        return
    model = dec.S6DecodeModel(dec.OuroShape(layers=args.layers), dec.DecodeBatch([args.ctx] * args.batch),
                              device='cuda', seed=0)
    for _ in range(args.steps):
        model.step(overlap_writer=False)
    torch.cuda.synchronize()
    print(f'ok: {args.steps} steps, {model.launches_per_step()} launches each')


def run_reader(args):
    import torch
    pkg = 'hybrid-latent-attention_b200'
    B, ctx = args.batch, args.ctx
    g = torch.Generator(device='cuda').manual_seed(0)
    if args.reader == 'contig':
        fh = importlib.import_module(f'{pkg}.fused_history')
        N = ctx - 32
        k = torch.randn(B, N, 512, generator=g, device='cuda').to(torch.bfloat16)
        v = torch.randn(B, N, 512, generator=g, device='cuda').to(torch.bfloat16)
        q = torch.randn(B, 16, 512, generator=g, device='cuda').to(torch.bfloat16)
        mask = torch.ones(B, N, dtype=torch.bool, device='cuda')
        for _ in range(2):
            fh.history_attention(q, k, v, mask, 128 ** -0.5)
    elif args.reader == 'heads':
        ops = importlib.import_module(f'{pkg}.s6_ops')
        pages = ctx // 16
        nb = B * pages + 1
        cache = torch.randn(nb, 16, 16, 160, generator=g, device='cuda').to(torch.bfloat16)
        table = (torch.randperm(nb - 1, device='cuda').to(torch.int32) + 1).view(B, pages)
        ctx_t = torch.full((B,), ctx, dtype=torch.int32, device='cuda')
        q = torch.randn(B, 16, 160, generator=g, device='cuda').to(torch.bfloat16)
        splits = ops.num_kv_splits(ctx, B, 512, torch.cuda.get_device_properties(0).multi_processor_count)
        ws = ops.S6Workspace(16, 128, B * splits)
        for _ in range(2):
            ops.history_attention_kv(q, cache, cache[..., :128], table, ctx_t, 128 ** -0.5, splits, ws, None, None,
                                     'b200', mla=True)
    else:
        ce = importlib.import_module(f'{pkg}.cache_export')
        need = ctx // 16
        nb = 4 * need
        main = [torch.randn(nb, 1, 16, 1024, generator=g, device='cuda').to(torch.bfloat16) for _ in range(24)]
        l1 = [torch.randn(nb, 1, 16, 512, generator=g, device='cuda').to(torch.bfloat16) for _ in range(24)]
        mb = torch.randperm(nb, device='cuda')[:need].to(torch.int32)
        lb = torch.randperm(nb, device='cuda')[:need].to(torch.int32)
        for _ in range(2):
            ce.export_rows(main, l1, mb, lb, ctx, 16)
    torch.cuda.synchronize()
    print(f'ok: 2 calls of the {args.reader} reader')


if __name__ == '__main__':
    main()
