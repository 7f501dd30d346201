"""Benchmark of the B200 S6 hybrid decode path (BASELINE config 2 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 2|3|4|5|contig|export|heads]

One step = one decode step of an Ouro-1.4B-shaped S6 model's attention path: 24 layers x 4 loops
of (writer projection, latent query, exact RoPE + window append, paged latent-history read,
fused window/B/merge combine, row commits), B = 64 sequences at context 8192 per GPU, paged
caches with a shuffled page table, random-init bf16 weights and synthetic activations.  The
dense Ouro body (QKV/O/MLP GEMMs) is not part of the step.

value: decode tokens/s over all ranks, device-timed (CUDA events around K graph replays,
barrier + synchronize on both sides, max over ranks); inputs resident in HBM and larger than
L2 (the latent caches are ~40 GB per GPU).  e2e: the same step with its per-step activations
copied host->device from pinned memory and its outputs read back, inside the timed region.
roofline: the dominant kernel (history split) timed alone in a graph of its 96 launches.
cpu_baseline / --impl reference: the CPU oracle (numpy fp32 restatement of the reference's
torch path) on bounded, measured samples of the same workload: one decode token of one sequence
through all 24 layers x 4 loops per sample (config 5: one layer of 24, scaled and flagged).

--config contig measures the HF engines' contiguous-layout reader (fused_history.history_attention) at
config-2 scale; --config export the rollout cache export of one 8192-token request (24 layers);
--config heads the per-head (LLA MLA-style) history reader at B = 64, ctx 8192.

--config full times BASELINE config 2 as a whole decode step: the Ouro dense body (RMSNorms, QKV/O
projections, MLP; torch/cuBLAS) around the same attention path, one CUDA graph.

--profile CASE runs a few eager steps of one workload for profilers (see run_profile).

--config 3 measures the latent writer of a prompt step instead (8 prompts x 4096 tokens, 24 layers x
4 loops of writer GEMM + bf16 register add + committed-row RoPE and scatter, tcgen05): rows/s, with
a tensor-pipe roofline; its e2e copies the four loops' hidden states in and one layer's latent
cache out every step.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PKG = 'hybrid-latent-attention_b200'
FALLBACK_HBM_GBS = 6650.0
METRIC = 'S6 decode tokens/s and latent-history HBM GB/s (% roofline), B=64 ctx 8K, 1/2/4/8 GPU'
METRIC3 = 'S6 latent writer (prefill) committed rows/s and tensor TFLOP/s (% roofline), 8 x 4096 prompt tokens'
METRIC_CONTIG = 'contiguous-layout latent history reader tokens/s and HBM GB/s (% roofline), B=64, 8160 keys'
METRIC_EXPORT = 'rollout cache export rows/s and HBM GB/s (% roofline), one 8192-token request, 24 layers'
METRIC_HEADS = 'per-head (LLA MLA-style) latent history reader tokens/s and HBM GB/s (% roofline), B=64 ctx 8K'
FALLBACK_TFLOPS = 1400.0
WINDOW_MODES = {'auto': None, 'on': True, 'off': False}


def dist_env():
    return int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1)), int(os.environ.get('LOCAL_RANK', 0))


def config_batch(config, rank, world, seed):
    """Per-rank workload.  Returns (request contexts, scaling, latent rows held here or None, max_position).

    Config 2: 64 sequences at 8192 per GPU (weak scaling).  Config 4: 256 log-uniform contexts in
    [64, 32768] (a few shorter than the window) split across ranks by greedy sum-of-context balance.
    Config 5: 4 sequences at 131072, each one's latent history split by pages across the ranks."""
    import numpy as np
    dec = importlib.import_module(f'{PKG}.decode')
    if config == 2:
        return [8192] * 64, 'weak', None, 65536
    if config == 5:
        ctx = [131072] * 4
        if world == 1:
            return ctx, 'strong', None, 131200
        split = dec.seq_split_rows([c - 32 for c in ctx], 16, rank, world)
        return ctx, 'strong', [rows for _, rows in split], 131200
    rng = np.random.default_rng(seed)
    ctx = np.exp(rng.uniform(math.log(64), math.log(32768), 256)).astype(np.int64)
    ctx[:8] = rng.integers(1, 32, 8)           # some sequences shorter than the window
    loads = [0] * world
    mine = [[] for _ in range(world)]
    for c in sorted(ctx.tolist(), reverse=True):
        r = loads.index(min(loads))
        loads[r] += c
        mine[r].append(c)
    return mine[rank], 'strong', None, 65536


def peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    return FALLBACK_HBM_GBS, 'fallback'


def tensor_peak():
    """Sustained bf16 dense TFLOP/s (a kernel timed inside a seconds-long loop)."""
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        if 'bf16_tflops_sustained' in d:
            return float(d['bf16_tflops_sustained']), 'measured (MEASURED_PEAKS.json bf16_tflops_sustained)'
    return FALLBACK_TFLOPS, 'fallback 1.4 PFLOP/s sustained'


def ncu_traffic():
    p = ROOT / 'profiles' / 'ncu_traffic.json'
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except json.JSONDecodeError:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms during the timed region (the first sample is
    taken just before it starts)."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, local_rank):
        # nvidia-smi numbers GPUs physically; CUDA_VISIBLE_DEVICES (indices or UUIDs) maps this rank's device
        visible = [v.strip() for v in os.environ.get('CUDA_VISIBLE_DEVICES', '').split(',') if v.strip()]
        self.gpu = visible[local_rank] if local_rank < len(visible) else str(local_rank)
        self.proc, self.file = None, None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
            self.proc = subprocess.Popen(['nvidia-smi', '-i', self.gpu, f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '100'], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a while to start: wait (up to 3 s) for its first sample, so that a timed region
        # shorter than the sampling period still has samples around it
        import time
        deadline = time.time() + 3
        while time.time() < deadline and self.proc.poll() is None:
            self.file.flush()
            if Path(self.file.name).stat().st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return None
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(',')]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == 'active'})
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': float(rows[0][2]),
                'samples': len(rows), 'reasons': reasons,
                'power_w_max': max(float(r[3]) for r in rows if r[3].replace('.', '').isdigit())}


# ----------------------------------------------------------------------------- CPU oracle baseline
class CpuSample:
    """The oracle's decode work for ONE token of one sequence at history ``ctx``: one (layer, loop) pass
    is the writer GEMM, latent query (absorb + RoPE), exact window + current token, paged history over
    ``ctx - W`` latent rows, B up-projection and merge - loop 0 at width rank1, loops 1-3 at rank.
    ``run()`` times ``layers`` x loops passes (every layer reads the same caches, each pass more bytes than
    the host's caches hold) and returns the measured seconds.  With ``layers == shape.layers`` a pass set
    is a whole decode token, so tokens/s needs no extrapolation; the CPU's time per token does not depend
    on how many sequences share a step (each has its own caches)."""

    def __init__(self, shape, ctx, layers, seed=0):
        import numpy as np
        from oracle import s6_oracle as orc
        self.orc, self.np, self.shape, self.ctx, self.layers = orc, np, shape, int(ctx), layers
        rng = np.random.default_rng(seed)
        H, d, page, W_ = shape.heads, shape.head_dim, shape.page, shape.window
        c = self.ctx
        self.scale = 1 / math.sqrt(d)
        self.data = {}
        for width in (shape.rank, shape.rank1):
            pages = -(-(c + 1) // page)
            lat = rng.standard_normal((pages + 1, 1, page, 2 * width), dtype=np.float32)
            ltab = np.arange(1, pages + 1, dtype=np.int32)[None]
            etab = np.zeros_like(ltab)            # exact cache: only the window's pages exist
            k = 1
            for col in range(max(0, c - W_) // page, c // page + 1):
                etab[0, col] = k
                k += 1
            self.data[width] = dict(
                lat=lat, ltab=ltab, etab=etab, ex=rng.standard_normal((k, H, page, 2 * d), dtype=np.float32),
                q_pre=rng.standard_normal((1, H, d), dtype=np.float32),
                h=rng.standard_normal((1, shape.hidden), dtype=np.float32),
                E=rng.standard_normal((2 * width, shape.hidden), dtype=np.float32),
                A=rng.standard_normal((H, d, width), dtype=np.float32),
                Bm=rng.standard_normal((H, width, d), dtype=np.float32),
                tab=np.zeros((c + 1, width), dtype=np.float32), pos=np.asarray([c]),
                qsl=np.arange(2, dtype=np.int32), seq=np.asarray([c + 1], dtype=np.int32),
                ctx_lat=np.maximum(np.asarray([c]) - W_, 0), invalid=np.zeros(1, dtype=bool))
        self._pass(shape.rank)                    # untimed: BLAS thread start, page faults
        self._pass(shape.rank1)

    def _pass(self, width):
        D, orc, np = self.data[width], self.orc, self.np
        _ = D['h'] @ D['E'].T                                                     # writer projection
        q_lat = orc.latent_query(D['q_pre'], D['A'], D['pos'], D['tab'], dt=np.float32)  # absorb + RoPE
        orc.attend_decode(q_lat, D['q_pre'], D['lat'], D['ltab'], D['ctx_lat'], D['ex'], D['etab'], D['qsl'],
                          D['seq'], self.shape.window, D['Bm'], self.scale, D['invalid'], dt=np.float32)

    def run(self):
        s = self.shape
        t0 = time.perf_counter()
        for _ in range(self.layers):
            for loop in range(s.loops):
                self._pass(s.rank1 if loop == 0 else s.rank)
        return time.perf_counter() - t0

    def describe(self):
        s = self.shape
        return (f'oracle numpy fp32 decode of one token at ctx {self.ctx}: {self.layers} layers x {s.loops} loops '
                f'of (writer GEMM, latent query, window, paged history, B, merge) at widths {s.rank1}/{s.rank}')


def cpu_decode_steps(shape, ctx_list, steps, warmup, seed, layers=None):
    """Time ``warmup + steps`` CPU steps of the decode work; step i decodes one token of one sequence,
    taken in a fixed stratified order over the batch's contexts (sorted, then spread) so that a few steps
    cover the length distribution.  Returns (seconds per timed step, contexts timed, layers per step)."""
    L = shape.layers if layers is None else layers
    srt = sorted(int(c) for c in ctx_list)
    n = steps + warmup
    order = [srt[min(len(srt) - 1, (i * len(srt)) // max(n, 1) + len(srt) // (2 * max(n, 1)))] for i in range(n)]
    samples, secs, timed = {}, [], []
    for i, c in enumerate(order):
        if c not in samples:
            samples.clear()                      # one sample's caches resident at a time
            samples[c] = CpuSample(shape, c, L, seed=seed + i)
        t = samples[c].run()
        if i >= warmup:
            secs.append(t)
            timed.append(c)
    return secs, timed, L, samples[order[-1]]


class PrefillCpuSample:
    """The oracle's writer of one layer (4 loops: fp32 GEMM rounded to bf16, bf16 register add, latent
    RoPE of the committed K halves) on ``rows`` tokens of one prompt; ``run()`` times one pass and
    extrapolates it to a step: layers x (T / rows) x the pass."""

    def __init__(self, shape, T, rows, seed=0):
        import numpy as np
        from oracle import s6_oracle as orc
        self.orc, self.np, self.shape, self.T, self.rows = orc, np, shape, T, rows
        rng = np.random.default_rng(seed)
        s = shape
        self.h = [orc.bf16(rng.standard_normal((rows, s.hidden), dtype=np.float32)) for _ in range(s.loops)]
        self.E = [orc.bf16(rng.standard_normal((2 * (s.rank1 if t == 0 else s.rank), s.hidden), dtype=np.float32)
                           / math.sqrt(s.hidden)) for t in range(s.loops)]
        self.pos = np.arange(rows)
        inv = 1.0 / (s.theta ** (np.arange(0, s.head_dim, 2) / s.head_dim))
        self.tab = {}
        for w in (s.rank, s.rank1):
            ang = self.pos[:, None] * inv[np.arange(w // 2) % inv.shape[0]][None]
            self.tab[w] = orc.bf16(np.concatenate((np.cos(ang), np.sin(ang)), -1).astype(np.float32))
        self._layer()                             # untimed: BLAS thread start, page faults

    def _layer(self):
        orc, s = self.orc, self.shape
        first = orc.bf16(self.h[0] @ self.E[0].T)
        orc.committed_row(first, s.rank1, self.pos, self.tab[s.rank1])
        reg = None
        for t in range(1, s.loops):
            reg = orc.write_step(reg, orc.bf16(self.h[t] @ self.E[t].T))
        orc.committed_row(reg, s.rank, self.pos, self.tab[s.rank])

    def pass_seconds(self):
        """Measured seconds of one layer's writer on ``rows`` tokens (it commits ``rows`` rows)."""
        t0 = time.perf_counter()
        self._layer()
        return time.perf_counter() - t0

    def describe(self):
        return (f'oracle numpy fp32 writer of one layer (4 loops: GEMM -> bf16, bf16 register add, latent RoPE of '
                f'the committed rows) on {self.rows} of a prompt step\'s {self.T} tokens; rows/s = rows committed '
                f'per measured second')


def cpu_threads():
    try:
        import threadpoolctl
        return max(i['num_threads'] for i in threadpoolctl.threadpool_info()) or os.cpu_count()
    except Exception:
        return os.cpu_count()


def use_all_host_threads():
    """Let the oracle's BLAS use every host thread (torchrun sets OMP_NUM_THREADS=1 for each rank)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else os.cpu_count()
    try:
        import threadpoolctl
        threadpoolctl.threadpool_limits(limits=n)
    except Exception:
        pass
    return n


def run_reference(args):
    """--impl reference: the CPU oracle port of the reference path on this host, rank 0 only.  Each step is
    one bounded, measured sample: one decode token of one sequence through every (layer, loop) - configs
    2 and 4 - or through one layer's 4 loops at config 5's 131072-token context (then scaled to 24 layers,
    flagged in the line).  ms_per_step is the measured time of that sample."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    dec = importlib.import_module(f'{PKG}.decode')
    shape = dec.OuroShape()
    cores = use_all_host_threads()
    if args.config == 3:
        return run_reference_prefill(args, shape, world)
    ctx, scaling, _, _ = config_batch(args.config, 0, 1, args.seed)
    if args.config == 4:
        ctx = config_batch(4, 0, 1, args.seed)[0]
    layers = 1 if args.config == 5 else shape.layers
    secs, timed, L, last = cpu_decode_steps(shape, ctx, args.steps, args.warmup, args.seed, layers)
    scale = shape.layers / L                    # 1 except at config 5
    tok = len(secs) / (sum(secs) * scale)
    batch = len(ctx) * (world if scaling == 'weak' else 1)
    sample = (f'{last.describe()}; step i decodes one token of one of the batch\'s sequences (contexts timed: '
              f'{sorted(set(timed))[:8]}{"..." if len(set(timed)) > 8 else ""})' +
              (f'; one layer of 24 timed per step, tokens/s scaled by 24' if scale != 1 else ''))
    line = {'metric': METRIC, 'value': tok, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': statistics.mean(secs) * 1e3, 'higher_is_better': True,
            'scaling': scaling, 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic (seeded)', 'impl': 'reference',
            'step': 'one bounded sample: one decode token of one sequence (all 24 layers x 4 loops' +
                    (', of which one layer is timed' if scale != 1 else '') + ')',
            'sample_ms': [round(x * 1e3, 3) for x in secs], 'extrapolated': scale != 1,
            'extrapolation': {'layers_timed': L, 'layers': shape.layers} if scale != 1 else None,
            'config': {'workload': f'BASELINE config {args.config}: S6 decode step attention path, one token of one '
                                   f'sequence per step', 'global_batch': batch, 'ctx': max(ctx),
                       'parallelism': 'host cores'},
            'cpu_baseline': {'value': tok, 'unit': 'tokens/s', 'cores': cores, 'kind': 'port', 'sample': sample},
            'e2e': {'value': tok, 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def prefill_config(world):
    return {'workload': 'BASELINE config 3: latent writer of a prompt step, 24 layers x 4 loops (GEMM + bf16 '
                        'register add + committed-row latent RoPE and paged scatter)',
            'global_batch': 8 * 4096 * world, 'prompts_per_gpu': 8, 'seq_len': 4096, 'hidden': 2048,
            'parallelism': f'request-partitioned x{world} (no collectives)',
            'l2': 'inputs larger than L2 (each loop reads a 128 MiB hidden-state matrix), no flush'}


def run_reference_prefill(args, shape, world):
    """Config 3's reference arm: each step is one layer's writer (4 loops) on --cpu-tokens tokens of one
    prompt, measured; rows/s = the rows that step committed per second (no extrapolation)."""
    T = 8 * 4096
    cs = PrefillCpuSample(shape, T, args.cpu_tokens, seed=args.seed)
    secs = []
    for i in range(args.warmup + args.steps):
        sec = cs.pass_seconds()
        if i >= args.warmup:
            secs.append(sec)
    rows = len(secs) * args.cpu_tokens / sum(secs)
    line = {'metric': METRIC3, 'value': rows, 'unit': 'rows/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': statistics.mean(secs) * 1e3, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic (seeded)', 'impl': 'reference',
            'step': f'one bounded sample: one layer\'s writer (4 loops) on {args.cpu_tokens} prompt tokens',
            'sample_ms': [round(x * 1e3, 3) for x in secs], 'extrapolated': False,
            'config': prefill_config(world),
            'cpu_baseline': {'value': rows, 'unit': 'rows/s', 'cores': cpu_threads(), 'kind': 'port',
                             'sample': cs.describe()},
            'e2e': {'value': rows, 'unit': 'rows/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def time_graph(torch, graph, steps, dist, flush=None):
    """Device time of ``steps`` replays (ms, max over ranks), barrier + synchronize on both sides."""
    stream = torch.cuda.current_stream()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device='cuda')
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_ours(args):
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    importlib.import_module(f'{PKG}._lib').load()
    dec = importlib.import_module(f'{PKG}.decode')
    shape = dec.OuroShape()
    ctx, scaling, latent_rows, max_pos = config_batch(args.config, rank, world, args.seed)
    shape = dec.OuroShape(max_position=max_pos)
    exchange = (rank, world, dist.group.WORLD) if (args.config == 5 and world > 1) else None
    model = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=args.seed + rank,
                              latent_rows=latent_rows, exchange=exchange, exchange_mode=args.exchange,
                              window_overlap=WINDOW_MODES[args.side_window])
    torch.cuda.synchronize()
    model.step()                       # eager warm-up: descriptor caches, occupancy
    graph = model.capture()
    hist_graph = model.capture_history()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    # ---- value: device-timed graph replays, clocks sampled meanwhile
    with ClockSampler(local) as clk:
        ms_total = time_graph(torch, graph, args.steps, dist)
    clocks = clk.summary()
    ms_step = ms_total / args.steps
    tokens_all = len(ctx) * world if scaling == 'weak' else {4: 256, 5: 4}[args.config]
    value = tokens_all / (ms_step / 1e3)

    # ---- roofline of the dominant kernel: the 96 history launches of a step, alone
    for _ in range(3):
        hist_graph.replay()
    ms_hist = time_graph(torch, hist_graph, args.steps, dist) / args.steps
    hist_launches = shape.layers * shape.loops
    bytes_hist = model.latent_bytes_per_step()
    achieved = bytes_hist / (ms_hist / 1e3) / 1e9
    peak, peak_kind = peaks()
    traffic = None
    tr = ncu_traffic()
    if tr and args.config == 2:
        traffic = tr.get('history_split_avg_bytes_per_launch_config2')

    # ---- e2e: pinned host activations in, outputs out, every step
    host_in = torch.empty(model.acts.shape, dtype=model.acts.dtype, pin_memory=True)
    host_in.copy_(model.acts)
    host_out = torch.empty(model.out.shape, dtype=model.out.dtype, pin_memory=True)
    stream = torch.cuda.current_stream()
    io_graph = model.capture_io(host_in, host_out)   # copies pipelined with the launches per (layer, loop)
    for _ in range(2):
        io_graph.replay()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 2)
    e0.record(stream)
    for _ in range(e2e_steps):
        io_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / e2e_steps
    if dist is not None:
        t = torch.tensor([ms_e2e], device='cuda')
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = {'value': tokens_all / (ms_e2e / 1e3), 'unit': 'tokens/s',
           'h2d_bytes_per_step': host_in.numel() * host_in.element_size(),
           'd2h_bytes_per_step': host_out.numel() * host_out.element_size(),
           'path': 'S6DecodeModel.step_io CUDA graph (public API): every (layer, loop)\'s activations copied in from '
                   'pinned host memory and its output copied back, pipelined with the launches'}

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cores = use_all_host_threads()
            layers = 1 if args.config == 5 else shape.layers
            secs, timed, L, last = cpu_decode_steps(shape, ctx, args.cpu_reps, 1, args.seed, layers)
            scale = shape.layers / L
            cpu = {'value': len(secs) / (sum(secs) * scale), 'unit': 'tokens/s', 'cores': cores, 'kind': 'port',
                   'sample': f'{last.describe()}; {len(secs)} timed tokens, one sequence each (contexts '
                             f'{sorted(set(timed))[:6]}{"..." if len(set(timed)) > 6 else ""})' +
                             ('; one layer of 24 timed, scaled by 24' if scale != 1 else ''),
                   'sample_ms': [round(x * 1e3, 3) for x in secs], 'extrapolated': scale != 1}
        attn_bytes = model.latent_bytes_per_step() + model.window_bytes_per_step()
        line = {
            'metric': METRIC, 'value': value, 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True, 'scaling': scaling,
            'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded), random-init weights',
            'config': {'workload': f'BASELINE config {args.config}: Ouro-1.4B-shaped S6 decode step, attention path '
                                   f'(24 layers x 4 loops), dense body excluded' +
                                   ((', latent history sequence-split across GPUs, (z, lse) parts stored into '
                                     'every GPU by the reduce kernel over NVLink (peer memory, tagged exchange words) per (layer, '
                                     'loop)' if args.exchange == 'peer' else
                                     ', latent history sequence-split across GPUs, NCCL all-gather of (z, lse) per '
                                     '(layer, loop)') if exchange is not None else ''),
                       'global_batch': tokens_all, 'batch_per_gpu': len(ctx), 'ctx': max(ctx),
                       'seq_len': max(ctx) + 1, 'page': shape.page, 'window': shape.window,
                       'parallelism': ((f'sequence-split x{world} (fused reduce + peer stores per layer x loop)'
                                        if args.exchange == 'peer' else
                                        f'sequence-split x{world} (NCCL all_gather per layer x loop)')
                                       if exchange is not None else f'request-partitioned x{world} (no collectives)'),
                       'l2': 'inputs larger than L2 (latent caches ~40 GB per GPU), no flush',
                       'side_window': model.window_overlap},
            'latent_history': {'bytes_per_step': bytes_hist, 'GBps_in_step': bytes_hist / (ms_step / 1e3) / 1e9,
                               'attention_bytes_per_step': attn_bytes,
                               'attention_GBps': attn_bytes / (ms_step / 1e3) / 1e9,
                               'frac_of_peak_in_step': attn_bytes / (ms_step / 1e3) / 1e9 / peak},
            'roofline': {'bound': 'hbm', 'kernel': 'history_split_kernel (96 launches per step)',
                         'achieved': achieved, 'peak': peak, 'unit': 'GB/s', 'frac': achieved / peak,
                         'peak_source': f'{peak_kind} (MEASURED_PEAKS.json hbm_gbs)' if peak_kind == 'measured'
                         else 'fallback 6.65 TB/s', 'ms_per_launch': ms_hist / hist_launches,
                         'bytes_per_launch': bytes_hist / hist_launches, 'traffic': traffic},
            'cpu_baseline': cpu,
            'e2e': e2e,
            'gpu_launches': model.launches_per_step() * args.steps,
            'clocks': clocks,
        }
        print(json.dumps(line), flush=True)
    # CUDA graphs that hold NCCL calls must be released before the process group is destroyed
    model.graph = model.history_graph = model.io_graph = None
    del graph, hist_graph, io_graph
    import gc
    gc.collect()
    torch.cuda.synchronize()
    model.close_exchange()             # peer mappings: every rank, after its last launch
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return line


# ----------------------------------------------------------------------------- full decode step
class FullStep:
    """BASELINE config 2's whole decode step: the Ouro decoder layer (hla/vllm_latent/ouro_latent.py:134-154)
    around the B200 attention of OuroLatentAttention.forward (:106-131), 24 layers x 4 loops (:266-275).

    Per (layer, loop): input RMSNorm (with the residual add from the second layer on), the fused QKV
    projection, the S6 attention through ``S6DecodeModel.layer_loop`` (writer on a side stream, prepare,
    history split, combine - q, k, v and h come from this dense body), the O projection, RMSNorm,
    post-attention RMSNorm with the residual add, the SiLU MLP (intermediate 5632) and its RMSNorm;
    after each loop the final RMSNorm.  Dense weights are random-init bf16 on cuBLAS (torch); they are
    not this repository's kernels and are read from HBM every step (about 9.8 GB)."""

    def __init__(self, model, seed, intermediate=5632, eps=1e-6, dropin=False):
        import torch
        self.torch, self.m, self.eps, self.I = torch, model, eps, intermediate
        self.dropin = dropin
        s, B, dev = model.s, model.B, model.device
        D = s.hidden
        g = torch.Generator(device=dev).manual_seed(seed + 7)
        lin = lambda o, i: (torch.randn(o, i, generator=g, device=dev) / math.sqrt(i)).to(torch.bfloat16)
        norm = lambda: (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
        self.w = [dict(qkv=lin(3 * D, D), o=lin(D, D), gate_up=lin(2 * intermediate, D), down=lin(D, intermediate),
                       n1=norm(), n2=norm(), n3=norm(), n4=norm()) for _ in range(s.layers)]
        self.final = norm()
        self.x0 = torch.randn(B, D, generator=g, device=dev).to(torch.bfloat16)
        self.out = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        self.attn = torch.empty(B, s.heads, s.head_dim, dtype=torch.bfloat16, device=dev)
        self.side = torch.cuda.Stream(dev)
        if dropin:
            # the drop-in path: the adapter's per-layer attention (ouro_attention.LatentAttention, a mirror of
            # OuroLatentAttention.forward) over the model's own caches, with a reference-style StepContext
            oa = importlib.import_module(f'{PKG}.ouro_attention')
            lay = importlib.import_module(f'{PKG}.s6_layer')
            ops = importlib.import_module(f'{PKG}.s6_ops')
            self.mods = [oa.LatentAttention(model.layers[l], self.w[l]['qkv'], self.w[l]['o'], model.cos_sin, s.window)
                         for l in range(s.layers)]
            self.caches = [oa.PagedCaches(model.main[l], model.l1[l], model.latent_table, model.exact[l],
                                          model.exact_table) for l in range(s.layers)]
            self.sctx = lay.StepContext(model.positions, model.qsl, model.seq_lens, 1, B, model.tables, model.scale,
                                        ops.B200_BACKENDS, model.workspace, model.splits, window=s.window)

    def weight_bytes_per_step(self):
        per_layer = sum(v.numel() * v.element_size() for v in self.w[0].values())
        return per_layer * self.m.s.layers * self.m.s.loops

    def _rms(self, x, w):
        return self.torch.nn.functional.rms_norm(x, (x.shape[-1],), w, self.eps)

    def step(self):
        torch, F, m = self.torch, self.torch.nn.functional, self.m
        s, B, D = m.s, m.B, m.s.hidden
        main = torch.cuda.current_stream(m.device)
        stream = pkg_lib().stream_of(self.out)
        wstream = pkg_lib().ctypes.c_void_p(self.side.cuda_stream)
        hidden = self.x0
        states = [None] * s.layers
        for loop in range(s.loops):
            residual = None
            for layer in range(s.layers):
                W = self.w[layer]
                residual = hidden if residual is None else hidden + residual
                h = self._rms(residual, W['n1'])
                if self.dropin:
                    o, states[layer] = self.mods[layer].forward(m.positions, h, loop, states[layer], self.sctx,
                                                                self.caches[layer])
                    x = self._rms(o, W['n2'])
                    residual = x + residual
                    x = self._rms(residual, W['n3'])
                    gu = F.linear(x, W['gate_up'])
                    x = F.linear(F.silu(gu[:, :self.I]) * gu[:, self.I:], W['down'])
                    hidden = self._rms(x, W['n4'])
                    continue
                qkv = F.linear(h, W['qkv'])
                q, k, v = (x.view(B, s.heads, s.head_dim) for x in qkv.split(D, -1))
                self.side.wait_stream(main)               # the writer reads h
                h.record_stream(self.side)
                m.layer_loop(layer, loop, stream, wstream, io=(q, k, v, h, self.attn))
                x = self._rms(F.linear(self.attn.view(B, D), W['o']), W['n2'])
                residual = x + residual
                x = self._rms(residual, W['n3'])
                gu = F.linear(x, W['gate_up'])
                x = F.linear(F.silu(gu[:, :self.I]) * gu[:, self.I:], W['down'])
                hidden = self._rms(x, W['n4'])
            hidden = self._rms(hidden + residual, self.final)
        self.out.copy_(hidden)
        if not self.dropin:
            main.wait_stream(self.side)

    def capture(self):
        torch = self.torch
        warm = torch.cuda.Stream(self.m.device)
        warm.wait_stream(torch.cuda.current_stream(self.m.device))
        with torch.cuda.stream(warm):
            self.step()
        torch.cuda.current_stream(self.m.device).wait_stream(warm)
        torch.cuda.synchronize(self.m.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.step()
        return graph


def pkg_lib():
    return importlib.import_module(f'{PKG}._lib')


def run_full(args):
    """--config full: BASELINE config 2 as a whole Ouro-1.4B-shaped decode step (dense body included), one
    GPU per rank, weak scaling (64 sequences at ctx 8192 each)."""
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    pkg_lib().load()
    dec = importlib.import_module(f'{PKG}.decode')
    ctx, scaling, _, max_pos = config_batch(2, rank, world, args.seed)
    model = dec.S6DecodeModel(dec.OuroShape(max_position=max_pos), dec.DecodeBatch(ctx), device='cuda',
                              seed=args.seed + rank, window_overlap=WINDOW_MODES[args.side_window])
    native_ms = None
    if args.dropin:
        # the native step of the same build first, on the same model and weights, for comparison
        native = FullStep(model, args.seed + rank)
        ngraph = native.capture()
        for _ in range(args.warmup):
            ngraph.replay()
        native_ms = time_graph(torch, ngraph, args.steps, dist) / args.steps
        del ngraph
    full = FullStep(model, args.seed + rank, dropin=args.dropin)
    full.step()
    torch.cuda.synchronize()
    graph = full.capture()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms_total = time_graph(torch, graph, args.steps, dist)
    clocks = clk.summary()
    ms_step = ms_total / args.steps
    tokens_all = len(ctx) * world
    # e2e: the step's input embeddings in from pinned memory, its final hidden states out
    host_in = torch.empty(full.x0.shape, dtype=full.x0.dtype, pin_memory=True)
    host_in.copy_(full.x0)
    host_out = torch.empty(full.out.shape, dtype=full.out.dtype, pin_memory=True)
    stream = torch.cuda.current_stream()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 2)
    e0.record(stream)
    for _ in range(e2e_steps):
        full.x0.copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(full.out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / e2e_steps
    if dist is not None:
        t = torch.tensor([ms_e2e], device='cuda')
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    line = None
    if rank == 0:
        attn = model.latent_bytes_per_step() + model.window_bytes_per_step()
        wbytes = full.weight_bytes_per_step()
        peak, peak_kind = peaks()
        line = {
            'metric': METRIC, 'value': tokens_all / (ms_step / 1e3), 'unit': 'tokens/s', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded), random-init weights',
            'config': {'workload': 'BASELINE config 2: whole Ouro-1.4B-shaped S6 decode step - the dense body '
                                   '(RMSNorms, QKV / O projections, SiLU MLP 5632; torch/cuBLAS bf16) around the B200 '
                                   'attention path, 24 layers x 4 loops, one CUDA graph' +
                                   ('; attention through the drop-in mirror of the adapter\'s per-layer path '
                                    '(ouro_attention.LatentAttention over s6_layer.StepContext / attend, as '
                                    'hla/vllm_latent/ouro_latent.py:106-131 calls them)' if args.dropin else ''),
                       'global_batch': tokens_all, 'batch_per_gpu': len(ctx), 'ctx': max(ctx), 'seq_len': max(ctx) + 1,
                       'parallelism': f'request-partitioned x{world} (no collectives)',
                       'l2': 'inputs larger than L2 (latent caches ~40 GB, dense weights 2.5 GB per GPU), no flush'},
            'step_bytes': {'latent_and_window': attn, 'dense_weights': wbytes,
                           'frac_of_peak_in_step': (attn + wbytes) / (ms_step / 1e3) / 1e9 / peak},
            'roofline': {'bound': 'hbm', 'kernel': 'whole step (attention latent/window bytes + dense weights)',
                         'achieved': (attn + wbytes) / (ms_step / 1e3) / 1e9, 'peak': peak, 'unit': 'GB/s',
                         'frac': (attn + wbytes) / (ms_step / 1e3) / 1e9 / peak, 'peak_source': peak_kind,
                         'traffic': None},
            'cpu_baseline': None,
            'e2e': {'value': tokens_all / (ms_e2e / 1e3), 'unit': 'tokens/s',
                    'h2d_bytes_per_step': host_in.numel() * host_in.element_size(),
                    'd2h_bytes_per_step': host_out.numel() * host_out.element_size(),
                    'path': 'FullStep graph: input embeddings copied in from pinned memory, final hidden states out'},
            'gpu_launches': model.launches_per_step() * args.steps,
            'clocks': clocks}
        if args.dropin:
            line['native_step'] = {'ms_per_step': native_ms, 'value': tokens_all / (native_ms / 1e3),
                                   'note': 'the same step with the attention through S6DecodeModel.layer_loop '
                                           '(writer on a forked branch, prepare, history split, combine)'}
            # per (layer, loop): writer, latent query, exact RoPE + append, history split, combine; plus the
            # row commits at loops 0 and 3
            sh = model.s
            line['gpu_launches'] = (5 * sh.layers * sh.loops + 2 * sh.layers) * args.steps
        print(json.dumps(line), flush=True)
    del graph
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return line


def run_prefill(args):
    """--config 3: the writer of a prompt step (8 x 4096 tokens per GPU, weak scaling)."""
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    importlib.import_module(f'{PKG}._lib').load()
    dec = importlib.import_module(f'{PKG}.decode')
    pre = importlib.import_module(f'{PKG}.prefill')
    shape = dec.OuroShape()
    model = pre.PrefillWriter(shape, 8, 4096, device='cuda', seed=args.seed + rank)
    torch.cuda.synchronize()
    model.step()
    graph = model.capture()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms_total = time_graph(torch, graph, args.steps, dist)
    clocks = clk.summary()
    ms_step = ms_total / args.steps
    rows_all = model.rows_per_step() * world
    value = rows_all / (ms_step / 1e3)
    flops = model.flops_per_step()
    achieved = flops / (ms_step / 1e3) / 1e12
    peak, peak_kind = tensor_peak()
    traffic = None
    tr = ncu_traffic()
    if tr:
        traffic = tr.get('writer_tc_avg_bytes_per_launch_config3')

    # ---- e2e: the four loops' hidden states in from pinned memory, the last layer's main cache out
    host_in = torch.empty(model.h.shape, dtype=model.h.dtype, pin_memory=True)
    host_in.copy_(model.h)
    out_dev = model.main[-1]
    host_out = torch.empty(out_dev.shape, dtype=out_dev.dtype, pin_memory=True)
    stream = torch.cuda.current_stream()
    io_graph = model.capture_io(host_in, host_out, out_dev)   # each loop's copy-in overlaps the previous loop
    for _ in range(2):
        io_graph.replay()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 4)
    e0.record(stream)
    for _ in range(e2e_steps):
        io_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / e2e_steps
    if dist is not None:
        t = torch.tensor([ms_e2e], device='cuda')
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = {'value': rows_all / (ms_e2e / 1e3), 'unit': 'rows/s',
           'h2d_bytes_per_step': host_in.numel() * host_in.element_size(),
           'd2h_bytes_per_step': host_out.numel() * host_out.element_size(),
           'path': 'PrefillWriter.step_io CUDA graph (hla_s6_writer_project / hla_s6_writer_commit): each loop\'s '
                   'hidden states copied in from pinned memory on a copy stream during the previous loop, the last '
                   'layer\'s main latent cache read back at the end'}
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cores = use_all_host_threads()
            cs = PrefillCpuSample(shape, model.T, args.cpu_tokens, seed=args.seed)
            secs = [cs.pass_seconds() for _ in range(3)]
            cpu = {'value': len(secs) * args.cpu_tokens / sum(secs), 'unit': 'rows/s', 'cores': cores,
                   'kind': 'port', 'sample': cs.describe() + f'; {len(secs)} timed passes',
                   'sample_ms': [round(x * 1e3, 3) for x in secs], 'extrapolated': False}
        line = {
            'metric': METRIC3, 'value': value, 'unit': 'rows/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded), random-init weights',
            'config': prefill_config(world),
            'writer': {'flops_per_step': flops, 'bytes_per_step': model.bytes_per_step(),
                       'GBps_in_step': model.bytes_per_step() / (ms_step / 1e3) / 1e9},
            'roofline': {'bound': 'tensor', 'kernel': 'writer_tc2_kernel (CTA-pair tcgen05 GEMM + epilogue; 96 launches per step, the whole step)',
                         'achieved': achieved, 'peak': peak, 'unit': 'TFLOP/s', 'frac': achieved / peak,
                         'peak_source': peak_kind, 'ms_per_launch': ms_step / model.launches_per_step(),
                         'flops_per_launch': flops / model.launches_per_step(), 'traffic': traffic},
            'cpu_baseline': cpu,
            'e2e': e2e,
            'gpu_launches': model.launches_per_step() * args.steps,
            'clocks': clocks,
        }
        print(json.dumps(line), flush=True)
    model.graph = model.io_graph = None
    del graph, io_graph
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return line


def _events_ms(torch, fn, reps):
    """Device time of ``reps`` calls of fn on the current stream (ms per call), synchronized around."""
    st = torch.cuda.current_stream()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(reps):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_contig(args):
    """--config contig: the contiguous-layout reader of the HF engines (fused_history.history_attention)
    at config-2 scale - 64 rows, 8160 visible keys (ctx 8192 minus the 32-row window) - for the 96
    reads of a decode step (24 layers x 3 reads at width 512 + 1 at width 256), one GPU."""
    import numpy as np
    import torch
    rank, world, local = dist_env()
    if world > 1 and rank != 0:
        return None
    torch.cuda.set_device(local)
    importlib.import_module(f'{PKG}._lib').load()
    fh = importlib.import_module(f'{PKG}.fused_history')
    dec = importlib.import_module(f'{PKG}.decode')
    s = dec.OuroShape()
    B, N, H = 64, 8192 - s.window, s.heads
    g = torch.Generator(device='cuda').manual_seed(args.seed)
    kv = {w: [(torch.randn(B, N, w, generator=g, device='cuda').to(torch.bfloat16),
               torch.randn(B, N, w, generator=g, device='cuda').to(torch.bfloat16)) for _ in range(s.layers)]
          for w in (s.rank, s.rank1)}
    q = {w: torch.randn(B, H, w, generator=g, device='cuda').to(torch.bfloat16) for w in (s.rank, s.rank1)}
    mask = torch.ones(B, N, dtype=torch.bool, device='cuda')
    scale = s.head_dim ** -0.5

    def step():
        for loop in range(s.loops):
            w = s.rank1 if loop == 0 else s.rank
            for layer in range(s.layers):
                k, v = kv[w][layer]
                fh.history_attention(q[w], k, v, mask, scale)

    step()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    with ClockSampler(local) as clk:
        ms = time_graph(torch, graph, args.steps, None) / args.steps
    bytes_step = s.layers * B * N * 2 * 2 * ((s.loops - 1) * s.rank + s.rank1)
    peak, peak_kind = peaks()
    achieved = bytes_step / (ms / 1e3) / 1e9
    # e2e: q and mask in from pinned memory per loop, z and lse out to pinned memory per read; the copies run
    # on their own streams (copy-in one loop ahead, copy-out behind each read), pipelined with the reads
    hq = {w: q[w].cpu().pin_memory() for w in q}
    hm = mask.cpu().pin_memory()
    reads = [(s.rank1 if loop == 0 else s.rank, layer) for loop in range(s.loops) for layer in range(s.layers)]
    hz = [torch.empty(B, H, w, dtype=torch.bfloat16, pin_memory=True) for w, _ in reads]
    hl = [torch.empty(B, H, dtype=torch.float32, pin_memory=True) for _ in reads]
    dq = {w: torch.empty_like(q[w]) for w in q}
    dm = torch.empty_like(mask)
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    keep = []

    def e2e_step():
        main = torch.cuda.current_stream()
        keep.clear()
        h2d.wait_stream(main)
        d2h.wait_stream(main)
        for loop in range(s.loops):
            w = s.rank1 if loop == 0 else s.rank
            with torch.cuda.stream(h2d):
                dq[w].copy_(hq[w], non_blocking=True)
                dm.copy_(hm, non_blocking=True)
            main.wait_stream(h2d)
            for layer in range(s.layers):
                i = loop * s.layers + layer
                k, v = kv[w][layer]
                z, lse = fh.history_attention(dq[w], k, v, dm, scale)
                d2h.wait_stream(main)
                with torch.cuda.stream(d2h):
                    hz[i].copy_(z, non_blocking=True)
                    hl[i].copy_(lse, non_blocking=True)
                keep.append((z, lse))     # outputs stay alive until their copy-out has run
            h2d.wait_stream(main)         # the next loop's copy-in waits for this loop's reads of dq / dm
        main.wait_stream(d2h)
    e2e_step()
    ms_e2e = _events_ms(torch, e2e_step, max(3, args.steps // 4))
    h2d = s.loops * (B * H * s.rank * 2 + B * N)
    d2h = s.layers * s.loops * B * H * (s.rank * 2 + 4)
    cpu = None
    if not args.no_cpu:
        from oracle import s6_oracle as orc
        use_all_host_threads()
        rows = 1
        kk = kv[s.rank][0][0][:rows].float().cpu().numpy()
        vv = kv[s.rank][0][1][:rows].float().cpu().numpy()
        qq = q[s.rank][:rows].float().cpu().numpy()
        mm = np.ones((rows, N), dtype=bool)
        orc.contiguous_history(qq, kk, vv, mm, scale, dt=np.float32)
        t0 = time.perf_counter()
        for _ in range(3):
            orc.contiguous_history(qq, kk, vv, mm, scale, dt=np.float32)
        sec_row = (time.perf_counter() - t0) / 3 / rows
        sec = sec_row * B * s.layers * ((s.loops - 1) + s.rank1 / s.rank)
        cpu = {'value': B / sec, 'unit': 'tokens/s', 'cores': cpu_threads(), 'kind': 'port', 'extrapolated': True,
               'sample': f'oracle numpy fp32 contiguous reader, {rows} of {B} rows at width {s.rank} x {N} keys, '
                         f'extrapolated to 96 reads of a step (the width-256 read scaled by width)'}
    line = {'metric': METRIC_CONTIG, 'value': B / (ms / 1e3), 'unit': 'tokens/s', 'n_gpus': 1, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded)',
            'config': {'workload': 'contiguous-layout latent history reader (fused_history.history_attention '
                                   'forward): 96 reads of a decode step, K/V [64, 8160, R] per layer, all keys '
                                   'visible', 'global_batch': B, 'keys': N, 'widths': [s.rank, s.rank1],
                       'l2': 'inputs larger than L2 (K/V ~38 GB), no flush'},
            'roofline': {'bound': 'hbm', 'kernel': 'history_split_kernel (contiguous front end) + reduce, the whole '
                                                   'step', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s',
                         'frac': achieved / peak, 'peak_source': peak_kind, 'bytes_per_step': bytes_step,
                         'traffic': None},
            'cpu_baseline': cpu,
            'e2e': {'value': B / (ms_e2e / 1e3), 'unit': 'tokens/s', 'h2d_bytes_per_step': h2d,
                    'd2h_bytes_per_step': d2h,
                    'path': 'fused_history.history_attention per read, q and mask copied in from pinned memory per '
                            'loop and z and lse copied out per read, on copy streams pipelined with the reads'},
            'gpu_launches': 2 * s.layers * s.loops * args.steps, 'clocks': clk.summary()}
    print(json.dumps(line), flush=True)
    return line


def run_heads(args):
    """--config heads: the per-head history reader of the LLA serving path (history_attention_kv,
    mla=True) at config-2 scale - 64 sequences at ctx 8192, 16 KV heads, rows [c (rank) | k_rope
    (d_rope)] - for the 4 loops of 6 layers (each layer's cache is read at every loop), one GPU."""
    import numpy as np
    import torch
    rank_, world, local = dist_env()
    if world > 1 and rank_ != 0:
        return None
    torch.cuda.set_device(local)
    importlib.import_module(f'{PKG}._lib').load()
    ops = importlib.import_module(f'{PKG}.s6_ops')
    B, H, page, ctx, layers, loops = 64, 16, 16, 8192, 6, 4
    r, dr = args.heads_rank, args.heads_rope
    Lk = r + dr
    pages = ctx // page
    nb = B * pages + 1
    g = torch.Generator(device='cuda').manual_seed(args.seed)
    caches = [torch.randn(nb, H, page, Lk, generator=g, device='cuda').to(torch.bfloat16) for _ in range(layers)]
    perm = torch.randperm(nb - 1, generator=torch.Generator().manual_seed(args.seed)).to(torch.int32) + 1
    table = perm.view(B, pages).cuda()
    ctx_t = torch.full((B,), ctx, dtype=torch.int32, device='cuda')
    q = torch.randn(B, H, Lk, generator=g, device='cuda').to(torch.bfloat16)
    props = torch.cuda.get_device_properties(local)
    splits = ops.num_kv_splits(ctx, B, 512, props.multi_processor_count)
    ws = ops.S6Workspace(H, r, B * splits)
    ws.ensure('cuda')
    scale = 128 ** -0.5

    def step():
        for _ in range(loops):
            for c in caches:
                ops.history_attention_kv(q, c, c[..., :r], table, ctx_t, scale, splits, ws, None, None, 'b200',
                                         mla=True)
    step()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    with ClockSampler(local) as clk:
        ms = time_graph(torch, graph, args.steps, None) / args.steps
    reads = layers * loops
    bytes_step = reads * B * H * ctx * Lk * 2
    peak, peak_kind = peaks()
    achieved = bytes_step / (ms / 1e3) / 1e9
    # e2e: q in from pinned memory per loop, o and lse out to pinned memory per read, on copy streams pipelined
    # with the reads (as in the contiguous reader's bench)
    hq = q.cpu().pin_memory()
    dq = torch.empty_like(q)
    ho = [torch.empty(B, H, r, dtype=torch.bfloat16, pin_memory=True) for _ in range(layers * loops)]
    hl = [torch.empty(H, B, dtype=torch.float32, pin_memory=True) for _ in range(layers * loops)]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    keep = []

    def e2e_step():
        main = torch.cuda.current_stream()
        keep.clear()
        h2d.wait_stream(main)
        d2h.wait_stream(main)
        for loop in range(loops):
            with torch.cuda.stream(h2d):
                dq.copy_(hq, non_blocking=True)
            main.wait_stream(h2d)
            for j, c in enumerate(caches):
                i = loop * layers + j
                o, lse = ops.history_attention_kv(dq, c, c[..., :r], table, ctx_t, scale, splits, ws, None, None,
                                                  'b200', mla=True)
                d2h.wait_stream(main)
                with torch.cuda.stream(d2h):
                    ho[i].copy_(o, non_blocking=True)
                    hl[i].copy_(lse, non_blocking=True)
                keep.append((o, lse))
            h2d.wait_stream(main)
        main.wait_stream(d2h)
    e2e_step()
    ms_e2e = _events_ms(torch, e2e_step, max(3, args.steps // 4))
    h2d = loops * B * H * Lk * 2
    d2h = reads * B * H * (r * 2 + 4)
    cpu = None
    if not args.no_cpu:
        from oracle import s6_oracle as orc
        use_all_host_threads()
        rows = 1   # sequences (each with its 16 heads) in the sample
        ids = table[:rows].cpu().numpy()
        kc = caches[0][torch.from_numpy(ids.reshape(-1)).long().cuda()].float().cpu().numpy()
        tab = np.arange(rows * pages, dtype=np.int32).reshape(rows, pages)
        qq = q[:rows].float().cpu().numpy()
        cc = np.full(rows, ctx, dtype=np.int32)
        orc.history_attention_kv(qq, kc, kc[..., :r], tab, cc, scale, dt=np.float32)
        reps = 10
        t0 = time.perf_counter()
        for _ in range(reps):
            orc.history_attention_kv(qq, kc, kc[..., :r], tab, cc, scale, dt=np.float32)
        sec = (time.perf_counter() - t0) / reps / rows * B * reads
        cpu = {'value': B / sec, 'unit': 'tokens/s', 'cores': cpu_threads(), 'kind': 'port', 'extrapolated': True,
               'sample': f'oracle numpy fp32 per-head reader, {rows} of {B} sequences (16 heads, ctx {ctx}), '
                         f'extrapolated to the {reads} reads of a step'}
    line = {'metric': METRIC_HEADS, 'value': B / (ms / 1e3), 'unit': 'tokens/s', 'n_gpus': 1, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded)',
            'config': {'workload': f'per-head paged history read MLA-style (LLA serving path): {reads} reads '
                                   f'({layers} layers x {loops} loops), B={B}, ctx {ctx}, {H} KV heads, rows '
                                   f'[{r} | {dr}]', 'global_batch': B, 'ctx': ctx, 'rank': r, 'd_rope': dr,
                       'splits': splits, 'l2': 'inputs larger than L2 (per-head caches ~%d GB), no flush' %
                       round(layers * nb * H * page * Lk * 2 / 1e9)},
            'roofline': {'bound': 'hbm', 'kernel': 'history_heads_split_kernel + reduce, the whole step',
                         'achieved': achieved, 'peak': peak, 'unit': 'GB/s', 'frac': achieved / peak,
                         'peak_source': peak_kind, 'bytes_per_step': bytes_step, 'traffic': None},
            'cpu_baseline': cpu,
            'e2e': {'value': B / (ms_e2e / 1e3), 'unit': 'tokens/s', 'h2d_bytes_per_step': h2d,
                    'd2h_bytes_per_step': d2h,
                    'path': 's6_ops.history_attention_kv(mla=True) per read, q copied in from pinned memory per '
                            'loop and o and lse copied out per read, on copy streams pipelined with the reads'},
            'gpu_launches': 2 * reads * args.steps, 'clocks': clk.summary()}
    print(json.dumps(line), flush=True)
    return line


def run_export(args):
    """--config export: the rollout cache export of one finished 8192-token request over 24 layers
    (cache_export.export_rows: one gather launch, one pinned copy out), one GPU."""
    import numpy as np
    import torch
    rank, world, local = dist_env()
    if world > 1 and rank != 0:
        return None
    torch.cuda.set_device(local)
    lib = importlib.import_module(f'{PKG}._lib')
    lib.load()
    ce = importlib.import_module(f'{PKG}.cache_export')
    dec = importlib.import_module(f'{PKG}.decode')
    s = dec.OuroShape()
    L, bs, length = s.layers, s.page, 8192
    need = length // bs
    nb = 4 * need                          # the request's blocks among others' (shuffled)
    g = torch.Generator(device='cuda').manual_seed(args.seed)
    main = [torch.randn(nb, 1, bs, 2 * s.rank, generator=g, device='cuda').to(torch.bfloat16) for _ in range(L)]
    l1 = [torch.randn(nb, 1, bs, 2 * s.rank1, generator=g, device='cuda').to(torch.bfloat16) for _ in range(L)]
    rng = np.random.default_rng(args.seed)
    mb = torch.from_numpy(rng.permutation(nb)[:need].astype(np.int32)).cuda()
    lb = torch.from_numpy(rng.permutation(nb)[:need].astype(np.int32)).cuda()
    W = 2 * s.rank + 2 * s.rank1
    out = torch.empty(L, length, W, dtype=torch.bfloat16, device='cuda')
    mp = lib.pointer_array([c.data_ptr() for c in main])
    lp = lib.pointer_array([c.data_ptr() for c in l1])
    st = lib.stream_of(out)

    def gather():
        lib.call('hla_s6_export_rows', mp, lp, L, nb, main[0].stride(0), main[0].stride(2), 2 * s.rank, bs,
                 lib.ptr(mb), mb.numel(), nb, l1[0].stride(0), l1[0].stride(2), 2 * s.rank1, bs, lib.ptr(lb),
                 lb.numel(), length, lib.ptr(out), None, st)
    for _ in range(args.warmup):
        gather()
    with ClockSampler(local) as clk:
        ms = _events_ms(torch, gather, args.steps)
    bytes_step = 2 * L * length * W * 2          # read + write
    peak, peak_kind = peaks()
    achieved = bytes_step / (ms / 1e3) / 1e9
    for _ in range(2):
        ce.export_rows(main, l1, mb, lb, length, bs)
    ms_e2e = _events_ms(torch, lambda: ce.export_rows(main, l1, mb, lb, length, bs), max(3, args.steps // 10))
    cpu = None
    if not args.no_cpu:
        from oracle import s6_oracle as orc
        layers = 2
        mh = [m.view(torch.int16).cpu().numpy() for m in main[:layers]]   # bf16 bits: a byte copy
        lh = [x.view(torch.int16).cpu().numpy() for x in l1[:layers]]
        mbh, lbh = mb.cpu().numpy(), lb.cpu().numpy()
        orc.export_rows(mh, lh, mbh, lbh, bs, length)
        t0 = time.perf_counter()
        for _ in range(3):
            orc.export_rows(mh, lh, mbh, lbh, bs, length)
        sec = (time.perf_counter() - t0) / 3 * (L / layers)
        cpu = {'value': L * length / sec, 'unit': 'rows/s', 'cores': 1, 'kind': 'port', 'extrapolated': True,
               'sample': f'oracle numpy gather (the reference exporter\'s indexing) of {layers} of {L} layers, '
                         f'host-resident caches, extrapolated'}
    line = {'metric': METRIC_EXPORT, 'value': L * length / (ms / 1e3), 'unit': 'rows/s', 'n_gpus': 1,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded)',
            'config': {'workload': 'rollout cache export gather of one finished request: 24 layers x 8192 positions '
                                   'x (1024 main + 512 loop-1) bf16, shuffled blocks', 'length': length,
                       'layers': L, 'l2': 'caches 1.2 GB (larger than L2), no flush'},
            'roofline': {'bound': 'hbm', 'kernel': 'export_rows_kernel', 'achieved': achieved, 'peak': peak,
                         'unit': 'GB/s', 'frac': achieved / peak, 'peak_source': peak_kind,
                         'bytes_per_step': bytes_step, 'traffic': None},
            'cpu_baseline': cpu,
            'e2e': {'value': L * length / (ms_e2e / 1e3), 'unit': 'rows/s', 'h2d_bytes_per_step': 2 * need * 4,
                    'd2h_bytes_per_step': L * length * W * 2,
                    'path': 'cache_export.export_rows: block lists in, rows out into pinned host memory'},
            'gpu_launches': args.steps, 'clocks': clk.summary()}
    print(json.dumps(line), flush=True)
    return line


# ----------------------------------------------------------------------------- profiler workloads
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


def run_profile(args):
    """--profile CASE: a few eager steps of one workload, small enough for ncu (a few GB on the device).

    decode     the launches per (layer, loop) of S6DecodeModel.step in order (writer, prepare, history
               split, combine, plus the side-stream exact part and window for batches whose fused combine would
               exceed one wave; loop 0 reads the 256-wide latent, loops 1-3 the 512-wide one), so
               ``ncu -k regex:history_split -s 1 -c 2`` selects one launch of each width (2 layers: ~3 GB)
    prefill    the config-3 prompt-step writer (prefill.PrefillWriter: four writer launches per layer,
               N = 512 at loop 0 and 1024 at loops 1-3, 4096 tokens per prompt; 1 layer x 8 prompts: ~1 GB)
    seq-split  rank 0's share of an --split N-way sequence split (config 5: --batch 4 --ctx 131072) as a
               one-rank job: the latent rows of the first of N page slices, the reduce with its peer-store
               exchange (to this GPU only) and the one-part poll in the combine; with --time it also
               times the step and its history launches alone as CUDA graphs
    contig / heads / export   two calls of the other readers at the config-2 shape
    """
    import torch
    dec = importlib.import_module(f'{PKG}.decode')
    importlib.import_module(f'{PKG}._lib').load()
    case = args.profile
    if case in ('contig', 'heads', 'export'):
        return _profile_reader(args, torch)
    if case == 'seq-split':
        import torch.distributed as dist
        dist.init_process_group('gloo', init_method='tcp://127.0.0.1:29531', rank=0, world_size=1)
        shape = dec.OuroShape(layers=args.layers, max_position=args.ctx + 128)
        ctx = [args.ctx] * args.batch
        split = dec.seq_split_rows([c - shape.window for c in ctx], shape.page, 0, args.split)
        model = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=0,
                                  latent_rows=[n for _, n in split], exchange=(0, 1, dist.group.WORLD))
        for _ in range(args.profile_steps):
            model.step(overlap_writer=False)
        torch.cuda.synchronize()
        if args.time:
            ms, ms_hist = _graph_ms(torch, model.capture(), 20), _graph_ms(torch, model.capture_history(), 20)
            loops = shape.layers * shape.loops
            print(f'1/{args.split} slice: step {ms:.3f} ms, history launches alone {ms_hist:.3f} ms, the rest '
                  f'{(ms - ms_hist) / loops * 1e3:.1f} us per (layer, loop)')
            model.graph = model.history_graph = None
        model.close_exchange()
        dist.destroy_process_group()
        print(f'ok: {args.profile_steps} steps of a 1/{args.split} sequence-split slice, '
              f'{model.launches_per_step()} launches each')
        return
    if case == 'prefill':
        pre = importlib.import_module(f'{PKG}.prefill')
        model = pre.PrefillWriter(dec.OuroShape(layers=args.layers), args.prompts, 4096, device='cuda', seed=0)
        for _ in range(args.profile_steps):
            model.step()
        torch.cuda.synchronize()
        print(f'ok: {args.profile_steps} prefill steps, {model.launches_per_step()} launches each')
        return
    model = dec.S6DecodeModel(dec.OuroShape(layers=args.layers, max_position=max(65536, args.ctx + 128)),
                              dec.DecodeBatch([args.ctx] * args.batch),
                              device='cuda', seed=0)
    for _ in range(args.profile_steps):
        model.step(overlap_writer=False)
    torch.cuda.synchronize()
    print(f'ok: {args.profile_steps} steps, {model.launches_per_step()} launches each')


def _profile_reader(args, torch):
    B, ctx = args.batch, args.ctx
    g = torch.Generator(device='cuda').manual_seed(0)
    if args.profile == 'contig':
        fh = importlib.import_module(f'{PKG}.fused_history')
        N = ctx - 32
        k = torch.randn(B, N, 512, generator=g, device='cuda').to(torch.bfloat16)
        v = torch.randn(B, N, 512, generator=g, device='cuda').to(torch.bfloat16)
        q = torch.randn(B, 16, 512, generator=g, device='cuda').to(torch.bfloat16)
        mask = torch.ones(B, N, dtype=torch.bool, device='cuda')
        for _ in range(2):
            fh.history_attention(q, k, v, mask, 128 ** -0.5)
    elif args.profile == 'heads':
        ops = importlib.import_module(f'{PKG}.s6_ops')
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
        ce = importlib.import_module(f'{PKG}.cache_export')
        need = ctx // 16
        nb = 4 * need
        main = [torch.randn(nb, 1, 16, 1024, generator=g, device='cuda').to(torch.bfloat16) for _ in range(24)]
        l1 = [torch.randn(nb, 1, 16, 512, generator=g, device='cuda').to(torch.bfloat16) for _ in range(24)]
        mb = torch.randperm(nb, device='cuda')[:need].to(torch.int32)
        lb = torch.randperm(nb, device='cuda')[:need].to(torch.int32)
        for _ in range(2):
            ce.export_rows(main, l1, mb, lb, ctx, 16)
    torch.cuda.synchronize()
    print(f'ok: 2 calls of the {args.profile} reader')


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=100)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--config', default='2', choices=['2', '3', '4', '5', 'full', 'contig', 'export', 'heads'])
    ap.add_argument('--heads-rank', type=int, default=128, help='--config heads: latent rank r of the LLA rows')
    ap.add_argument('--heads-rope', type=int, default=32, help='--config heads: RoPE tail d_rope of the LLA rows')
    ap.add_argument('--seed', type=int, default=0)
    ap.add_argument('--cpu-reps', type=int, default=8,
                    help='tokens (one sequence each, every layer and loop) timed by the CPU baseline leg')
    ap.add_argument('--cpu-tokens', type=int, default=4096, help='tokens of the config-3 CPU oracle sample')
    ap.add_argument('--exchange', default='peer', choices=['peer', 'nccl'],
                    help='config 5 on several GPUs: how the (z, lse) parts move')
    ap.add_argument('--no-cpu', action='store_true', help='skip the CPU baseline leg')
    ap.add_argument('--side-window', default='auto', choices=sorted(WINDOW_MODES),
                    help='decode configs: exact part and window on a side stream beside the history split '
                         '(S6DecodeModel window_overlap; auto = when the fused combine would exceed one wave)')
    ap.add_argument('--dropin', action='store_true',
                    help='--config full: run the attention through the drop-in mirror of the adapter (ouro_attention)')
    prof = ap.add_argument_group('profiler workloads (--profile CASE; no JSON line, for ncu)')
    prof.add_argument('--profile', choices=['decode', 'prefill', 'seq-split', 'contig', 'heads', 'export'])
    prof.add_argument('--profile-steps', type=int, default=2, help='eager steps of the profiled workload')
    prof.add_argument('--layers', type=int, default=2)
    prof.add_argument('--batch', type=int, default=64)
    prof.add_argument('--ctx', type=int, default=8192)
    prof.add_argument('--prompts', type=int, default=8)
    prof.add_argument('--split', type=int, default=2, help='--profile seq-split: ways of the sequence split')
    prof.add_argument('--time', action='store_true', help='--profile seq-split: also time the step as CUDA graphs')
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
        return
    if args.warmup < 3:
        raise SystemExit('--warmup must be >= 3')
    if args.config == 'full':
        if args.impl == 'reference':
            args.config = 2          # the CPU arm times the same attention path per token (dense body excluded)
            run_reference(args)
            return
        run_full(args)
        return
    if args.config in ('contig', 'export', 'heads'):
        if args.impl == 'reference':
            print(json.dumps({'impl': 'reference', 'unavailable': f'--config {args.config} has no reference arm; '
                              'its line carries the oracle as cpu_baseline'}), flush=True)
            return
        {'contig': run_contig, 'export': run_export, 'heads': run_heads}[args.config](args)
        return
    args.config = int(args.config)
    if args.impl == 'reference':
        run_reference(args)
    elif args.config == 3:
        run_prefill(args)
    else:
        run_ours(args)


if __name__ == '__main__':
    main()
