"""TEST INFRASTRUCTURE: time the reference's own torch CPU path of one decode token against this repository's
numpy oracle port (the CPU arm that bench.py runs), on the same host and thread count.

bench.py's reference arm has to time the oracle port: the reference checkout is not importable where the bench
runs.  This script, run where a checkout exists, measures how the port's time per token compares with the
reference's torch implementation of the same work, so the bench's CPU number can be read against the
reference itself.

Per (layer, loop), both sides do the CPU composition of s6_layer.attend's decode step (the reference's GPU-only
FA2 window replaced by its own torch window path, as its CPU tests do - s6_ops.py:234-259, 290-314, 353-361):
the writer projection (register.py:45-61), the latent query (s6_layer.py:32-40 with latent_rope('torch')), the
causal chunk over the current token + the window history of W = 32 exact rows + merge_lse, the paged latent
history (s6_ops.py:204-222, torch backend), the B up-projection (s6_layer.py:114) and merge_states('torch').
One token of one sequence at context --ctx; loop 0 at width 256, loops 1-3 at 512; a token is 24 x that.

    HLA_REFERENCE_ROOT=/path/to/checkout python oracle/time_reference_cpu.py [--ctx 8192] [--reps 5]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ctx', type=int, default=8192)
    ap.add_argument('--reps', type=int, default=5)
    ap.add_argument('--reference', default=os.environ.get('HLA_REFERENCE_ROOT'))
    args = ap.parse_args()
    if not args.reference:
        ap.error('pass --reference or set HLA_REFERENCE_ROOT to a checkout of the reference project')
    sys.path.insert(0, args.reference)
    import torch
    from hla.latent.register import LatentLayer
    from hla.vllm_latent import s6_layer, s6_ops

    H, d, page, W, hidden = 16, 128, 16, 32, 2048
    c = args.ctx
    g = torch.Generator().manual_seed(0)
    scale = 1 / math.sqrt(d)
    sl = LatentLayer(hidden, H, d, 4, 512, 512, 256)
    inv = s6_layer.latent_inv_freq(d, 1e6)
    tables = {w: s6_layer.latent_rope_table(c + 1, inv, w, torch.float32) for w in (512, 256)}
    pages = -(-(c + 1) // page)
    ctx_lat = max(c - W, 0)
    data = {}
    for w in (512, 256):
        data[w] = dict(cache=torch.randn(pages + 1, 1, page, 2 * w, generator=g),
                       exact=torch.randn(pages + 1, H, page, 2 * d, generator=g))
    table = torch.arange(1, pages + 1, dtype=torch.int32)[None]
    q_pre = torch.randn(1, H, d, generator=g)
    k = torch.randn(1, H, d, generator=g)
    v = torch.randn(1, H, d, generator=g)
    h = torch.randn(1, hidden, generator=g)
    qsl = torch.tensor([0, 1], dtype=torch.int32)
    positions = torch.tensor([c])
    invalid = torch.zeros(1, dtype=torch.bool)
    ctx_t = torch.tensor([c], dtype=torch.int32)
    ctx_lat_t = torch.tensor([ctx_lat], dtype=torch.int32)
    empty = torch.zeros(1, dtype=torch.bool)

    def reference_pass(loop):
        w = 256 if loop == 0 else 512
        D = data[w]
        sl.write1(h) if loop == 0 else sl.write_step(h, loop, None)
        A, B, _ = sl.readers(loop)
        q_lat = s6_layer.latent_query(q_pre, A, positions, tables[w], 'torch')
        o_c, lse_c = s6_ops.chunk_attention(q_pre, k, v, qsl, 1, invalid, scale, 'torch')
        o_w, lse_w = s6_ops.window_attention(q_pre, D['exact'], table, ctx_t, W, scale)
        o_c, lse_c = s6_ops.merge_lse(o_c, lse_c, o_w, lse_w)
        cache = D['cache']
        o_h, lse_h = s6_ops.history_attention(q_lat, cache, table, ctx_lat_t, scale, 1, None, None, None, 'torch',
                                              empty)
        o_h = torch.einsum('thr,hrd->thd', o_h, B)
        return s6_ops.merge_states(o_h, lse_h, o_c, lse_c, invalid, 'torch')

    bench = __import__('bench')
    dec = __import__('importlib').import_module('hybrid-latent-attention_b200.decode')
    port = bench.CpuSample(dec.OuroShape(), c, 1, seed=0)       # one layer: 4 passes

    def time_it(fn, reps):
        fn()
        out = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            out.append(time.perf_counter() - t0)
        return min(out), float(np.median(out))

    with torch.no_grad():
        ref_layer = time_it(lambda: [reference_pass(loop) for loop in range(4)], args.reps)
    port_layer = time_it(port.run, args.reps)
    line = {'ctx': c, 'torch_threads': torch.get_num_threads(), 'host_cpus': os.cpu_count(),
            'reference_torch_s_per_token': {'min': 24 * ref_layer[0], 'median': 24 * ref_layer[1]},
            'oracle_port_s_per_token': {'min': 24 * port_layer[0], 'median': 24 * port_layer[1]},
            'port_over_reference': port_layer[1] / ref_layer[1],
            'work': 'one decode token of one sequence: 24 layers x 4 loops (timed: one layer, x24)'}
    print(json.dumps(line))


if __name__ == '__main__':
    main()
