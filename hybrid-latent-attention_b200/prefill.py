"""The latent writer over a prompt batch through the B200 kernels.

Per step: for loop in 0..3, for layer in 0..23, the writer of one (layer, loop) of a prompt step
(s6_layer.write_rows, reference s6_layer.py:124-132 -> register.py:45-61) with its row commit
(s6_layer.committed_row + unified_kv_cache_update, ouro_latent.py:127-129):

  loop 0   first = E_1' h_1            [T, 512]  -> committed: loop-1 latent row (K 256 rotated | V 256)
  loop 1   reg   = E_2 h_2             [T, 1024]
  loop 2   reg   = bf16(reg + E_3 h_3) [T, 1024]
  loop 3   row   = bf16(reg + E_4 h_4) [T, 1024] -> committed: main latent row (K 512 rotated | V 512)

one launch each (hla_s6_writer_project / hla_s6_writer_commit), 96 per step.  T = 8 prompts x 4096
tokens = 32768 rows per GEMM: the tensor-core path of the writer (tcgen05, writer_tc.cu).

The attention inputs ``h`` of the four loops are synthetic (seeded N(0, 1)) and shared by the 24
layers, since the dense Ouro body that would make them differ is not part of the step; each is
128 MiB, larger than L2, and consecutive launches read different ones.  Committed rows land in
per-layer paged latent caches with a shuffled page table (block 0 is the null block).
"""
from __future__ import annotations

import math

import torch

from . import _lib, s6_layer
from .decode import OuroShape
from .latent import LatentLayer

BF16 = torch.bfloat16


class PrefillWriter:
    """Config-3 state and launches: ``prompts`` requests of ``prompt_len`` tokens each, positions
    0 .. prompt_len - 1."""

    def __init__(self, shape: OuroShape, prompts=8, prompt_len=4096, device='cuda', seed=0):
        self.s, self.device = shape, torch.device(device)
        s = shape
        if prompt_len > s.max_position:
            raise ValueError(f'prompt length {prompt_len} exceeds max_position {s.max_position}')
        self.R, self.L = prompts, prompt_len
        T = self.T = prompts * prompt_len
        g = torch.Generator(device=self.device).manual_seed(seed)
        gen = lambda *shape_, std=1.0: (torch.randn(*shape_, generator=g, device=self.device) * std).to(BF16)
        self.layers = []
        for _ in range(s.layers):
            lat = LatentLayer(s.hidden, s.heads, s.head_dim, s.loops, s.rank, s.rank, s.rank1)
            with torch.no_grad():
                lat = lat.to(self.device, BF16)
                for lin in (*lat.cand_s, lat.cand1):
                    lin.weight.copy_(gen(*lin.weight.shape, std=1 / math.sqrt(s.hidden)))
            self.layers.append(lat.requires_grad_(False))
        # ---- step metadata: R prompts, positions 0 .. L-1 each
        self.positions = torch.arange(prompt_len, dtype=torch.int64, device=self.device).repeat(prompts)
        self.qsl = torch.arange(0, T + 1, prompt_len, dtype=torch.int32, device=self.device)
        pages = -(-prompt_len // s.page)
        nb = prompts * pages + 1
        perm = torch.randperm(nb - 1, generator=torch.Generator().manual_seed(seed + 1)).to(torch.int32) + 1
        self.block_table = perm.view(prompts, pages).to(self.device)
        self.main = [torch.full((nb, 1, s.page, 2 * s.rank), float('inf'), dtype=BF16, device=self.device)
                     for _ in range(s.layers)]
        self.l1 = [torch.full((nb, 1, s.page, 2 * s.rank1), float('inf'), dtype=BF16, device=self.device)
                   for _ in range(s.layers)]
        inv = s6_layer.latent_inv_freq(s.head_dim, s.theta)
        self.tables = {w: s6_layer.latent_rope_table(s.max_position, inv, w, BF16).to(self.device)
                       for w in (s.rank, s.rank1)}
        # ---- activations and running registers
        self.h = gen(s.loops, T, s.hidden)
        self.reg = [torch.empty(T, 2 * s.rank, dtype=BF16, device=self.device) for _ in range(s.layers)]
        self.graph = None

    # ------------------------------------------------------------------ work
    def flops_per_step(self):
        """2 * T * hidden * (2 rank1 + 3 * 2 rank) per layer (one GEMM per loop)."""
        s = self.s
        return s.layers * 2 * self.T * s.hidden * (2 * s.rank1 + (s.loops - 1) * 2 * s.rank)

    def bytes_per_step(self):
        """Algorithmic HBM bytes: h and E read by every GEMM, the register written at loops 1-2 and
        read at loops 2-3, the committed rows written at loops 0 and 3."""
        s, T = self.s, self.T
        n = [2 * s.rank1] + [2 * s.rank] * (s.loops - 1)
        per_layer = sum(T * s.hidden * 2 + N * s.hidden * 2 for N in n)
        per_layer += 2 * T * 2 * s.rank * 2          # register out (loops 1, 2)
        per_layer += 2 * T * 2 * s.rank * 2          # register in (loops 2, 3)
        per_layer += T * 2 * (2 * s.rank1 + 2 * s.rank)  # committed rows
        return s.layers * per_layer

    def rows_per_step(self):
        """Committed cache rows (one main + one loop-1 latent row per token and layer, 3072 B)."""
        return self.T * self.s.layers

    def launches_per_step(self):
        return self.s.layers * self.s.loops

    def layer_loop(self, layer, loop, stream):
        s = self.s
        lat = self.layers[layer]
        E = lat.writer(loop)
        h = self.h[loop]
        T = self.T
        if loop == 0 or loop == s.loops - 1:
            width = s.rank1 if loop == 0 else s.rank
            cache = self.l1[layer] if loop == 0 else self.main[layer]
            table = self.tables[width]
            reg_in = None if loop == 0 else self.reg[layer]
            _lib.call('hla_s6_writer_commit', _lib.ptr(h), h.stride(0), _lib.ptr(E), E.stride(0), _lib.ptr(reg_in),
                      0 if reg_in is None else reg_in.stride(0), None, 0, T, E.shape[0], E.shape[1],
                      _lib.ptr(self.positions), _lib.ptr(table), table.stride(0), table.shape[0], _lib.ptr(cache),
                      cache.shape[0], cache.stride(0), cache.stride(2), s.page, _lib.ptr(self.block_table),
                      self.block_table.stride(0), self.block_table.shape[1], _lib.ptr(self.qsl), self.R, stream)
        else:
            reg = self.reg[layer]
            reg_in = None if loop == 1 else reg
            _lib.call('hla_s6_writer_project', _lib.ptr(h), h.stride(0), _lib.ptr(E), E.stride(0), _lib.ptr(reg_in),
                      0 if reg_in is None else reg_in.stride(0), _lib.ptr(reg), reg.stride(0), T, E.shape[0],
                      E.shape[1], stream)

    def step(self):
        stream = _lib.stream_of(self.h)
        for loop in range(self.s.loops):
            for layer in range(self.s.layers):
                self.layer_loop(layer, loop, stream)

    def step_io(self, host_in, host_out, out_src):
        """One prompt step fed from pinned host memory (``host_in``: ``h``'s shape, the four loops' hidden
        states) with ``out_src`` (a device tensor the step writes, e.g. a layer's latent cache) read back
        into ``host_out``.  Each loop's hidden states arrive on a copy stream and that loop's launches
        wait only for them, so loops 1-3 are copied in during the previous loop's writers; the read-back
        follows the last launch.  The results equal ``h.copy_(host_in); step(); host_out.copy_(out_src)``."""
        main = torch.cuda.current_stream(self.device)
        if getattr(self, '_io', None) is None:
            self._io = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
        h2d, d2h = self._io
        h2d.wait_stream(main)
        d2h.wait_stream(main)
        ready = []
        with torch.cuda.stream(h2d):
            for loop in range(self.s.loops):
                self.h[loop].copy_(host_in[loop], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                ready.append(ev)
        stream = _lib.stream_of(self.h)
        for loop in range(self.s.loops):
            main.wait_event(ready[loop])
            for layer in range(self.s.layers):
                self.layer_loop(layer, loop, stream)
        d2h.wait_stream(main)
        with torch.cuda.stream(d2h):
            host_out.copy_(out_src, non_blocking=True)
        main.wait_stream(h2d)
        main.wait_stream(d2h)

    def capture_io(self, host_in, host_out, out_src):
        """``step_io`` captured as one CUDA graph (copies and kernels)."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.step_io(host_in, host_out, out_src)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.io_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.io_graph):
            self.step_io(host_in, host_out, out_src)
        return self.io_graph

    def capture(self):
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        return self.graph
