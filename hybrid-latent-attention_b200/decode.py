"""A whole S6 decode step of an Ouro-1.4B-shaped model through the B200 kernels.

Per step: for loop in 0..3, for layer in 0..23 (the hot loop of hla/vllm_latent/ouro_latent.py:270-274),
one (layer, loop) of OuroLatentAttention.forward (ouro_latent.py:106-131) without the dense projections:

  1. writer (+ commit)       s6_layer.write_rows (register.py:45-61); at loops 0 and 3 the committed
                             row (s6_layer.committed_row + unified_kv_cache_update, ouro_latent.py:127-129)
                             is written by the same kernel's epilogue
  2. prepare                 ctx.latent_query (s6_layer.py:32-40, 82-84) + rotary_emb and the exact
                             unified_kv_cache_update (ouro_latent.py:113-123), one launch
  3. history split           s6_ops.history_attention stage 1 (s6_ops.py:117-161)
  4. fused combine           window_attention_fa + stage 2 + einsum B + merge_states (s6_layer.py:97-115)

The inputs of a (layer, loop) - pre-RoPE q, k, v and the attention input h - come from a resident
activation buffer (synthetic, seeded); its output goes to an output buffer.  Caches are paged with
a shuffled page table (block 0 is the null block); the exact window cache keeps only the pages a
W-row sliding window touches, as vLLM's sliding-window KV manager does for the reference.

``step()`` issues the launches eagerly; ``capture()`` records one step as a CUDA graph (what the
reference's FULL_DECODE_ONLY serving replays) and ``replay()`` runs it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import _lib, s6_layer, s6_ops
from .latent import LatentLayer

BF16 = torch.bfloat16


@dataclass
class OuroShape:
    """Ouro-1.4B geometry (hla/vendor/config.json) and the S6 student widths (register.py:98-100)."""
    layers: int = 24
    hidden: int = 2048
    heads: int = 16
    head_dim: int = 128
    loops: int = 4
    rank: int = 512
    rank1: int = 256
    page: int = 16
    window: int = 32
    theta: float = 1e6
    max_position: int = 65536


def step_arrangement(requests, heads, sms, sequence_split):
    """Default arrangement of a decode step's launches for ``requests`` rows on a GPU with ``sms`` SMs:
    ``(window_overlap, reduce_first)``.  The side-stream exact part and window pay when the fused
    combine's grid (heads x ceil(requests / 8) CTAs, one per SM) would exceed one wave; the reduce before
    the combine pays when the history split (2 CTAs per SM) leaves more than about 16 partials per row.
    Neither is used with a sequence split, whose reduce and combine exchange parts between GPUs."""
    if sequence_split:
        return False, False
    return heads * -(-requests // 8) > sms, 2 * sms > 16 * requests


def seq_split_rows(latent_rows, page, rank, world):
    """Sequence split of each request's latent history across ``world`` GPUs by whole pages: rank r holds
    pages ``[r * P // world, (r + 1) * P // world)`` of a request with P pages.  Returns, per request,
    ``(first_page, rows)``; the slices of all ranks tile the history exactly."""
    out = []
    for n in latent_rows:
        pages = -(-int(n) // page)
        p0, p1 = rank * pages // world, (rank + 1) * pages // world
        rows = max(0, min(int(n), p1 * page) - p0 * page)
        out.append((p0, rows))
    return out


@dataclass
class DecodeBatch:
    """Per-request history lengths (tokens before the current one)."""
    ctx: list = field(default_factory=lambda: [8192] * 64)


class S6DecodeModel:
    """Decode-step state and launches.

    ``latent_rows`` (optional, per request) is the number of latent history rows this GPU holds; by
    default every request's whole latent history ``ctx - W``.  ``exchange = (rank, world, group)``
    turns on the sequence split: each GPU holds a contiguous slice of every request's latent pages,
    reduces its slice's partials to fp32 ``(z, lse)``, exchanges them and merges the ``world``
    parts in the combine (the window, query and writer work is replicated).  ``exchange_mode``:

    * ``'peer'`` (default): the reduce stores its part straight into every rank's receive slot over
      NVLink (CUDA IPC mappings of one exchange region per GPU: a slot per (layer, loop), each
      holding ``world`` parts) as tagged exchange words, which the combine polls.  No fence, flag or
      collective library call is on the step.
    * ``'nccl'``: the reduce writes a local part and an NCCL ``all_gather_into_tensor`` moves it.

    ``pdl`` (default on): the history split is launched as a programmatic dependent of the prepare
    (it streams pages while the prepare runs and reads q_lat after it), and the combine (or the
    sequence split's reduce) as one of the history split.  ``pdl=False`` serialises these launches
    (the library's stage-2 reduce kernels are always programmatic dependents of the split and wait for
    it before their first read); the results are bit-identical.

    ``window_overlap``: the exact part of the prepare (exact RoPE, exact-cache append) and the exact
    window run on a side stream, beside the history split, so that only the latent query stays ahead
    of the split; the combine takes the window as an external exact part (16 tokens per CTA when its
    grid exceeds one wave).  ``None`` (default) turns it on when the fused combine's grid (heads x
    ceil(B / 8) CTAs, one per SM) would exceed one wave, without a sequence split, and keeps the
    window inside the combine otherwise.  Measured on one GPU: 256 requests (config 4) 51.4 -> 47.1 ms
    per step, end to end with host copies 4999 -> 5269 tokens/s; 64 requests (config 2) within 0.7%
    on the device but 3% slower end to end (3963 -> 3850 tokens/s); 4 requests (config 5) unchanged.

    ``reduce_first``: the history split's partials are reduced by the block-cooperative reduce kernel
    into one fp32 part that the combine merges, instead of inside the combine (one warp per (row,
    head) walking all of the row's partials).  ``None`` (default) turns it on without a sequence split
    when the split leaves more than about 16 partials per row (fewer than ~18 requests on a B200).
    """

    def __init__(self, shape: OuroShape, batch: DecodeBatch, device='cuda', seed=0, split_max_tokens=512,
                 latent_rows=None, exchange=None, exchange_mode='peer', window_overlap=None, pdl=True,
                 reduce_first=None):
        self.s, self.device = shape, torch.device(device)
        self.pdl = pdl
        s = shape
        B = len(batch.ctx)
        self.B = B
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        auto_window, auto_reduce = step_arrangement(B, s.heads, sms, exchange is not None)
        self.window_overlap = bool(auto_window if window_overlap is None else window_overlap)
        self.reduce_first = bool(auto_reduce if reduce_first is None else reduce_first)
        g = torch.Generator(device=self.device).manual_seed(seed)
        gen = lambda *shape_, std=1.0, dtype=BF16: (torch.randn(*shape_, generator=g, device=self.device) * std).to(dtype)
        ctx = torch.tensor(batch.ctx, dtype=torch.int64)
        self.ctx_host = ctx
        if int(ctx.max()) + 1 > s.max_position:
            raise ValueError(f'context {int(ctx.max())} exceeds max_position {s.max_position}')
        # ---- weights: one latent student per layer (random init, bf16)
        self.layers = []
        for _ in range(s.layers):
            lat = LatentLayer(s.hidden, s.heads, s.head_dim, s.loops, s.rank, s.rank, s.rank1)
            with torch.no_grad():
                lat = lat.to(self.device, BF16)
                for p in (lat.q_absorb, lat.q_absorb1):
                    p.copy_(gen(*p.shape, std=1 / math.sqrt(s.head_dim)))
                lat.out_absorb.copy_(gen(*lat.out_absorb.shape, std=1 / math.sqrt(s.rank)))
                lat.out_absorb1.copy_(gen(*lat.out_absorb1.shape, std=1 / math.sqrt(s.rank1)))
                for lin in (*lat.cand_s, lat.cand1):
                    lin.weight.copy_(gen(*lin.weight.shape, std=1 / math.sqrt(s.hidden)))
            self.layers.append(lat.requires_grad_(False))
        # ---- step metadata (decode: one token per request)
        self.positions = ctx.to(self.device)
        self.qsl = torch.arange(B + 1, dtype=torch.int32, device=self.device)
        self.seq_lens = (ctx + 1).to(torch.int32).to(self.device)
        rows = (ctx - s.window).clamp(min=0) if latent_rows is None else torch.tensor(latent_rows, dtype=torch.int64)
        self.ctx_latent = rows.to(torch.int32).to(self.device)
        self.latent_rows = int(rows.sum())
        self.exchange = exchange
        # ---- latent caches: pages for rows [0, ctx] of every request (room for the committed row), shuffled;
        #      a sequence-split slice holds only its own rows (its commits fall outside the table: skipped)
        if latent_rows is None:
            lpages = [-(-(c + 1) // s.page) for c in batch.ctx]
        else:
            lpages = [max(1, -(-int(r) // s.page)) for r in latent_rows]
        self.lmax = max(lpages)
        self.emax = max(-(-(c + 1) // s.page) for c in batch.ctx)
        lnb = sum(lpages) + 1
        perm = torch.randperm(lnb - 1, generator=torch.Generator().manual_seed(seed + 1)).to(torch.int32) + 1
        ltab = torch.zeros(B, self.lmax, dtype=torch.int32)
        k = 0
        for r, n in enumerate(lpages):
            ltab[r, :n] = perm[k:k + n]
            k += n
        self.latent_table = ltab.to(self.device)
        self.main = [gen(lnb, 1, s.page, 2 * s.rank) for _ in range(s.layers)]
        self.l1 = [gen(lnb, 1, s.page, 2 * s.rank1) for _ in range(s.layers)]
        for c in (*self.main, *self.l1):
            c[0].fill_(float('inf'))   # null block: any read of it would be loud
        # ---- exact caches: only the pages of [ctx - W, ctx] exist per request
        etab = torch.zeros(B, self.emax, dtype=torch.int32)
        k = 1
        for r, c in enumerate(batch.ctx):
            for col in range(max(0, c - s.window) // s.page, c // s.page + 1):
                etab[r, col] = k
                k += 1
        self.exact_table = etab.to(self.device)
        self.exact = [[gen(k, s.page, s.heads, 2 * s.head_dim) for _ in range(s.loops)] for _ in range(s.layers)]
        self.exact_logical = [[e.transpose(1, 2) for e in row] for row in self.exact]
        # ---- RoPE tables
        inv = s6_layer.latent_inv_freq(s.head_dim, s.theta)
        self.tables = {w: s6_layer.latent_rope_table(s.max_position, inv, w, BF16).to(self.device)
                       for w in (s.rank, s.rank1)}
        ang = torch.arange(s.max_position).float()[:, None] * inv[None]
        self.cos_sin = torch.cat((ang.cos(), ang.sin()), -1).to(self.device)
        # ---- workspace and activations
        props = torch.cuda.get_device_properties(self.device)
        self.splits = s6_ops.num_kv_splits(s.max_position, B, split_max_tokens, props.multi_processor_count)
        self.workspace = s6_ops.S6Workspace(s.heads, s.rank, B * self.splits)
        self.ws = self.workspace.ensure(self.device)
        self.ws_floats = B * self.splits * s.heads * (s.rank + 1)
        D = s.heads * s.head_dim
        self.acts = gen(s.layers, s.loops, B, 3 * D + s.hidden)          # q | k | v | h per (layer, loop)
        self.out = torch.zeros(s.layers, s.loops, B, s.heads, s.head_dim, dtype=BF16, device=self.device)
        self.q_lat = torch.empty(B, s.heads, s.rank, dtype=BF16, device=self.device)
        self.q_rope = torch.empty(B, s.heads, s.head_dim, dtype=BF16, device=self.device)
        self.reg = [torch.empty(B, 2 * s.rank, dtype=BF16, device=self.device) for _ in range(s.layers)]
        self.exchange_mode = exchange_mode
        self.x_bases = None
        if self.reduce_first:          # the reduced history part (z fp32 [B, H, W], lse [H, B]) the combine merges
            self.zpart = torch.empty(B * s.heads * s.rank + s.heads * B, dtype=torch.float32, device=self.device)
        if exchange is not None and exchange_mode not in ('peer', 'nccl'):
            raise ValueError(f'unknown exchange mode {exchange_mode!r}')
        if exchange is not None and exchange_mode == 'peer':
            self._init_peer_exchange(*exchange)
        elif exchange is not None:
            world = exchange[1]
            part = B * s.heads * s.rank + s.heads * B          # z [B, H, W] then lse [H, B], W <= rank
            self.xsend = torch.empty(part, dtype=torch.float32, device=self.device)
            self.xrecv = torch.empty(world * part, dtype=torch.float32, device=self.device)
        self.scale = s.head_dim ** -0.5
        self.graph = None
        self.history_graph = None
        # exact-window part computed beside the history kernel (window_overlap): one buffer, reused by
        # every (layer, loop) - window i + 1 is ordered after prepare i + 1, which follows combine i
        self.win_o = torch.empty(B, s.heads, s.head_dim, dtype=BF16, device=self.device)
        self.win_lse = torch.empty(s.heads, B, dtype=torch.float32, device=self.device)
        self._win_stream = None

    # ------------------------------------------------------------------ peer exchange
    def _init_peer_exchange(self, rank, world, group):
        """One exchange region per GPU, mapped by every rank: ``slots x world`` parts of ``x_part``
        exchange words (z [B, H, rank] then lse [H, B]; 8 bytes each, zeroed so that no tag matches
        before the first exchange); plus two local counters per slot (its epoch, which tags the
        slot's exchanges, and the combine's CTA count).  A step cycles through all the slots, so a
        slot's next exchange follows every rank's combine of its previous one."""
        import ctypes
        import torch.distributed as dist
        s, B = self.s, self.B
        slots = s.layers * s.loops
        if slots < 2:
            raise ValueError('the peer exchange needs two or more (layer, loop) slots per step')
        self.x_part = -(-(B * s.heads * s.rank + s.heads * B) // 2) * 2
        self.x_region = slots * world * self.x_part * _lib.EXCHANGE_WORD_BYTES
        handle = ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
        base = ctypes.c_void_p()
        _lib.call('hla_s6_peer_alloc', self.x_region, ctypes.byref(base), handle)
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        bases = []
        try:
            for r in range(world):
                if r == rank:
                    bases.append(base.value)
                    continue
                peer = ctypes.c_void_p()
                _lib.call('hla_s6_peer_open', ctypes.create_string_buffer(handles[r], _lib.PEER_HANDLE_BYTES),
                          ctypes.byref(peer))
                bases.append(peer.value)
        except Exception:
            for r, b in enumerate(bases):
                _lib.call('hla_s6_peer_close' if r != rank else 'hla_s6_peer_free', ctypes.c_void_p(b))
            raise
        self.x_bases = bases
        self.x_counters = torch.zeros(2 * slots, dtype=torch.int32, device=self.device)

    def close_exchange(self):
        """Unmap the peers' regions and free this rank's (collective: every rank calls it, after its
        last step; no rank's memory is released while another may still write it)."""
        if self.x_bases is None:
            return
        import ctypes
        import torch.distributed as dist
        rank, world, group = self.exchange
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        for r, b in enumerate(self.x_bases):
            if r != rank:
                _lib.call('hla_s6_peer_close', ctypes.c_void_p(b))
        dist.barrier(group=group)
        _lib.call('hla_s6_peer_free', ctypes.c_void_p(self.x_bases[rank]))
        self.x_bases = None

    # ------------------------------------------------------------------ bytes
    def latent_bytes_per_step(self):
        """Algorithmic latent-history bytes of one step: every layer reads ctx_latent rows of the
        loop-1 latent (2 * rank1 bf16) at loop 0 and of the main latent (2 * rank bf16) at loops 1-3."""
        s = self.s
        return s.layers * self.latent_rows * 2 * (2 * s.rank1 + (s.loops - 1) * 2 * s.rank)

    def window_bytes_per_step(self):
        """Exact window bytes: W rows + the current row, K|V of every head, every loop and layer."""
        s = self.s
        rows = int(sum(min(c, s.window) + 1 for c in self.ctx_host.tolist()))
        return s.layers * s.loops * rows * s.heads * 2 * s.head_dim * 2

    # ------------------------------------------------------------------ launches
    def _views(self, layer, loop):
        s, B = self.s, self.B
        D = s.heads * s.head_dim
        a = self.acts[layer, loop]
        q = a[:, :D].view(B, s.heads, s.head_dim)
        k = a[:, D:2 * D].view(B, s.heads, s.head_dim)
        v = a[:, 2 * D:3 * D].view(B, s.heads, s.head_dim)
        h = a[:, 3 * D:]
        return q, k, v, h

    def _history(self, layer, loop, stream, flags=0):
        """The history split of one (layer, loop); ``flags=PARTIALS_AFTER_QUERY`` when the preceding launch
        on ``stream`` is this (layer, loop)'s prepare, which writes q_lat."""
        s, B = self.s, self.B
        A, _, width = self.layers[layer].readers(loop)
        cache = self.l1[layer] if loop == 0 else self.main[layer]
        q_lat = self.q_lat[..., :width] if width != s.rank else self.q_lat
        _lib.call('hla_s6_history_partials', _lib.ptr(q_lat), q_lat.stride(0), q_lat.stride(1), _lib.ptr(cache),
                  cache.shape[0], cache.stride(0), cache.stride(2), _lib.ptr(self.latent_table),
                  self.latent_table.stride(0), self.latent_table.shape[1], _lib.ptr(self.ctx_latent), B, s.heads,
                  width, s.page, float(self.scale), self.splits, _lib.ptr(self.ws), self.ws_floats, None, flags, stream)

    def layer_loop(self, layer, loop, stream, wstream=None, io=None):
        """The launches of one (layer, loop) (four, or six with the side-stream exact part and window); the
        writer goes to ``wstream`` when given (it reads only ``h`` and feeds only the commit and the next
        loop's writer, so it overlaps the attention chain).
        ``io = (q, k, v, h, out)`` takes the pre-RoPE q, k, v ``[B, H, d]`` (any token / head strides), the
        attention input ``h [B, hidden]`` and the output ``[B, H, d]`` from the caller - a dense body around
        the attention - instead of the resident activation and output buffers."""
        wstream = stream if wstream is None else wstream
        s, B = self.s, self.B
        lat = self.layers[layer]
        q, k, v, h = self._views(layer, loop) if io is None else io[:4]
        A, Bm, width = lat.readers(loop)
        table = self.tables[width]
        # 1. writer; at loop 0 (loop-1 latent) and the last loop (main latent) the row is committed in
        #    the epilogue.  The committed row sits at position ctx, which no history read of this step
        #    touches (they stop at ctx - W), so committing first equals the reference's commit-after-attend.
        E = lat.writer(loop)
        if loop == 0 or loop == s.loops - 1:
            cache = self.l1[layer] if loop == 0 else self.main[layer]
            reg_in = None if loop == 0 else self.reg[layer]
            _lib.call('hla_s6_writer_commit', _lib.ptr(h), h.stride(0), _lib.ptr(E), E.stride(0), _lib.ptr(reg_in),
                      0 if reg_in is None else reg_in.stride(0), None, 0, B, E.shape[0], E.shape[1],
                      _lib.ptr(self.positions), _lib.ptr(table), table.stride(0), table.shape[0], _lib.ptr(cache),
                      cache.shape[0], cache.stride(0), cache.stride(2), s.page, _lib.ptr(self.latent_table),
                      self.latent_table.stride(0), self.latent_table.shape[1], _lib.ptr(self.qsl), B, wstream)
        else:
            reg = self.reg[layer]
            reg_in = None if loop == 1 else reg
            _lib.call('hla_s6_writer_project', _lib.ptr(h), h.stride(0), _lib.ptr(E), E.stride(0), _lib.ptr(reg_in),
                      0 if reg_in is None else reg_in.stride(0), _lib.ptr(reg), reg.stride(0), B, E.shape[0],
                      E.shape[1], wstream)
        # 2. latent query from the pre-RoPE q + exact RoPE (q -> q_rope, k) + exact-cache append
        q_lat = self.q_lat[..., :width] if width != s.rank else self.q_lat
        ex = self.exact_logical[layer][loop]
        qr = self.q_rope

        def prepare(kv, flags, strm):
            k_, v_ = kv
            _lib.call('hla_s6_decode_prepare', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(A), A.stride(0),
                      A.stride(1), _lib.ptr(self.positions), _lib.ptr(table), table.stride(0), table.shape[0],
                      _lib.ptr(q_lat), q_lat.stride(0), q_lat.stride(1), B, s.heads, s.head_dim, width, _lib.ptr(qr),
                      qr.stride(0), qr.stride(1), _lib.ptr(k_), k.stride(0), k.stride(1), _lib.ptr(v_), v.stride(0),
                      v.stride(1), _lib.ptr(self.cos_sin), self.cos_sin.stride(0), self.cos_sin.shape[0],
                      _lib.ptr(ex), ex.shape[0], ex.stride(0), ex.stride(1), ex.stride(2), s.page,
                      _lib.ptr(self.exact_table), self.exact_table.stride(0), self.exact_table.shape[1],
                      _lib.ptr(self.qsl), B, None, flags, strm)

        early = _lib.PREPARE_EARLY_LAUNCH if self.pdl else 0
        # 2b. (window_overlap) the exact part and the exact window on a side stream, beside the history
        #     kernel: they need only this step's q, k, v and the exact cache, and the combine then takes the
        #     window as its external exact part.  The side stream forks after the previous combine (which
        #     was the last reader of q_rope and of the window buffers), so only the latent query stays ahead
        #     of the history split.  On by default when the fused combine would exceed one wave (see the class
        #     notes).
        win_done = None
        if self.window_overlap:
            main = torch.cuda.current_stream(self.device)
            if self._win_stream is None:
                self._win_stream = torch.cuda.Stream(self.device)
            fork = torch.cuda.Event()
            fork.record(main)
            self._win_stream.wait_event(fork)
            side = _lib.ctypes.c_void_p(self._win_stream.cuda_stream)
            prepare((k, v), _lib.PREPARE_EXACT_ONLY, side)
            _lib.call('hla_s6_window_attention', _lib.ptr(qr), qr.stride(0), qr.stride(1), _lib.ptr(ex), ex.shape[0],
                      ex.stride(0), ex.stride(1), ex.stride(2), s.page, _lib.ptr(self.exact_table),
                      self.exact_table.stride(0), self.exact_table.shape[1], _lib.ptr(self.qsl), B,
                      _lib.ptr(self.seq_lens), s.window, float(self.scale), B, s.heads, s.head_dim,
                      _lib.ptr(self.win_o), self.win_o.stride(0), self.win_o.stride(1), _lib.ptr(self.win_lse), side)
            win_done = torch.cuda.Event()
            win_done.record(self._win_stream)
            prepare((None, None), early, stream)       # the latent query alone
        else:
            prepare((k, v), early, stream)
        # 3. history split, a programmatic dependent of the prepare just launched (pages stream meanwhile;
        #    q_lat is read once the prepare has completed).
        self._history(layer, loop, stream, _lib.PARTIALS_AFTER_QUERY if self.pdl else 0)
        # 3b. sequence split: reduce this GPU's slice to (z, lse) and all-gather the parts
        z_in = lse_in = None
        after = _lib.COMBINE_AFTER_PARTIALS if self.pdl else 0
        parts, part_stride, flags = 0, 0, after
        x_epoch = part_seen = None        # the slot's epoch and CTA counter (peer exchange)
        if self.exchange is not None and self.exchange_mode == 'peer':
            import ctypes
            rank, world, _ = self.exchange
            i = loop * s.layers + layer          # exchange slot of this (layer, loop)
            part_stride, wb = self.x_part, _lib.EXCHANGE_WORD_BYTES
            parts = [b + (i * world + rank) * part_stride * wb for b in self.x_bases]
            epoch = _lib.ptr(self.x_counters[2 * i])
            _lib.call('hla_s6_history_reduce_exchange', B, s.heads, width, s.page, self.splits, _lib.ptr(self.ws),
                      self.ws_floats, None, _lib.pointer_array(parts), epoch, world,
                      _lib.REDUCE_AFTER_PARTIALS if self.pdl else 0, stream)
            own = self.x_bases[rank] + i * world * part_stride * wb
            z_in = ctypes.c_void_p(own)
            lse_in = ctypes.c_void_p(own + B * s.heads * width * wb)
            x_epoch, part_seen = epoch, _lib.ptr(self.x_counters[2 * i + 1])
            parts, flags = world, after   # its producer is the reduce just launched
        elif self.reduce_first:
            # few rows over the whole GPU (config 5 on one GPU: ~75 partials per row): the block-cooperative
            # reduce first, then the combine merges its single part, instead of one warp walking every
            # partial of a (row, head) inside the combine
            zf = B * s.heads * width
            z_in, lse_in = self.zpart[:zf], self.zpart[zf:zf + s.heads * B]
            _lib.call('hla_s6_history_reduce', B, s.heads, width, s.page, self.splits, _lib.ptr(self.ws),
                      self.ws_floats, None, None, 0, 0, _lib.ptr(z_in), _lib.ptr(lse_in), stream)
            parts, part_stride, flags = 1, zf + s.heads * B, after      # its producer is the reduce just launched
        elif self.exchange is not None:
            rank, world, group = self.exchange
            zf = B * s.heads * width
            part_stride = zf + s.heads * B
            send = self.xsend[:part_stride]
            _lib.call('hla_s6_history_reduce', B, s.heads, width, s.page, self.splits, _lib.ptr(self.ws),
                      self.ws_floats, None, None, 0, 0, _lib.ptr(send), _lib.ptr(send[zf:]), stream)
            recv = self.xrecv[:world * part_stride]
            torch.distributed.all_gather_into_tensor(recv, send, group=group)
            z_in, lse_in, parts, flags = recv, recv[zf:], world, 0
        # 4. fused combine -> out (with the side stream's window part when window_overlap)
        out = self.out[layer, loop] if io is None else io[4]
        if win_done is not None:
            torch.cuda.current_stream(self.device).wait_event(win_done)
            chunk = (_lib.ptr(self.win_o), self.win_o.stride(0), self.win_o.stride(1), _lib.ptr(self.win_lse))
        else:
            chunk = (None, 0, 0, None)
        _lib.call('hla_s6_decode_combine', B, s.heads, width, s.page, self.splits, _lib.ptr(self.ws), self.ws_floats,
                  _lib.ptr(z_in), _lib.ptr(lse_in), parts, part_stride, x_epoch, part_seen, None, _lib.ptr(Bm),
                  Bm.stride(0), Bm.stride(1), _lib.ptr(qr), qr.stride(0), qr.stride(1),
                  _lib.ptr(ex), ex.shape[0], ex.stride(0), ex.stride(1), ex.stride(2), s.page,
                  _lib.ptr(self.exact_table), self.exact_table.stride(0), self.exact_table.shape[1],
                  _lib.ptr(self.qsl), B, _lib.ptr(self.seq_lens), s.window, float(self.scale), *chunk,
                  _lib.ptr(out),
                  out.stride(0), out.stride(1), None, flags, None, stream)

    def launches_per_step(self):
        """Launches of this library per step (the sequence split adds one reduce per (layer, loop), the
        side-stream window an exact-part prepare and a window kernel)."""
        s = self.s
        return s.layers * s.loops * (4 + (self.exchange is not None or self.reduce_first) +
                                     2 * bool(self.window_overlap))

    def step(self, overlap_writer=True):
        """One decode step.  With ``overlap_writer`` the writer launches run on a side stream forked from
        and joined back into the current stream (a parallel branch when captured in a graph)."""
        main = torch.cuda.current_stream(self.device)
        stream = _lib.stream_of(self.out)
        if not overlap_writer:
            for loop in range(self.s.loops):
                for layer in range(self.s.layers):
                    self.layer_loop(layer, loop, stream)
            return
        if getattr(self, '_side', None) is None:
            self._side = torch.cuda.Stream(self.device)
        side = self._side
        side.wait_stream(main)
        wstream = _lib.ctypes.c_void_p(side.cuda_stream)
        for loop in range(self.s.loops):
            for layer in range(self.s.layers):
                self.layer_loop(layer, loop, stream, wstream)
        main.wait_stream(side)

    def step_io(self, host_in, host_out):
        """One decode step fed from and drained to pinned host memory: ``host_in`` is ``acts``' shape
        ([layers, loops, B, q | k | v | h]), ``host_out`` is ``out``'s.  The copies are pipelined
        with the compute per (layer, loop), in the step's order: a copy stream brings each (layer,
        loop)'s activations in ahead of its launches, which wait only for their own slice (the
        writer branch included), and each output goes back to the host as soon as its combine has
        finished.  Only the first slice's copy-in and the last output's copy-out stay exposed.  The
        results equal ``acts.copy_(host_in); step(); host_out.copy_(out)``."""
        s = self.s
        main = torch.cuda.current_stream(self.device)
        if getattr(self, '_io', None) is None:
            self._io = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
        h2d, d2h, side = self._io
        for st in (h2d, d2h, side):
            st.wait_stream(main)
        order = [(layer, loop) for loop in range(s.loops) for layer in range(s.layers)]
        ready = []
        with torch.cuda.stream(h2d):
            for layer, loop in order:
                self.acts[layer, loop].copy_(host_in[layer, loop], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                ready.append(ev)
        stream = _lib.stream_of(self.out)
        wstream = _lib.ctypes.c_void_p(side.cuda_stream)
        for (layer, loop), ev in zip(order, ready):
            main.wait_event(ev)
            side.wait_event(ev)
            self.layer_loop(layer, loop, stream, wstream)
            done = torch.cuda.Event()
            done.record(main)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                host_out[layer, loop].copy_(self.out[layer, loop], non_blocking=True)
        for st in (h2d, d2h, side):
            main.wait_stream(st)

    def capture_io(self, host_in, host_out):
        """``step_io`` captured as one CUDA graph (copies and kernels)."""
        self.io_graph = self._capture(lambda: self.step_io(host_in, host_out))
        return self.io_graph

    def history_only(self):
        """The 96 history-split launches of a step alone (roofline timing of the dominant kernel)."""
        stream = _lib.stream_of(self.out)
        for loop in range(self.s.loops):
            for layer in range(self.s.layers):
                self._history(layer, loop, stream)

    # ------------------------------------------------------------------ graphs
    def _capture(self, fn):
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            fn()                       # warm-up outside capture (descriptor caches, occupancy queries)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    def capture(self):
        self.graph = self._capture(self.step)
        return self.graph

    def capture_history(self):
        self.history_graph = self._capture(self.history_only)
        return self.history_graph

    def replay(self):
        self.graph.replay()
