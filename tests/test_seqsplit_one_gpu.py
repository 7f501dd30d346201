"""Sequence split of the latent history emulated on ONE GPU, through the C ABI.

The history is cut into N contiguous page slices (``decode.seq_split_rows``).  For each slice r the
history split runs over that slice alone and ``hla_s6_history_reduce_exchange`` stores the slice's
part (z, lse) as tagged exchange words into slot r of D receive regions (the D GPUs of a real run;
here D regions of this GPU's memory).  ``hla_s6_decode_combine`` then polls the N parts of one region,
LSE-merges them (the reference's merge semantics, s6_ops.py:353-361), up-projects by B and merges the
exact window (s6_layer.py:97-115).  Every region must give the same output, equal to the oracle over
the whole history, step after step, with each region's epoch advanced once per step and its CTA
counter left zeroed.

All reduces complete before a combine starts (plain stream order, no programmatic launches), so no
kernel here polls words that a concurrently running kernel on this GPU would store.

The timeout tests never deliver one of two parts (or leave last exchange's words in it) and lower the
wait limit to a few milliseconds: the combine must give up, report HLA_S6_ERR_WAIT_PEER through its
error word and return normally.
"""
import math

import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import s6_oracle as orc
from test_attend_gpu import build_step, oracle

pytestmark = pytest.mark.gpu
CUDA, BF16, F32, I32, I64 = 'cuda', torch.bfloat16, torch.float32, torch.int32, torch.int64
O_TOL = dict(atol=2e-2, rtol=1e-2)
PAGE, H, D_HEAD = 16, 16, 128


class SplitStep:
    """Device tensors of one decode (layer, loop) and the exchange buffers of an N-way split."""

    def __init__(self, s, parts, regions, splits=16):
        lib = pkg('_lib')
        self.lib, self.s, self.N, self.D, self.splits = lib, s, parts, regions, splits
        T, R, W = s['T'], s['R'], s['width']
        self.T, self.W = T, W
        dv = lambda a, dt=None: (lambda t: t.to(dt) if dt else t)(torch.from_numpy(np.ascontiguousarray(a)).to(CUDA))
        self.q_lat, self.q_rope = dv(s['q_lat'], BF16), dv(s['q_rope'], BF16)
        self.lat, self.B = dv(s['lat'], BF16), dv(s['B'], BF16)
        self.ex = dv(s['ex'], BF16).transpose(1, 2)            # logical [nb, H, page, 2d]
        self.etab, self.qsl, self.seq_lens = dv(s['etab']), dv(s['qsl']), dv(s['seq_lens'])
        ltab_tok = np.zeros((T, s['ltab'].shape[1]), dtype=np.int32)
        ltab_tok[:R] = s['ltab']
        ctx_lat = np.zeros(T, dtype=np.int64)
        ctx_lat[:R] = s['ctx_lat']
        dec = pkg('decode')
        self.slices = []
        for r in range(parts):
            split = dec.seq_split_rows(ctx_lat.tolist(), PAGE, r, parts)
            table = np.zeros_like(ltab_tok)
            rows = np.zeros(T, dtype=np.int32)
            for t, (p0, n) in enumerate(split):
                npg = -(-n // PAGE)
                table[t, :npg] = ltab_tok[t, p0:p0 + npg]
                rows[t] = n
            self.slices.append((dv(table), dv(rows)))
        self.ws_floats = T * splits * H * (W + 1)
        self.ws = torch.empty(self.ws_floats, dtype=F32, device=CUDA)
        self.part = -(-(T * H * W + H * T) // 2) * 2              # exchange words per part, even
        self.recv = torch.zeros(regions, parts, self.part, dtype=I64, device=CUDA)   # tag 0: nothing yet
        self.epochs = torch.zeros(regions, dtype=I32, device=CUDA)
        self.seen = torch.zeros(regions, dtype=I32, device=CUDA)
        self.err = torch.zeros(1, dtype=I32, device=CUDA)
        self.scale = 1 / math.sqrt(D_HEAD)

    def reduce_slice(self, r, world=None):
        """History split over slice r, then its part stored into slot r of every region (world
        regions, default all), tagged with the regions' common epoch + 1."""
        lib, T, W = self.lib, self.T, self.W
        table, rows = self.slices[r]
        stream = lib.stream_of(self.q_lat)
        lib.call('hla_s6_history_partials', lib.ptr(self.q_lat), self.q_lat.stride(0), self.q_lat.stride(1),
                 lib.ptr(self.lat), self.lat.shape[0], self.lat.stride(0), self.lat.stride(2), lib.ptr(table),
                 table.stride(0), table.shape[1], lib.ptr(rows), T, H, W, PAGE, float(self.scale), self.splits,
                 lib.ptr(self.ws), self.ws_floats, lib.ptr(self.err), 0, stream)
        world = self.D if world is None else world
        parts = [self.recv[d, r].data_ptr() for d in range(world)]
        lib.call('hla_s6_history_reduce_exchange', T, H, W, PAGE, self.splits, lib.ptr(self.ws), self.ws_floats,
                 None, lib.pointer_array(parts), lib.ptr(self.epochs), world, 0, stream)

    def combine(self, d):
        lib, s, T, W = self.lib, self.s, self.T, self.W
        out = torch.empty(T, H, D_HEAD, dtype=BF16, device=CUDA)
        z = self.recv[d, 0]
        stream = lib.stream_of(out)
        lib.call('hla_s6_decode_combine', T, H, W, PAGE, self.splits, lib.ptr(self.ws), self.ws_floats, lib.ptr(z),
                 lib.ptr(z[T * H * W:]), self.N, self.part, lib.ptr(self.epochs[d:]), lib.ptr(self.seen[d:]), None,
                 lib.ptr(self.B), self.B.stride(0), self.B.stride(1), lib.ptr(self.q_rope), self.q_rope.stride(0),
                 self.q_rope.stride(1), lib.ptr(self.ex), self.ex.shape[0], self.ex.stride(0), self.ex.stride(1),
                 self.ex.stride(2), PAGE, lib.ptr(self.etab), self.etab.stride(0), self.etab.shape[1],
                 lib.ptr(self.qsl), s['R'], lib.ptr(self.seq_lens), s['window'], float(self.scale), None, 0, 0, None,
                 lib.ptr(out), out.stride(0), out.stride(1), None, 0, lib.ptr(self.err), stream)
        return out

    def step(self):
        for r in range(self.N):
            self.reduce_slice(r)
        return [self.combine(d) for d in range(self.D)]


@pytest.mark.parametrize('width', [512, 256])
@pytest.mark.parametrize('parts', [2, 4])
def test_n_part_merge_matches_whole_history_oracle(width, parts):
    """N slices reduced into N regions, each region combined: every output equals the oracle over the
    whole history, over two steps (slots, epochs and counters reused; new q each step)."""
    ctxs = [4096, 1000, 40, 2000, 0, 33, 31, 700]
    for step in range(2):
        s = build_step(100 * parts + width + step, width, ctxs)
        run = SplitStep(s, parts, parts)
        if step:   # the second step reuses the first step's exchange buffers and counters
            run.recv, run.epochs, run.seen = prev.recv, prev.epochs, prev.seen
        outs = run.step()
        torch.cuda.synchronize()
        ref = oracle(s, run.scale)
        for out in outs:
            got = out.float().cpu().numpy()
            assert np.isfinite(got).all() and (got[s['R']:] == 0).all()
            np.testing.assert_allclose(got, ref, **O_TOL)
            assert torch.equal(out, outs[0])           # every region merges the same parts
        assert int(run.err.item()) == 0
        assert (run.epochs == step + 1).all() and int(run.seen.abs().sum()) == 0
        prev = run


def test_config5_split_equals_single_gpu_path_at_full_context():
    """BASELINE config 5's shape: B = 4 at ctx 131072, the history cut into 8 slices; the 8-part merge
    equals the single-GPU fused decode attend over the whole history (size-independent property)."""
    lay, ops = pkg('s6_layer'), pkg('s6_ops')
    width, ctx = 512, 131072
    rng = np.random.default_rng(5)
    T = R = 4
    window = 32
    g = torch.Generator(device=CUDA).manual_seed(5)
    pages = -(-(ctx + 1) // PAGE)
    nb = T * pages + 1
    lat = torch.randn(nb, 1, PAGE, 2 * width, dtype=BF16, device=CUDA, generator=g)
    lat[0] = float('inf')
    perm = torch.from_numpy(rng.permutation(np.arange(1, nb)).astype(np.int32))
    ltab = perm.view(T, pages).to(CUDA)
    enb = T * 4 + 1
    ex = torch.randn(enb, PAGE, H, 2 * D_HEAD, dtype=BF16, device=CUDA, generator=g)
    etab = torch.zeros(T, pages, dtype=I32)
    for r in range(T):
        for j, col in enumerate(range((ctx - window) // PAGE, ctx // PAGE + 1)):
            etab[r, col] = 1 + 4 * r + j
    s = dict(q_lat=None, T=T, R=R, width=width, window=window)
    q_lat = torch.randn(T, H, width, generator=g, device=CUDA).to(BF16)
    q_rope = torch.randn(T, H, D_HEAD, generator=g, device=CUDA).to(BF16)
    B = (torch.randn(H, width, D_HEAD, generator=g, device=CUDA) / math.sqrt(width)).to(BF16)
    qsl = torch.arange(R + 1, dtype=I32, device=CUDA)
    seq_lens = torch.full((R,), ctx + 1, dtype=I32, device=CUDA)
    scale = 1 / math.sqrt(D_HEAD)
    splits = 64
    ws = ops.S6Workspace(H, width, T * splits)
    sctx = lay.StepContext(torch.full((T,), ctx, dtype=torch.int64, device=CUDA), qsl, seq_lens, 1, T, {}, scale,
                           ops.B200_BACKENDS, ws, splits, window=window)

    class SL:
        def readers(self, loop):
            return None, B, width

    exl = ex.transpose(1, 2)
    whole = lay.attend(SL(), 1, q_lat, q_rope, None, None, lat, ltab, None, None, sctx, (exl, etab.to(CUDA)))
    # the split run, through the same tensors
    run = SplitStep.__new__(SplitStep)
    lib = pkg('_lib')
    run.lib, run.N, run.D, run.splits, run.T, run.W, run.scale = lib, 8, 1, splits, T, width, scale
    run.s = dict(R=R, window=window)
    run.q_lat, run.q_rope, run.lat, run.B, run.ex = q_lat, q_rope, lat, B, exl
    run.etab, run.qsl, run.seq_lens = etab.to(CUDA), qsl, seq_lens
    dec = pkg('decode')
    ltab_h = ltab.cpu().numpy()
    run.slices = []
    for r in range(8):
        split = dec.seq_split_rows([ctx - window] * T, PAGE, r, 8)
        table = np.zeros_like(ltab_h)
        rows = np.zeros(T, dtype=np.int32)
        for t, (p0, n) in enumerate(split):
            npg = -(-n // PAGE)
            table[t, :npg] = ltab_h[t, p0:p0 + npg]
            rows[t] = n
        run.slices.append((torch.from_numpy(table).to(CUDA), torch.from_numpy(rows).to(CUDA)))
    run.ws_floats = T * splits * H * (width + 1)
    run.ws = torch.empty(run.ws_floats, dtype=F32, device=CUDA)
    run.part = -(-(T * H * width + H * T) // 2) * 2
    run.recv = torch.zeros(1, 8, run.part, dtype=I64, device=CUDA)
    run.epochs = torch.zeros(1, dtype=I32, device=CUDA)
    run.seen = torch.zeros(1, dtype=I32, device=CUDA)
    run.err = torch.zeros(1, dtype=I32, device=CUDA)
    (split_out,) = run.step()
    torch.cuda.synchronize()
    assert int(run.err.item()) == 0
    assert torch.isfinite(split_out.float()).all()
    torch.testing.assert_close(split_out.float(), whole.float(), **O_TOL)
    assert int(run.epochs.item()) == 1 and int(run.seen.item()) == 0


def exchange_words(values, tag):
    """Exchange words (int64) of fp32 ``values`` tagged ``tag``: value bits low, tag high."""
    bits = torch.as_tensor(values, dtype=F32).view(I32).to(I64) & 0xFFFFFFFF
    return bits | (int(tag) << 32)


def test_exchange_wait_gives_up_and_reports():
    """Two parts, only part 0 delivered: with a 5 ms wait limit the combine reports
    HLA_S6_ERR_WAIT_PEER and returns; the missing part counts as empty, so the output equals the
    one-part merge, and the slot's epoch still advances.  The next exchange of the slot, with part 1
    delivered as an empty part, completes without error."""
    lib = pkg('_lib')
    s = build_step(77, 512, [900, 40, 3000])
    run = SplitStep(s, 1, 1)
    run.N = 2
    T, W = run.T, run.W
    run.recv = torch.zeros(1, 2, run.part, dtype=I64, device=CUDA)   # part 1's words stay untagged
    run.reduce_slice(0, world=1)
    prev = lib.set_wait_limit_ns(5_000_000)
    try:
        out = run.combine(0)
        torch.cuda.synchronize()                                  # the kernel returned
    finally:
        lib.set_wait_limit_ns(prev)
    assert int(run.err.item()) == lib.ERR_WAIT_PEER
    assert int(run.epochs.item()) == 1 and int(run.seen.item()) == 0
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle(s, run.scale), **O_TOL)
    # the context is still usable: the slot's next exchange (tag 2) with both parts completes cleanly
    run.err.zero_()
    run.reduce_slice(0, world=1)
    lse1 = run.recv[0, 1, T * H * W:T * H * W + H * T]
    lse1.copy_(exchange_words(torch.full((H * T,), float('-inf')), 2).to(CUDA))
    out2 = run.combine(0)
    torch.cuda.synchronize()
    assert int(run.err.item()) == 0 and int(run.epochs.item()) == 2
    assert torch.equal(out2, out)


def test_stale_tags_are_not_taken():
    """A part left over from the slot's previous exchange (tag = epoch) is not taken for the current
    one: with part 1 holding last exchange's words the combine times out on it, exactly as if it were
    missing."""
    lib = pkg('_lib')
    s = build_step(78, 256, [500, 70])
    run = SplitStep(s, 1, 1)
    run.N = 2
    T, W = run.T, run.W
    run.recv = torch.zeros(1, 2, run.part, dtype=I64, device=CUDA)
    run.epochs.fill_(4)                                           # this exchange's tag is 5
    run.recv[0, 1, :T * H * W] = exchange_words(torch.ones(T * H * W), 4).to(CUDA)
    run.recv[0, 1, T * H * W:T * H * W + H * T] = exchange_words(torch.zeros(H * T), 4).to(CUDA)
    run.reduce_slice(0, world=1)
    prev = lib.set_wait_limit_ns(5_000_000)
    try:
        out = run.combine(0)
        torch.cuda.synchronize()
    finally:
        lib.set_wait_limit_ns(prev)
    assert int(run.err.item()) == lib.ERR_WAIT_PEER and int(run.epochs.item()) == 5
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle(s, run.scale), **O_TOL)


def test_one_rank_peer_exchange_step_matches_the_plain_step(tmp_path):
    """The model's peer-exchange step on one rank (world 1): the reduce stores its part as exchange
    words into this GPU's region and releases the combine early, the combine polls the words - the
    programmatic-launch chain of a real sequence split, without a second GPU.  Eagerly and over two
    graph replays (every slot reused), its output matches the plain step (partials merged directly
    in the combine) within the output tolerance, and every slot's epoch advances once per step."""
    import torch.distributed as dist
    dec = pkg('decode')
    dist.init_process_group('gloo', init_method=f'file://{tmp_path / "rdv"}', rank=0, world_size=1)
    try:
        shape = dec.OuroShape(layers=2)
        ctx = [3000, 40, 8192, 700]
        plain = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device=CUDA, seed=3)
        split = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device=CUDA, seed=3,
                                  exchange=(0, 1, dist.group.WORLD))
        try:
            plain.step()
            split.step()
            torch.cuda.synchronize()
            torch.testing.assert_close(split.out.float(), plain.out.float(), **O_TOL)
            graph = split.capture()
            for _ in range(2):
                split.out.zero_()
                graph.replay()
                torch.cuda.synchronize()
                torch.testing.assert_close(split.out.float(), plain.out.float(), **O_TOL)
            epochs = split.x_counters.view(-1, 2).cpu()
            steps = int(epochs[0, 0])
            assert steps >= 3 and (epochs[:, 0] == steps).all() and (epochs[:, 1] == 0).all()
            del graph
        finally:
            split.close_exchange()
    finally:
        dist.destroy_process_group()
