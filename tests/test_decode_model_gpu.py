"""The whole decode step of S6DecodeModel (4-5 launches per (layer, loop), graph-captured) in its two
arrangements of the exact window - inside the fused combine, or as its own kernel on a side stream
beside the history kernel (window_overlap) - agree, eagerly and under graph replay.  GPU."""
import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu


def _model(overlap):
    dec = pkg('decode')
    shape = dec.OuroShape(layers=2)
    return dec.S6DecodeModel(shape, dec.DecodeBatch([4096, 1000, 40, 2000, 1, 33, 31, 0][:8]), device='cuda', seed=11,
                             window_overlap=overlap)


def test_side_stream_window_matches_fused_window():
    fused, side = _model(False), _model(True)
    assert torch.equal(fused.acts, side.acts)
    fused.step()
    side.step()
    torch.cuda.synchronize()
    assert torch.isfinite(side.out.float()).all()
    # the side-stream window is rounded to bf16 before the merge (as the reference's FA2 output is)
    torch.testing.assert_close(side.out.float(), fused.out.float(), atol=2e-2, rtol=1e-2)
    eager = side.out.clone()
    g = side.capture()
    side.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(side.out, eager)


def test_many_requests_side_window_and_sixteen_token_combine():
    """201 requests: by default the exact part and the window run beside the history kernel, and the
    combine, whose 8-token grid (16 x 26 CTAs) would exceed one wave, takes 16 tokens per CTA (the last
    CTA of each head holds 9).  It agrees with the window inside an 8-token combine, eagerly and under
    graph replay."""
    dec = pkg('decode')
    shape = dec.OuroShape(layers=1)
    ctx = [(37 * i * i + 11 * i) % 3000 for i in range(201)]
    ctx[:4] = [0, 1, 31, 32]
    auto = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=13)
    fused = dec.S6DecodeModel(shape, dec.DecodeBatch(ctx), device='cuda', seed=13, window_overlap=False)
    assert auto.window_overlap and not fused.window_overlap
    auto.step()
    fused.step()
    torch.cuda.synchronize()
    assert torch.isfinite(auto.out.float()).all()
    torch.testing.assert_close(auto.out.float(), fused.out.float(), atol=2e-2, rtol=1e-2)
    eager = auto.out.clone()
    g = auto.capture()
    auto.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(auto.out, eager)


def test_few_requests_reduce_before_the_combine():
    """4 long requests (about 75 stream-K partials per row): by default the block-cooperative reduce merges
    the partials before the combine, which then merges one part.  It agrees with the in-combine reduce
    (one warp per (row, head) over all partials), eagerly and under graph replay."""
    dec = pkg('decode')
    shape = dec.OuroShape(layers=1)
    batch = dec.DecodeBatch([30000, 17, 12000, 0])
    first = dec.S6DecodeModel(shape, batch, device='cuda', seed=21)
    inside = dec.S6DecodeModel(shape, batch, device='cuda', seed=21, reduce_first=False)
    assert first.reduce_first and not inside.reduce_first
    first.step()
    inside.step()
    torch.cuda.synchronize()
    assert torch.isfinite(first.out.float()).all()
    torch.testing.assert_close(first.out.float(), inside.out.float(), atol=2e-2, rtol=1e-2)
    eager = first.out.clone()
    g = first.capture()
    first.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(first.out, eager)


def test_programmatic_launches_match_serial_launches():
    """The step's programmatic dependent launches (history split beside the prepare that writes q_lat,
    combine beside the history split) give bit-identical outputs to fully serialised launches, for
    every (layer, loop) - each writes the shared q_lat buffer anew, so a stale read would show -
    eagerly and under graph replay."""
    dec = pkg('decode')
    shape = dec.OuroShape(layers=3)
    batch = dec.DecodeBatch([4096, 1000, 40, 2000, 1, 33, 31, 0, 8192, 300])
    chained = dec.S6DecodeModel(shape, batch, device='cuda', seed=5, pdl=True)
    serial = dec.S6DecodeModel(shape, batch, device='cuda', seed=5, pdl=False)
    chained.step()
    serial.step()
    torch.cuda.synchronize()
    assert torch.isfinite(serial.out.float()).all()
    assert torch.equal(chained.out, serial.out)
    g = chained.capture()
    expect = chained.out.clone()
    for _ in range(3):
        chained.out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(chained.out, expect)


def test_pipelined_host_io_step_matches_copy_step_copy():
    """step_io (per-(layer, loop) copy-in ahead of the launches, copy-out after each combine, on their own
    streams) gives exactly acts <- host_in; step(); host_out <- out - eagerly and as a replayed graph,
    with new host inputs between replays."""
    dec = pkg('decode')
    shape = dec.OuroShape(layers=2)
    batch = dec.DecodeBatch([3000, 17, 0, 500, 64, 1])
    piped = dec.S6DecodeModel(shape, batch, device='cuda', seed=9)
    plain = dec.S6DecodeModel(shape, batch, device='cuda', seed=9)
    g = torch.Generator().manual_seed(3)
    host_in = torch.empty(piped.acts.shape, dtype=piped.acts.dtype, pin_memory=True)
    host_out = torch.empty(piped.out.shape, dtype=piped.out.dtype, pin_memory=True)

    def check():
        plain.acts.copy_(host_in)
        plain.step()
        torch.cuda.synchronize()
        assert torch.equal(host_out, plain.out.cpu())

    host_in.copy_(torch.randn(host_in.shape, generator=g).to(host_in.dtype))
    piped.step_io(host_in, host_out)
    torch.cuda.synchronize()
    check()
    graph = piped.capture_io(host_in, host_out)
    for _ in range(2):
        host_in.copy_(torch.randn(host_in.shape, generator=g).to(host_in.dtype))
        host_out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        check()
