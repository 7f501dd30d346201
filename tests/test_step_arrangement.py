"""Default arrangement of a decode step's launches (decode.step_arrangement), host logic only.  CPU.

The side-stream exact part and window are chosen when the fused combine (heads x ceil(T / 8) CTAs, one
per SM) would exceed one wave; the reduce before the combine when the history split (2 CTAs per SM)
leaves more than about 16 partials per row; neither under a sequence split."""
import pytest

from conftest import pkg

SMS, HEADS = 148, 16


@pytest.mark.parametrize('requests,expect', [
    (64, (False, False)),      # config 2: 128 combine CTAs, ~5 partials per row
    (256, (True, False)),      # config 4: 512 combine CTAs
    (201, (True, False)),
    (72, (False, False)),      # 144 CTAs: still one wave
    (73, (True, False)),       # 160 CTAs
    (4, (False, True)),        # config 5 on one GPU: ~75 partials per row
    (18, (False, True)),       # 296 > 288
    (19, (False, False)),      # 296 < 304
])
def test_default_arrangement(requests, expect):
    assert pkg('decode').step_arrangement(requests, HEADS, SMS, False) == expect


@pytest.mark.parametrize('requests', [4, 64, 256])
def test_sequence_split_keeps_the_fused_step(requests):
    assert pkg('decode').step_arrangement(requests, HEADS, SMS, True) == (False, False)
