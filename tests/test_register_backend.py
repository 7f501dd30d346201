"""register_backend installs the B200 kernels as the 'b200' backend of the REFERENCE's own ops module
(hla/vllm_latent/s6_ops.py), read-only from a reference checkout: every other backend keeps running
the reference's code, 'b200' reaches this package's ops (which refuse CPU tensors - there is no CPU
path - proving the routing without a GPU), select_backends answers 'b200', and unregister restores the
module.  CPU only; skipped unless HLA_REFERENCE_ROOT names a checkout of the reference project."""
import importlib
import os
import sys
from pathlib import Path

import pytest
import torch

from conftest import pkg

REF = Path(os.environ.get('HLA_REFERENCE_ROOT', '') or '/nonexistent')
pytestmark = pytest.mark.skipif(not (REF / 'hla' / 'vllm_latent' / 's6_ops.py').exists(),
                                reason='set HLA_REFERENCE_ROOT to a checkout of the reference project')


@pytest.fixture()
def ref_ops():
    sys.path.insert(0, str(REF))
    try:
        mod = importlib.import_module('hla.vllm_latent.s6_ops')
        yield mod
        pkg('register_backend').unregister(mod)
    finally:
        sys.path.remove(str(REF))


def paged(T=3, H=16, W=64, page=16, ctx=(0, 5, 40)):
    g = torch.Generator().manual_seed(0)
    nb = 8
    cache = torch.randn(nb, 1, page, 2 * W, generator=g)
    table = torch.arange(1, nb, dtype=torch.int32)[None, :].repeat(T, 1)
    q = torch.randn(T, H, W, generator=g)
    return q, cache, table, torch.tensor(ctx, dtype=torch.int32)


def test_other_backends_keep_the_reference_code(ref_ops):
    q, cache, table, ctx = paged()
    before = ref_ops.history_attention(q, cache, table, ctx, 0.1, 1, None, None, None, 'torch')
    pkg('register_backend').register(ref_ops)
    after = ref_ops.history_attention(q, cache, table, ctx, 0.1, 1, None, None, None, 'torch')
    for a, b in zip(before, after):
        assert torch.equal(a, b)
    with pytest.raises(ValueError, match='Unknown history backend'):
        ref_ops.history_attention(q, cache, table, ctx, 0.1, 1, None, None, None, 'nonsense')
    o = torch.randn(3, 16, 8)
    lse = torch.randn(16, 3)
    inval = torch.zeros(3, dtype=torch.bool)
    assert torch.equal(ref_ops.merge_states(o, lse, o, lse, inval, 'torch'), ref_ops._merge_reference(o, lse, o, lse))


def test_b200_backend_reaches_this_package(ref_ops):
    q, cache, table, ctx = paged()
    with pytest.raises(ValueError, match='Unknown history backend'):       # before: the reference refuses 'b200'
        ref_ops.history_attention(q, cache, table, ctx, 0.1, 1, None, None, None, 'b200')
    pkg('register_backend').register(ref_ops)
    # the reference's history_attention -> its (wrapped) history_attention_kv -> this package's op
    with pytest.raises(ValueError, match='CUDA tensors'):
        ref_ops.history_attention(q, cache, table, ctx, 0.1, 1, None, None, None, 'b200')
    with pytest.raises(ValueError, match='CUDA tensors'):
        ref_ops.history_attention_kv(q, cache[..., :64], cache[..., 64:], table, ctx, 0.1, 1, None, None, None,
                                     backend='b200')
    o = torch.randn(3, 16, 8)
    lse = torch.randn(16, 3)
    with pytest.raises(ValueError, match='CUDA'):
        ref_ops.merge_states(o, lse, o, lse, torch.zeros(3, dtype=torch.bool), 'b200')
    with pytest.raises(ValueError, match='CUDA'):
        ref_ops.window_attention_fa(torch.randn(1, 16, 128), torch.randn(2, 16, 16, 256), table[:1],
                                    torch.tensor([0, 1], dtype=torch.int32), torch.tensor([3], dtype=torch.int32), 32,
                                    0.1, 4, torch.zeros(1, dtype=torch.bool))
    assert ref_ops.window_attention_fa.__name__ == 'window_attention_fa'


def test_select_backends_and_unregister(ref_ops):
    reg = pkg('register_backend')
    originals = {n: getattr(ref_ops, n) for n in ('history_attention_kv', 'merge_states', 'latent_rope',
                                                   'chunk_attention', 'window_attention_fa', 'window_history_fa',
                                                   'select_backends', 'probe_latent_rope')}
    reg.register(ref_ops)
    reg.register(ref_ops)                                                     # idempotent
    assert ref_ops.history_attention_kv.__wrapped__ is originals['history_attention_kv']
    if torch.cuda.is_available():
        assert tuple(ref_ops.select_backends()) == ('b200',) * 4
    else:
        with pytest.raises(RuntimeError, match='CUDA'):
            ref_ops.select_backends()
    reg.unregister(ref_ops)
    for name, fn in originals.items():
        assert getattr(ref_ops, name) is fn


def test_window_ops_are_replaced_whatever_the_backend(ref_ops):
    """The two window ops take no backend argument: once registered with window=True, the reference's own
    s6_layer.attend reaches the B200 window even under TORCH_BACKENDS (here: this package's CUDA-only
    ValueError on CPU tensors); with window=False the reference's own ops stay in place."""
    layer = importlib.import_module('hla.vllm_latent.s6_layer')
    reg = pkg('register_backend')
    T, H, d = 1, 16, 128
    ctx = layer.StepContext(torch.zeros(T, dtype=torch.long), torch.tensor([0, 1], dtype=torch.int32),
                            torch.tensor([3], dtype=torch.int32), 1, T, {}, 0.1, ref_ops.TORCH_BACKENDS, window=32)
    q = torch.randn(T, H, d)
    window = (torch.randn(2, H, 16, 2 * d), torch.tensor([[1]], dtype=torch.int32))
    original = ref_ops.window_attention_fa
    reg.register(ref_ops, window=False)
    assert ref_ops.window_attention_fa is original
    reg.unregister(ref_ops)
    reg.register(ref_ops)
    assert ref_ops.window_attention_fa is not original
    with pytest.raises(ValueError, match='CUDA'):
        layer.attend(None, 1, None, q, q, q, None, None, None, None, ctx, window)
    # the start-up probe now checks the B200 kernel (CUDA-only: refuses a CPU table)
    with pytest.raises(ValueError, match='CUDA'):
        ref_ops.probe_latent_rope(torch.zeros(16, 64, dtype=torch.bfloat16))
