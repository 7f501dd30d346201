"""Run the reference's own serving code on the B200 kernels: register them as the ``'b200'`` backend of
the reference's ops module (``hla/vllm_latent/s6_ops.py``) at run time, without editing its source.

    from hla.vllm_latent import s6_ops, s6_layer                       # the reference modules
    reg = importlib.import_module('hybrid-latent-attention_b200.register_backend')
    reg.register(s6_ops)
    ctx = s6_layer.StepContext(..., s6_ops.select_backends(), ...)     # Backends('b200', 'b200', 'b200', 'b200')
    out = s6_layer.attend(...)                                         # the reference's attend, B200 kernels

What changes in the module (the backend dispatch points of s6_ops.py:23, :44, :128, :234, :262, :317, :334,
:364):

* ``history_attention_kv``, ``chunk_attention``, ``merge_states`` and ``latent_rope`` gain a ``'b200'`` branch in
  front of the reference's dispatch; for these four, every other backend string reaches the original function
  unchanged.  ``history_attention`` needs no wrapper: the reference implements it through the module's
  ``history_attention_kv``.
* ``window_attention_fa`` / ``window_history_fa`` (the exact window of the decode and prefill branches of
  ``s6_layer.attend``) take no backend argument, so they cannot dispatch: with ``window=True`` (the default)
  they are REPLACED by the B200 kernels for every caller, whatever backends its ``StepContext`` holds - a
  ``'torch'`` or FA2 set-up then runs the B200 window too (and, on CPU tensors, gets this package's
  ``ValueError``).  Pass ``window=False`` to keep the reference's FA2 window ops.
* ``probe_latent_rope`` (no backend argument either; the adapter calls it once at start-up, right after
  ``select_backends``) is replaced by this package's probe of the B200 latent-RoPE kernel, whose answer is
  ``(flat=False, exact)``.
* ``select_backends`` returns the module's own ``Backends`` namedtuple filled with ``'b200'``.

``unregister`` restores the originals.  The B200 functions keep the reference's signatures, layouts and
errors (this package's ``s6_ops``), so the reference's callers - ``s6_layer.attend``, ``latent_query``,
``committed_row``, the vLLM attention layer - run unchanged.
"""
from __future__ import annotations

import functools
import importlib

_B200 = 'b200'
_ATTR = '_b200_originals'
_BACKEND_OPS = ('history_attention_kv', 'chunk_attention', 'merge_states', 'latent_rope')
_WINDOW_OPS = ('window_attention_fa', 'window_history_fa')


def _mine():
    return importlib.import_module(f'{__package__}.s6_ops')


def _with_b200(name, original, mine):
    """``original`` with a 'b200' branch: the backend is the ``backend`` keyword or, positionally, the
    parameter of that name in the reference signature."""
    import inspect
    params = list(inspect.signature(original).parameters)
    index = params.index('backend')
    target = getattr(mine, name)

    @functools.wraps(original)
    def op(*args, **kwargs):
        backend = kwargs.get('backend', args[index] if len(args) > index else None)
        if backend == _B200:
            return target(*args, **kwargs)
        return original(*args, **kwargs)
    op.__b200__ = target
    return op


def register(s6_ops, window=True):
    """Install the 'b200' backend into the reference module ``s6_ops`` (idempotent).  Returns the module."""
    if getattr(s6_ops, _ATTR, None) is not None:
        return s6_ops
    mine = _mine()
    originals = {}
    for name in _BACKEND_OPS:
        originals[name] = getattr(s6_ops, name)
        setattr(s6_ops, name, _with_b200(name, originals[name], mine))
    if window:
        for name in _WINDOW_OPS:
            originals[name] = getattr(s6_ops, name)
            setattr(s6_ops, name, functools.wraps(originals[name])(getattr(mine, name)))
    originals['probe_latent_rope'] = s6_ops.probe_latent_rope
    s6_ops.probe_latent_rope = functools.wraps(originals['probe_latent_rope'])(mine.probe_latent_rope)
    originals['select_backends'] = s6_ops.select_backends

    @functools.wraps(originals['select_backends'])
    def select_backends(head_size=128):
        mine.select_backends(head_size)          # the library loads and the device is a CUDA GPU
        return s6_ops.Backends(_B200, _B200, _B200, _B200)
    s6_ops.select_backends = select_backends
    setattr(s6_ops, _ATTR, originals)
    return s6_ops


def unregister(s6_ops):
    """Restore the functions ``register`` replaced."""
    originals = getattr(s6_ops, _ATTR, None)
    if originals is None:
        return s6_ops
    for name, fn in originals.items():
        setattr(s6_ops, name, fn)
    setattr(s6_ops, _ATTR, None)
    return s6_ops
