"""ctypes binding of libhla_s6.so (the C ABI declared in include/hla_s6.h).

The shared library is built in-tree by ``build.py``.  There is no fallback: if the library
is missing or was built for another ABI version, importing the ops raises.
"""
from __future__ import annotations

import ctypes  # noqa: F401  (re-exported for callers that build stream handles)
import os
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get('HLA_S6_LIB', _PKG / 'libhla_s6.so'))
ABI_VERSION = 4

OK, EINVAL, EOVERFLOW, ECUDA = 0, 1, 2, 3
# codes a kernel writes to its optional device error word (HLA_S6_ERR_*)
ERR_WAIT_COPY, ERR_WAIT_STAGE, ERR_RANGE, ERR_WAIT_PEER, ERR_BLOCK = 1, 2, 3, 4, 5
COMBINE_AFTER_PARTIALS = 1   # hla_s6_decode_combine flag (include/hla_s6.h)
PARTIALS_AFTER_QUERY = 1     # hla_s6_history_partials flag
REDUCE_AFTER_PARTIALS = 1    # hla_s6_history_reduce_exchange flag
PREPARE_EARLY_LAUNCH = 1     # hla_s6_decode_prepare flags
PREPARE_EXACT_ONLY = 2
PEER_HANDLE_BYTES = 64       # HLA_S6_PEER_HANDLE_BYTES
EXCHANGE_WORD_BYTES = 8      # HLA_S6_EXCHANGE_WORD_BYTES: fp32 value | 32-bit tag

_c_void_p, _i32, _i64, _f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
P = _c_void_p

# name -> argtypes (restype is always int32 status unless noted)
SIGNATURES = {
    'hla_s6_history_attention': [P, _i64, _i64, P, _i64, _i64, _i64, P, _i64, _i32, P, P, _i32, _i32, _i32, _i32,
                                 _f32, _i32, P, _i64, P, _i64, _i64, P, P, P],
    'hla_s6_history_partials': [P, _i64, _i64, P, _i64, _i64, _i64, P, _i64, _i32, P, _i32, _i32, _i32, _i32, _f32,
                                _i32, P, _i64, P, _i32, P],
    'hla_s6_history_reduce': [_i32, _i32, _i32, _i32, _i32, P, _i64, P, P, _i64, _i64, P, P, P],
    'hla_s6_history_plan': [_i32, _i32, _i32, _i32, _i32, _i64, P, P, P],
    'hla_s6_window_attention': [P, _i64, _i64, P, _i64, _i64, _i64, _i64, _i32, P, _i64, _i32, P, _i32, P, _i32, _f32,
                                _i32, _i32, _i32, P, _i64, _i64, P, P],
    'hla_s6_merge_states': [P, _i64, _i64, P, P, _i64, _i64, P, P, P, _i64, _i64, _i32, _i32, _i32, P],
    'hla_s6_merge_lse': [P, _i64, _i64, P, P, _i64, _i64, P, P, _i64, _i64, P, _i32, _i32, _i32, P],
    'hla_s6_latent_rope': [P, _i64, _i64, _i32, _i32, _i32, P, P, _i64, _i64, P],
    'hla_s6_latent_query': [P, _i64, _i64, P, _i64, _i64, P, P, _i64, _i64, P, _i64, _i64, _i32, _i32, _i32, _i32, P],
    'hla_s6_exact_append': [P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, P, P, _i64, _i64, P, _i64,
                            _i64, _i64, _i64, _i32, P, _i64, _i32, P, _i32, _i32, _i32, _i32, P, P],
    'hla_s6_writer_project': [P, _i64, P, _i64, P, _i64, P, _i64, _i32, _i32, _i32, P],
    'hla_s6_writer_commit': [P, _i64, P, _i64, P, _i64, P, _i64, _i32, _i32, _i32, P, P, _i64, _i64, P, _i64, _i64,
                             _i64, _i32, P, _i64, _i32, P, _i32, P],
    'hla_s6_decode_prepare': [P, _i64, _i64, P, _i64, _i64, P, P, _i64, _i64, P, _i64, _i64, _i32, _i32, _i32, _i32,
                              P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, _i64, _i64,
                              _i32, P, _i64, _i32, P, _i32, P, _i32, P],
    'hla_s6_commit_rows': [P, _i64, _i32, P, P, _i64, _i64, P, _i64, _i64, _i64, _i32, P, _i64, _i32, P, _i32, _i32,
                           P, P],
    'hla_s6_decode_combine': [_i32, _i32, _i32, _i32, _i32, P, _i64, P, P, _i32, _i64, P, P, P, P, _i64, _i64, P,
                              _i64, _i64, P, _i64,
                              _i64, _i64, _i64, _i32, P, _i64, _i32, P, _i32, P, _i32, _f32, P, _i64, _i64, P, P,
                              _i64, _i64, P, _i32, P, P],
    'hla_s6_history_attention_contig': [P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, P, _i64, _i32, _i32, _i32,
                                        _i32, _f32, _i32, P, _i64, P, _i64, _i64, P, P, P, P],
    'hla_s6_export_rows': [P, P, _i32, _i64, _i64, _i64, _i32, _i32, P, _i64, _i64, _i64, _i64, _i32, _i32, P, _i64,
                           _i64, P, P, P],
    'hla_s6_history_attention_heads': [P, _i64, _i64, P, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32, P, _i64,
                                       _i32, P, _i32, _i32, _f32, _i32, P, _i64, P, P, _i64, _i64, P, P, P],
    'hla_s6_peer_alloc': [_i64, P, P],
    'hla_s6_peer_open': [P, P],
    'hla_s6_peer_close': [P],
    'hla_s6_peer_free': [P],
    'hla_s6_history_reduce_exchange': [_i32, _i32, _i32, _i32, _i32, P, _i64, P, P, P, _i32, _i32, P],
    'hla_s6_window_history': [P, _i64, _i64, P, _i64, _i64, _i64, _i64, _i32, P, _i64, _i32, P, _i32, _f32, _i32,
                              _i32, _i32, P, _i64, _i64, P, P],
    'hla_s6_step_metadata': [P, _i32, P, _i32, _i32, P, P, P, P, P, P, P, P, P],
    'hla_s6_gather_block_table': [P, _i64, _i32, _i32, P, _i32, P, _i64, P],
    'hla_s6_chunk_attention': [P, _i64, _i64, P, _i64, _i64, P, _i64, _i64, P, _i32, _i32, _i32, _i32, _f32, P, _i64,
                               _i64, P, P],
}

_lib = None


def load():
    """Load the library once; raises RuntimeError when it is absent or mismatched."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f'libhla_s6.so not found at {LIB_PATH}: build it with '
                           f'`python {_PKG / "build.py"}` (no CPU fallback exists)')
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.hla_s6_version.restype = ctypes.c_int
    lib.hla_s6_last_error.restype = ctypes.c_char_p
    if lib.hla_s6_version() != ABI_VERSION:
        raise RuntimeError(f'libhla_s6 ABI {lib.hla_s6_version()} != expected {ABI_VERSION}; rebuild it')
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int32
    lib.hla_s6_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
    lib.hla_s6_set_wait_limit_ns.restype = ctypes.c_uint64
    _lib = lib
    return lib


def set_wait_limit_ns(ns: int) -> int:
    """Limit (device ns) of the kernels' bounded waits for launches issued from now on; 0 restores the
    2 s default.  Returns the previous limit (``hla_s6_set_wait_limit_ns``)."""
    return int(load().hla_s6_set_wait_limit_ns(int(ns)))


def check(rc: int, what: str):
    if rc == OK:
        return
    msg = load().hla_s6_last_error().decode(errors='replace')
    if rc == EINVAL:
        raise ValueError(f'{what}: {msg}')
    raise RuntimeError(f'{what}: {msg}')


def call(name: str, *args):
    rc = getattr(load(), name)(*args)
    check(rc, name)


def ptr(t):
    """Device pointer of a tensor (None -> NULL; a ctypes pointer or an int passes through)."""
    if t is None or isinstance(t, ctypes.c_void_p):
        return t
    if isinstance(t, int):
        return ctypes.c_void_p(t)
    return ctypes.c_void_p(t.data_ptr())


def pointer_array(ptrs):
    """Host array of device pointers (ints or None) for the ``T* const*`` arguments."""
    return (ctypes.c_void_p * len(ptrs))(*[None if p is None else int(p) for p in ptrs])


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
