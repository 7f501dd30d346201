"""The C-ABI library builds, loads and exports every entry point include/hla_s6.h declares;
host-side validation returns the documented status codes without touching a GPU.  CPU only."""
import ctypes
import re

import pytest

from conftest import ROOT, pkg

HEADER = ROOT / 'include' / 'hla_s6.h'


@pytest.fixture(scope='module')
def lib():
    build = pkg('build')
    build.build()
    return pkg('_lib').load()


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r'^\s*(?:int|const char\*|void|uint64_t)\s+(hla_s6_\w+)\s*\(', text, re.M)))


def test_header_declares_the_boundary():
    names = declared()
    assert 'hla_s6_history_attention' in names and 'hla_s6_version' in names
    assert len(names) >= 6


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), f'{name} declared in include/hla_s6.h but not exported'


def test_abi_version_and_bindings(lib):
    _lib = pkg('_lib')
    assert lib.hla_s6_version() == _lib.ABI_VERSION
    for name in _lib.SIGNATURES:
        assert name in declared(), f'{name} bound in _lib.py but not declared in the header'


def test_invalid_arguments_return_einval_with_message(lib):
    _lib = pkg('_lib')
    fn = lib.hla_s6_history_attention
    # page 5 is rejected on the host before any device work
    rc = fn(None, 0, 0, None, 1, 0, 0, None, 0, 0, None, None, 1, 16, 512, 5, 1.0, 1, None, 0, None, 0, 0, None,
            None, None)
    assert rc == _lib.EINVAL
    assert b'page' in lib.hla_s6_last_error()
    rc = fn(None, 0, 0, None, 1, 0, 0, None, 0, 0, None, None, 1, 17, 512, 16, 1.0, 1, None, 0, None, 0, 0, None,
            None, None)
    assert rc == _lib.EINVAL and b'heads' in lib.hla_s6_last_error()


def test_wait_limit_is_process_wide_and_restorable(lib):
    _lib = pkg('_lib')
    prev = _lib.set_wait_limit_ns(5_000_000)
    try:
        assert prev == 2_000_000_000
        assert _lib.set_wait_limit_ns(7_000_000) == 5_000_000
    finally:
        assert _lib.set_wait_limit_ns(0) == 7_000_000      # 0 restores the 2 s default
    assert _lib.set_wait_limit_ns(0) == 2_000_000_000


def test_workspace_overflow_is_reported(lib):
    _lib = pkg('_lib')
    mode, grid, slots = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    T, H, W, splits = 64, 16, 512, 16
    need = T * splits * H * (W + 1)
    rc = lib.hla_s6_history_plan(T, H, W, 16, splits, need - 1, ctypes.byref(mode), ctypes.byref(grid),
                                 ctypes.byref(slots))
    assert rc == _lib.EOVERFLOW and b'overflow' in lib.hla_s6_last_error()
    rc = lib.hla_s6_history_plan(T, H, W, 16, splits, need, ctypes.byref(mode), ctypes.byref(grid),
                                 ctypes.byref(slots))
    assert rc == _lib.OK
    assert mode.value == 1 and grid.value >= 1 and grid.value + T - 1 <= slots.value
    # one split per row: one CTA per row, one slot per row
    rc = lib.hla_s6_history_plan(T, H, W, 16, 1, T * H * (W + 1), ctypes.byref(mode), ctypes.byref(grid),
                                 ctypes.byref(slots))
    assert rc == _lib.OK and mode.value == 0 and grid.value == T and slots.value == T


def test_ops_reject_cpu_tensors_and_unknown_backends():
    import torch
    ops = pkg('s6_ops')
    q = torch.zeros(1, 16, 512, dtype=torch.bfloat16)
    cache = torch.zeros(2, 1, 16, 1024, dtype=torch.bfloat16)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    ctx = torch.zeros(1, dtype=torch.int32)
    ws = ops.S6Workspace(16, 512, 16)
    with pytest.raises(ValueError, match='Unknown history backend'):
        ops.history_attention(q, cache, bt, ctx, 1.0, 1, ws, None, None, 'torch')
    with pytest.raises(ValueError, match='CUDA'):
        ops.history_attention(q, cache, bt, ctx, 1.0, 1, ws, None, None, 'b200')


def test_python_constants_match_the_header_defines():
    """Every status code, device error code, launch flag and size that _lib.py mirrors from
    include/hla_s6.h carries the header's value."""
    _lib = pkg('_lib')
    defines = {m.group(1): int(m.group(2))
               for m in re.finditer(r'^#define HLA_S6_(\w+)\s+(\d+)\s*$', HEADER.read_text(), re.M)}
    mirrored = ['OK', 'EINVAL', 'EOVERFLOW', 'ECUDA', 'ERR_WAIT_COPY', 'ERR_WAIT_STAGE', 'ERR_RANGE', 'ERR_WAIT_PEER',
                'ERR_BLOCK', 'COMBINE_AFTER_PARTIALS', 'PARTIALS_AFTER_QUERY', 'REDUCE_AFTER_PARTIALS',
                'PREPARE_EARLY_LAUNCH', 'PREPARE_EXACT_ONLY', 'PEER_HANDLE_BYTES', 'EXCHANGE_WORD_BYTES']
    for name in mirrored:
        assert getattr(_lib, name) == defines[name], name
    assert _lib.ABI_VERSION == defines['ABI_VERSION']


def test_prepare_exact_part_alone_needs_k(lib):
    """HLA_S6_PREPARE_EXACT_ONLY without k is refused on the host (EINVAL) before any launch."""
    _lib = pkg('_lib')
    T, H, d, W = 1, 16, 128, 512
    rc = lib.hla_s6_decode_prepare(None, 0, 0, None, 0, 0, None, None, W, 1, None, 0, 0, T, H, d, W, None, 0, 0,
                                   None, 0, 0, None, 0, 0, None, 128, 1, None, 1, 0, 0, 0, 16, None, 0, 1, None, 1,
                                   None, _lib.PREPARE_EXACT_ONLY, None)
    assert rc == _lib.EINVAL
    assert b'exact part alone needs k' in lib.hla_s6_last_error()
