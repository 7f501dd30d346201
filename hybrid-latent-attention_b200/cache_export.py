"""Rollout cache export (format ``s6-rollout-cache-v1``) on the B200 gather kernel.

Mirrors the data path of hla/vllm_latent/cache_export.py: RolloutCacheExporter.export
(:160-188) gathers, for one finished request, positions 0 .. length-1 of every layer's main and
loop-1 paged latent caches through each kv group's physical block list, concatenates main | l1
per layer into ``[1, length, 2 rank + 2 rank1]`` rows, moves them to the CPU and ``torch.save``s
them with the request's metadata.  Here the gather of all layers is one kernel launch
(csrc/export.cu) into one device buffer, followed by a single copy into pinned host memory.

The vLLM runner hooks around it (request bookkeeping, scheduler block lists, logits capture) are
serving control plane and stay with the engine; ``export_rows`` and ``write_snapshot`` are the
parts they call.
"""
from __future__ import annotations

from pathlib import Path

import torch

from . import _lib

SCHEMA = 's6-rollout-cache-v1'


def _check_cache(cache, block_size):
    # the reference's layout guard (cache_export.py:166-167)
    if cache.ndim != 4 or cache.shape[1] != 1 or cache.shape[2] != block_size:
        raise RuntimeError('Unsupported TRITON_ATTN cache layout')


def export_rows(main_caches, l1_caches, main_blocks, l1_blocks, length, block_size, l1_block_size=None):
    """Per-layer rows ``[1, length, main_w + l1_w]`` (CPU, the caches' dtype) of one request.

    main_caches / l1_caches: per-layer paged caches ``[nb, 1, block_size, w]`` (bf16, CUDA);
    main_blocks / l1_blocks: the request's physical block ids in each kv group (``blocks[pos //
    block_size]`` holds position pos), any integer tensor or sequence.  Raises IndexError when a list
    does not cover ``length`` positions or names a block outside its cache, as the reference's
    indexing would."""
    l1_block_size = block_size if l1_block_size is None else l1_block_size
    L = len(main_caches)
    if L != len(l1_caches) or L < 1:
        raise ValueError('one main and one loop-1 cache per layer')
    for m, l in zip(main_caches, l1_caches):
        _check_cache(m, block_size)
        _check_cache(l, l1_block_size)
    m0, l0 = main_caches[0], l1_caches[0]
    dev = m0.device
    if m0.dtype != torch.bfloat16 or l0.dtype != torch.bfloat16 or not m0.is_cuda:
        raise ValueError('the B200 export takes bf16 CUDA caches')
    for group, first in ((main_caches, m0), (l1_caches, l0)):
        for c in group:
            if c.shape != first.shape or c.stride() != first.stride() or c.dtype != first.dtype:
                raise ValueError("every layer must share its kv group's cache geometry")
    length = int(length)
    mb = torch.as_tensor(main_blocks).to(device=dev, dtype=torch.int32).contiguous()
    lb = torch.as_tensor(l1_blocks).to(device=dev, dtype=torch.int32).contiguous()
    if -(-length // block_size) > mb.numel() or -(-length // l1_block_size) > lb.numel():
        raise IndexError('the block list does not cover the exported positions')
    mw, lw = m0.shape[-1], l0.shape[-1]
    out = torch.empty(L, length, mw + lw, dtype=m0.dtype, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call('hla_s6_export_rows', _lib.pointer_array([c.data_ptr() for c in main_caches]),
              _lib.pointer_array([c.data_ptr() for c in l1_caches]), L, m0.shape[0], m0.stride(0), m0.stride(2), mw,
              block_size, _lib.ptr(mb), mb.numel(), l0.shape[0], l0.stride(0), l0.stride(2), lw, l1_block_size,
              _lib.ptr(lb), lb.numel(), length, _lib.ptr(out), _lib.ptr(err), _lib.stream_of(out))
    host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    host.copy_(out, non_blocking=True)
    torch.cuda.current_stream(dev).synchronize()
    if int(err.item()):
        raise IndexError('a block id of the request lies outside its cache')
    return tuple(host[i:i + 1] for i in range(L))


def write_snapshot(directory, index, version, request_id, cfg, prompt_ids, length, first_response_logits, rows):
    """Write ``<directory>/<index>.pt`` with the reference's payload (cache_export.py:175-188): written
    to ``.tmp`` first and renamed.  Returns the exporter's per-request record."""
    path = Path(directory) / f'{index}.pt'
    payload = dict(schema=SCHEMA, version=version, request_id=request_id, cfg=cfg, prompt_ids=list(prompt_ids),
                   length=int(length), first_response_logits=first_response_logits, rows=tuple(rows))
    temp = path.with_suffix('.tmp')
    torch.save(payload, temp)
    temp.replace(path)
    return dict(path=str(path), request_id=request_id, version=version, length=int(length),
                bytes=path.stat().st_size)
