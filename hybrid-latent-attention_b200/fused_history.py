"""Contiguous-layout latent history reader of the HF reference engines, on the B200 kernels.

Mirrors hla/latent/fused_history.py (history_attention, :49-54) and the forward of
hla/latent/history_kernels.py (forward, :84-89; the Triton _forward, :11-33): per row b and head h,

    z[b, h]   = softmax_n(scale * q[b, h] . k[b, n]  over keys with mask[b, n]) . v[b, :]
    lse[b, h] = logsumexp of the same scores (natural log)

with q [B, H, R], k / v [B, N, R] (one K/V row shared by the H heads), mask [B, N] bool.  A row
with no visible key gives z = 0 and lse = -inf (fused_history.reference, :11-20).

The kernel is the paged reader's (csrc/history.cu) with a contiguous front end: each 16-key tile
of a row is fetched by two TMA maps (K, V) into the same shared-memory layout as a cache page,
the mask is applied per key, and the rows' tiles are stream-K balanced over the SMs; partials are
merged by the block-cooperative reduce.  Forward only: the reference's analytical backward
(history_kernels.backward) is training-side and out of scope here, so inputs that require grad
are refused.  There is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib, s6_ops

SPLIT_MAX_TOKENS = 512


def _check(q, k, v, mask):
    # the reference's own shape contract (fused_history.py:50-51)
    if (q.ndim != 3 or k.ndim != 3 or k.shape != v.shape or mask.shape != k.shape[:2] or q.shape[0] != k.shape[0]
            or q.shape[-1] != k.shape[-1]):
        raise ValueError('Expected Q[B,H,R], K/V[B,N,R], mask[B,N]')


def forward(q, k, v, mask, scale):
    """``(z, lse, z32)`` like history_kernels.forward (history_kernels.py:84-89): z in q's dtype
    (bf16), lse fp32 [B, H], z32 the fp32 result before rounding."""
    _check(q, k, v, mask)
    if k.shape[1] < 1:
        raise ValueError('History must contain a storage row')
    if not q.is_cuda:
        raise RuntimeError('the B200 contiguous history reader needs CUDA tensors (no CPU path)')
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError('the B200 contiguous history reader takes bf16 q, k and v')
    B, H, R = q.shape
    N = k.shape[1]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    m = mask.contiguous()
    m = m.view(torch.uint8) if m.dtype == torch.bool else (m != 0).to(torch.uint8)
    props = torch.cuda.get_device_properties(q.device)
    splits = s6_ops.num_kv_splits(N, B, SPLIT_MAX_TOKENS, props.multi_processor_count)
    ws = torch.empty(max(1, B * splits * H * (R + 1)), dtype=torch.float32, device=q.device)
    z = torch.empty_like(q)
    z32 = torch.empty(B, H, R, dtype=torch.float32, device=q.device)
    lse = torch.empty(B, H, dtype=torch.float32, device=q.device)
    _lib.call('hla_s6_history_attention_contig', _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(k), k.stride(0),
              k.stride(1), _lib.ptr(v), v.stride(0), v.stride(1), _lib.ptr(m), m.stride(0), B, N, H, R, float(scale),
              int(splits), _lib.ptr(ws), ws.numel(), _lib.ptr(z), z.stride(0), z.stride(1), _lib.ptr(z32),
              _lib.ptr(lse), None, _lib.stream_of(q))
    return z, lse, z32


def history_attention(q, k, v, mask, scale, reference_forward=False):
    """``(z, lse)`` of the contiguous reader (fused_history.history_attention, :49-54), forward only."""
    _check(q, k, v, mask)
    if reference_forward:
        raise ValueError('reference_forward selects the reference torch path, which this backend does not run')
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        raise NotImplementedError('the B200 contiguous history reader is forward-only (backward is training-side)')
    z, lse, _ = forward(q, k, v, mask, scale)
    return z, lse
