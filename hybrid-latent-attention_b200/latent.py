"""S6 latent-layer weights with the reference's parameter names and shapes (hla/latent/register.py:28-95).

Only the data layout is mirrored here: ``cand_s`` (E_2..E_T, ``nn.Linear(hidden, rank + rank_v)``),
``cand1`` (E_1', ``nn.Linear(hidden, 2 * rank1)``), ``q_absorb`` ``[T-1, H, d, rank]``, ``out_absorb``
``[T-1, H, rank_v, d]``, ``q_absorb1`` ``[H, d, rank1]``, ``out_absorb1`` ``[H, rank1, d]``, so a
reference student state dict loads strictly.  All arithmetic on them runs in the B200 kernels
(``s6_layer``); the reference's torch methods (write_step, pack, scores, ...) are not reproduced.
"""
from __future__ import annotations

import math

import torch
from torch import nn

ARCHITECTURE = 's6-block-v1'


class LatentLayer(nn.Module):
    def __init__(self, hidden, heads, head_dim, loops, rank, rank_v, rank1):
        super().__init__()
        if loops < 2 or min(rank, rank_v, rank1) < 1 or rank % 2 or rank1 % 2:
            raise ValueError('S6 requires T>=2, positive K/V/rank1 and even K ranks')
        self.hidden, self.heads, self.head_dim = hidden, heads, head_dim
        self.loops, self.rank, self.rank_v, self.rank1 = loops, rank, rank_v, rank1
        self.cand_s = nn.ModuleList(nn.Linear(hidden, rank + rank_v, bias=False) for _ in range(loops - 1))
        self.cand1 = nn.Linear(hidden, 2 * rank1, bias=False)
        self.q_absorb = nn.Parameter(torch.empty(loops - 1, heads, head_dim, rank))
        self.out_absorb = nn.Parameter(torch.empty(loops - 1, heads, rank_v, head_dim))
        self.q_absorb1 = nn.Parameter(torch.empty(heads, head_dim, rank1))
        self.out_absorb1 = nn.Parameter(torch.empty(heads, rank1, head_dim))
        for p in (self.q_absorb, self.out_absorb, self.q_absorb1, self.out_absorb1):
            nn.init.normal_(p, std=1 / math.sqrt(hidden))

    def readers(self, loop):
        """``(A, B, width)`` of a loop: loop 0 reads the loop-1 latent, later loops the main latent."""
        if loop == 0:
            return self.q_absorb1, self.out_absorb1, self.rank1
        return self.q_absorb[loop - 1], self.out_absorb[loop - 1], self.rank

    def writer(self, loop):
        """The projection weight written at ``loop`` (E_1' at loop 0, E_{loop+1} after)."""
        return self.cand1.weight if loop == 0 else self.cand_s[loop - 1].weight


class LatentStudent(nn.Module):
    """Per-layer S6 students (register.py:98-119): same config keys and strict checkpoint load."""

    def __init__(self, num_layers, hidden, heads, head_dim, loops=4, rank=512, rank_v=512, rank1=256,
                 architecture=ARCHITECTURE):
        super().__init__()
        if architecture != ARCHITECTURE:
            raise ValueError('Only S6 block checkpoints are supported')
        self.cfg = dict(num_layers=num_layers, hidden=hidden, heads=heads, head_dim=head_dim, loops=loops, rank=rank,
                        rank_v=rank_v, rank1=rank1, architecture=architecture)
        self.layers = nn.ModuleList(LatentLayer(hidden, heads, head_dim, loops, rank, rank_v, rank1)
                                    for _ in range(num_layers))

    def cache_bytes_per_token(self, dtype_bytes=2):
        c = self.cfg
        return c['num_layers'] * (c['rank'] + c['rank_v'] + 2 * c['rank1']) * dtype_bytes

    @classmethod
    def from_checkpoint(cls, checkpoint, device='cpu'):
        state = checkpoint['student']
        cfg = dict(checkpoint['cfg'])
        if cfg.pop('gated', False) or any('.inter_s.' in k for k in state):
            raise ValueError('Gated-residual S6 checkpoints are no longer supported')
        cfg.pop('bottleneck', None)
        cfg.pop('legacy', None)
        student = cls(**cfg).to(device)
        student.load_state_dict(state, strict=True)
        if any(not torch.isfinite(p).all() for p in student.parameters()):
            raise ValueError('Nonfinite student checkpoint')
        return student
