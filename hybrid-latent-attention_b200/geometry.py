"""Model / checkpoint / cache geometry checks of the S6 serving adapter, host-side only.

Mirrors hla/vllm_latent/geometry.py (validate_geometry :4-16, rope_theta :19-25) and the one-shot
S6_RUNTIME_CHECK of the paged-cache geometry (ouro_latent.py:237-247), extended with what the B200
kernels themselves require of the latent caches, so that an adapter fails at start-up with a
readable message instead of at the first launch.
"""
from __future__ import annotations

from .latent import ARCHITECTURE

# B200 history kernel: latent widths and page sizes it is instantiated for (csrc/history.cu)
KERNEL_WIDTHS = (256, 512, 1024)
KERNEL_PAGES = {256: (16, 32), 512: (16, 32), 1024: (16,)}


def validate_geometry(config, latent_cfg):
    """Reject model/checkpoint policies the adapter cannot execute (geometry.py:4-16): an S6 block
    checkpoint whose layer count, hidden size, heads, head dim and loop count match the model, and
    multi-head attention."""
    if latent_cfg.get('architecture') != ARCHITECTURE:
        raise ValueError('Only S6 block checkpoints are supported')
    expected = dict(num_layers=config.num_hidden_layers, hidden=config.hidden_size, heads=config.num_attention_heads,
                    head_dim=config.hidden_size // config.num_attention_heads, loops=config.total_ut_steps)
    for key, value in expected.items():
        if latent_cfg.get(key) != value:
            raise ValueError(f'S6 model/checkpoint {key} mismatch: {value} != {latent_cfg.get(key)}')
    if config.num_key_value_heads != config.num_attention_heads:
        raise ValueError('S6 adapter requires multi-head attention')


def rope_theta(config) -> float:
    """The teacher's RoPE base from ``rope_parameters`` (geometry.py:19-25): default RoPE only, and
    ``rope_parameters.rope_theta`` must agree with ``rope_theta``."""
    params = config.rope_parameters
    theta = params['rope_theta']
    if params.get('rope_type', 'default') != 'default' or theta != config.rope_theta:
        raise ValueError(f'S6 requires default RoPE with rope_parameters.rope_theta == rope_theta: {params}, '
                         f'{config.rope_theta}')
    return float(theta)


def check_latent_caches(caches: dict) -> dict:
    """``{width: cache}`` of the latent caches (vLLM TRITON_ATTN layout ``[num_blocks, 1, block, 2 * width]``)
    -> the runtime-check record the reference prints (ouro_latent.py:243-246).  Raises RuntimeError for a
    layout the reference rejects (block not a multiple of 16, last dim != 2 * width) or the B200 kernels
    cannot read (width / block size outside their instantiations, non-bf16, misaligned rows)."""
    record = {}
    for w, c in caches.items():
        shape, stride = tuple(c.shape), tuple(c.stride())
        if len(shape) != 4 or shape[1] != 1 or shape[2] % 16 or shape[-1] != 2 * w:
            raise RuntimeError(f'unexpected latent cache geometry: {shape}')
        if w not in KERNEL_WIDTHS or shape[2] not in KERNEL_PAGES[w]:
            raise RuntimeError(f'B200 history kernel has no instance for width {w} with block size {shape[2]}')
        if str(c.dtype) != 'torch.bfloat16' or stride[-1] != 1 or stride[0] % 8 or stride[2] % 8:
            raise RuntimeError(f'B200 latent cache must be bf16 with 16-byte aligned rows: {str(c.dtype)} {stride}')
        record[w] = [list(shape), list(stride), str(c.dtype)]
    return {'caches': record}
