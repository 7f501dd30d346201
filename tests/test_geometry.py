"""Host-side geometry checks (reference hla/vllm_latent/geometry.py and ouro_latent.py:237-247). CPU."""
from types import SimpleNamespace as NS

import pytest
import torch

from conftest import pkg


def _config(**kw):
    base = dict(num_hidden_layers=24, hidden_size=2048, num_attention_heads=16, total_ut_steps=4,
                num_key_value_heads=16, rope_theta=1e6, rope_parameters={'rope_theta': 1e6})
    base.update(kw)
    return NS(**base)


CFG = dict(architecture='s6-block-v1', num_layers=24, hidden=2048, heads=16, head_dim=128, loops=4)


def test_validate_geometry_accepts_and_rejects():
    geo = pkg('geometry')
    geo.validate_geometry(_config(), CFG)
    with pytest.raises(ValueError, match='S6 block'):
        geo.validate_geometry(_config(), dict(CFG, architecture='other'))
    with pytest.raises(ValueError, match='loops mismatch'):
        geo.validate_geometry(_config(total_ut_steps=3), CFG)
    with pytest.raises(ValueError, match='multi-head'):
        geo.validate_geometry(_config(num_key_value_heads=8), CFG)


def test_rope_theta():
    geo = pkg('geometry')
    assert geo.rope_theta(_config()) == 1e6
    with pytest.raises(ValueError, match='default RoPE'):
        geo.rope_theta(_config(rope_parameters={'rope_theta': 1e6, 'rope_type': 'yarn'}))
    with pytest.raises(ValueError, match='default RoPE'):
        geo.rope_theta(_config(rope_parameters={'rope_theta': 1e4}))


def test_latent_cache_geometry():
    geo = pkg('geometry')
    caches = {512: torch.zeros(5, 1, 16, 1024, dtype=torch.bfloat16), 256: torch.zeros(5, 1, 16, 512, dtype=torch.bfloat16)}
    rec = geo.check_latent_caches(caches)
    assert rec['caches'][512][0] == [5, 1, 16, 1024]
    with pytest.raises(RuntimeError, match='unexpected latent cache geometry'):
        geo.check_latent_caches({512: torch.zeros(5, 1, 8, 1024, dtype=torch.bfloat16)})
    with pytest.raises(RuntimeError, match='no instance'):
        geo.check_latent_caches({512: torch.zeros(5, 1, 48, 1024, dtype=torch.bfloat16)})
    with pytest.raises(RuntimeError, match='bf16'):
        geo.check_latent_caches({512: torch.zeros(5, 1, 16, 1024)})
