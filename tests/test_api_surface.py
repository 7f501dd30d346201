"""The drop-in boundary, checked without a GPU:

* every public function and class of the reference modules this package mirrors (s6_ops, s6_layer,
  fused_history) exists here with the same parameters, order and defaults, as recorded from the
  reference by tests/golden/gen_api.py (inspect.signature) in tests/golden/api_signatures.json;
* the hot-path ops are sync-free and loop-free on the host, the contract the reference states for
  its serving path (s6_ops.py:1-10; the adapter's AST test, test_ouro_latent_static.py:61-72): no
  .item() / .tolist() / .cpu() / .nonzero() / .numpy(), and no Python loop except over a literal tuple
  of arguments (never over tokens, requests or a tensor).
"""
import ast
import inspect
import json
import sys
from pathlib import Path

import pytest

from conftest import GOLDEN, ROOT, pkg

sys.path.insert(0, str(GOLDEN))
from gen_api import signature_text  # noqa: E402

TABLE = json.loads((GOLDEN / 'api_signatures.json').read_text())
CASES = [(mod, name) for mod, entry in TABLE.items() for name in entry['api']]
SYNC_ATTRS = {'item', 'tolist', 'cpu', 'nonzero', 'numpy'}
# the ops a serving step calls (s6_layer's decode / prefill branches and the HF reader)
HOT = {'s6_ops': ['history_attention', 'history_attention_kv', '_history_heads', 'chunk_attention', 'merge_states',
                  'merge_lse', 'window_attention_fa', 'window_history_fa', 'latent_rope', 'token_requests',
                  'history_lengths'],
       's6_layer': ['latent_query', 'attend', 'write_rows', 'committed_row'],
       'fused_history': ['history_attention', 'forward']}


@pytest.mark.parametrize('mod,name', CASES)
def test_signature_matches_the_reference(mod, name):
    ref = TABLE[mod]['api'][name]
    mine = getattr(pkg(mod), name, None)
    assert mine is not None, f'{mod}.{name} is missing'
    if 'function' in ref:
        assert signature_text(mine) == ref['function'], f'{mod}.{name}'
    else:
        for meth, params in ref['class'].items():
            fn = getattr(mine, meth, None)
            assert fn is not None, f'{mod}.{name}.{meth} is missing'
            assert signature_text(fn) == params, f'{mod}.{name}.{meth}'


@pytest.mark.parametrize('mod', sorted(HOT))
def test_hot_path_is_sync_free_and_loop_free(mod):
    path = ROOT / 'hybrid-latent-attention_b200' / f'{mod}.py'
    tree = ast.parse(path.read_text())
    fns = {n.name: n for n in tree.body if isinstance(n, ast.FunctionDef)}
    for name in HOT[mod]:
        assert name in fns, f'{mod}.{name}'
        for node in ast.walk(fns[name]):
            if isinstance(node, ast.Attribute):
                assert node.attr not in SYNC_ATTRS, f'{mod}.{name}: .{node.attr} syncs with the host'
            assert not isinstance(node, ast.While), f'{mod}.{name}: a while loop on the serving path'
            # loops only over a literal tuple / list (argument checks of a fixed set of tensors),
            # never over tokens, requests or a tensor
            if isinstance(node, (ast.For, ast.comprehension)):
                assert isinstance(node.iter, (ast.Tuple, ast.List)), \
                    f'{mod}.{name}: a Python loop over {ast.unparse(node.iter)} on the serving path'


def test_reference_signature_fixture_covers_the_mirrored_modules():
    assert {m: TABLE[m]['reference'] for m in TABLE} == {
        's6_ops': 'hla.vllm_latent.s6_ops', 's6_layer': 'hla.vllm_latent.s6_layer',
        'fused_history': 'hla.latent.fused_history'}
    assert len(CASES) == 22
    assert inspect.isfunction(signature_text)
