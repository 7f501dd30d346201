"""Record the public call signatures of the reference modules this package mirrors.

Usage (needs the reference checkout, read-only):
    python tests/golden/gen_api.py --reference /path/to/hybrid-latent-attention

Writes tests/golden/api_signatures.json: for every public function (and the methods of the classes
listed below) of hla/vllm_latent/s6_ops.py, hla/vllm_latent/s6_layer.py and
hla/latent/fused_history.py, its parameter names, kinds and defaults (inspect.signature).  The
reference modules import without vLLM or a GPU (their GPU imports are lazy, s6_ops.py:3-5).
"""
from __future__ import annotations

import argparse
import os
import importlib
import inspect
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
# module (as this package names it) -> (reference module, public names the mirror must provide)
MIRRORED = {
    's6_ops': ('hla.vllm_latent.s6_ops',
               ['latent_rope', 'token_requests', 'history_lengths', 'num_kv_splits', 'S6Workspace',
                'history_attention', 'history_attention_kv', 'chunk_attention', 'merge_states', 'window_attention_fa',
                'window_history_fa', 'merge_lse', 'select_backends', 'probe_latent_rope']),
    's6_layer': ('hla.vllm_latent.s6_layer',
                 ['latent_inv_freq', 'latent_rope_table', 'latent_query', 'StepContext', 'attend', 'write_rows',
                  'committed_row']),
    'fused_history': ('hla.latent.fused_history', ['history_attention']),
}


def param_text(p):
    """'name', 'name=default', '*name', '**name'; keyword-only parameters follow a bare '*'."""
    if p.kind is p.VAR_POSITIONAL:
        return '*' + p.name
    if p.kind is p.VAR_KEYWORD:
        return '**' + p.name
    return p.name if p.default is inspect.Parameter.empty else f'{p.name}={p.default!r}'


def signature_text(fn):
    """Parameter list of fn as strings, with '*' before the first keyword-only parameter."""
    out, star = [], False
    for p in inspect.signature(fn).parameters.values():
        if p.kind is p.KEYWORD_ONLY and not star:
            out.append('*')
            star = True
        if p.kind is p.VAR_POSITIONAL:
            star = True
        out.append(param_text(p))
    return out


def describe(obj):
    """Parameters of a function, or of a class's __init__ and public methods."""
    params = signature_text
    if inspect.isclass(obj):
        methods = {'__init__': params(obj.__init__)}
        for name, member in vars(obj).items():
            if not name.startswith('_') and inspect.isfunction(member):
                methods[name] = params(member)
        return {'class': methods}
    return {'function': params(obj)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', default=os.environ.get('HLA_REFERENCE_ROOT'),
                    help='checkout of the reference project (default: $HLA_REFERENCE_ROOT)')
    args = ap.parse_args()
    if not args.reference:
        ap.error('pass --reference or set HLA_REFERENCE_ROOT to a checkout of the reference project')
    sys.path.insert(0, args.reference)
    table = {}
    for mine, (ref_name, names) in MIRRORED.items():
        mod = importlib.import_module(ref_name)
        table[mine] = {'reference': ref_name, 'api': {n: describe(getattr(mod, n)) for n in names}}
    (HERE / 'api_signatures.json').write_text(json.dumps(table, sort_keys=True, indent=None) + '\n')
    print('wrote api_signatures.json:', {k: len(v['api']) for k, v in table.items()})


if __name__ == '__main__':
    main()
