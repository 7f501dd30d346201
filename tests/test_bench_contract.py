"""bench.py's output contract, checked on the CPU through its reference arm (the oracle port timed on
the host cores): one JSON line carrying every key the contract names, the reference arm's
cpu_baseline / e2e objects, and the rank rule (under torchrun only rank 0 runs and prints; the other
ranks exit 0 without work).  The GPU arm prints the same keys plus roofline, clocks and gpu_launches
(covered on a B200 by the bench runs themselves)."""
import json
import os
import subprocess
import sys

from conftest import ROOT

KEYS = {'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better', 'scaling',
        'vs_baseline', 'dtype', 'data', 'config'}


def run_bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / 'bench.py'), *args], capture_output=True, text=True, env=e,
                          timeout=600)


def test_reference_arm_prints_one_contract_line():
    p = run_bench('--impl', 'reference', '--steps', '1', '--warmup', '3', '--cpu-reps', '2')
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith('{')]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert KEYS <= set(line), KEYS - set(line)
    assert line['impl'] == 'reference' and line['n_gpus'] == 1 and line['steps'] == 1 and line['warmup'] == 3
    assert line['value'] > 0 and line['higher_is_better'] is True and line['vs_baseline'] is None
    assert line['metric'].startswith('S6 decode tokens/s') and line['unit'] == 'tokens/s'
    cpu = line['cpu_baseline']
    assert cpu['kind'] == 'port' and cpu['cores'] >= 1 and cpu['value'] == line['value'] and cpu['sample']
    assert line['e2e'] == {'value': line['value'], 'unit': 'tokens/s', 'h2d_bytes_per_step': 0,
                           'd2h_bytes_per_step': 0}


def test_reference_arm_runs_on_rank_zero_only():
    p = run_bench('--impl', 'reference', '--steps', '1', '--warmup', '3', '--cpu-reps', '2',
                  env={'RANK': '1', 'WORLD_SIZE': '2', 'LOCAL_RANK': '1'})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith('{')]


def test_warmup_below_three_is_refused():
    p = run_bench('--impl', 'reference', '--steps', '1', '--warmup', '2')
    assert p.returncode != 0 and 'warmup' in (p.stdout + p.stderr)
