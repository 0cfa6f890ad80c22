"""bench.py's JSON line on the CPU: the reference arm (`--impl reference`, the float32 port of
the reference's closed form on the host cores) prints one line with every key of the contract,
and a rank other than 0 prints nothing and exits 0."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--impl', 'reference',
                           '--steps', '1', '--warmup', '1'], capture_output=True, text=True,
                          env=env, timeout=300, cwd=ROOT)


def test_reference_arm_line():
    r = run({'RANK': '0', 'WORLD_SIZE': '1'})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step',
                'higher_is_better', 'scaling', 'vs_baseline', 'dtype', 'data', 'config', 'impl',
                'cpu_baseline', 'e2e'):
        assert key in line, key
    assert line['impl'] == 'reference' and line['value'] > 0 and line['steps'] == 1
    assert line['higher_is_better'] is True and line['unit'] == 'TFLOP/s'
    assert 'workload' in line['config']
    cb = line['cpu_baseline']
    assert cb['kind'] in ('port', 'reference') and cb['cores'] >= 1 and cb['sample']
    assert cb['value'] == line['value']
    e2e = line['e2e']
    assert e2e['value'] == line['value'] and e2e['unit'] == line['unit']
    assert e2e['h2d_bytes_per_step'] == 0 and e2e['d2h_bytes_per_step'] == 0


def test_reference_arm_other_ranks_silent():
    r = run({'RANK': '1', 'WORLD_SIZE': '2'})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ''
