"""bench.py's reference arm on the CPU: the reference's own CPU SpMM (or the C
restatement when the reference core is not built) on the native arm's
workload and format, printing one JSON line of the bench contract."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--impl', 'reference', *args],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith('{')]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize('config,gen_kw,fmt,nnz', [
    ('c1_laplacian2d', '{"n": 48}', 'boo', 5 * 48 * 48 - 4 * 48),
    ('c5_uniform', '{"n": 4096}', 'pbr', 8 * 4096),
])
def test_reference_arm_line(config, gen_kw, fmt, nnz):
    d = _run('--config', config, '--gen-kw', gen_kw, '--steps', '2', '--warmup', '1')
    assert d['impl'] == 'reference'
    assert d['config']['workload'] == config and d['config']['format'] == fmt
    assert d['config']['nnz'] == nnz
    assert d['unit'] == 'GFLOP/s' and d['higher_is_better'] is True and d['steps'] == 2
    assert d['value'] > 0 and d['cpu_baseline']['value'] == d['value']
    assert d['cpu_baseline']['kind'] in ('reference', 'port') and d['cpu_baseline']['cores'] >= 1
    assert d['e2e'] == {'value': d['value'], 'unit': 'GFLOP/s', 'h2d_bytes_per_step': 0,
                        'd2h_bytes_per_step': 0}


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK='1')
    r = subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--impl', 'reference',
                        '--config', 'c1_laplacian2d', '--gen-kw', '{"n": 16}', '--steps', '1'],
                       capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert r.returncode == 0 and not [ln for ln in r.stdout.splitlines() if ln.startswith('{')]


@pytest.mark.parametrize('fmt', ['boo', 'pbr'])
def test_cpu_baseline_and_build_line(fmt):
    import bench
    from spmm_b200 import workloads as W
    mat = W.laplacian2d(n=64)
    x = W.dense_x(mat.shape[1], 32, seed=0).numpy()
    cpu = bench.cpu_baseline(mat, W.CONFIGS['c1_laplacian2d'], x, fmt, budget_s=0.5)
    assert cpu['value'] > 0 and cpu['cores'] == 1 and cpu['kind'] in ('reference', 'port')
    assert cpu['build_nnz'] == mat[:mat.shape[0] // 16].nnz and cpu['build_s'] > 0
    line = bench.build_line(0.25, mat.nnz, cpu)
    assert line['gpu_nnz_per_s'] == round(mat.nnz / 0.25)
    assert line['cpu_nnz_per_s'] == round(cpu['build_nnz'] / cpu['build_s'])
    assert line['gpu_over_cpu'] == round(line['gpu_nnz_per_s'] / line['cpu_nnz_per_s'], 2)
    assert 'cpu_reference_s' not in bench.build_line(0.25, mat.nnz, None)
