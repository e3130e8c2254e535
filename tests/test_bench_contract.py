"""The benchmark's JSON-line contract on CPU: the reference arm (the reference's eager PyTorch step, restated in
oracle/, on the host cores) prints one line with the metric, unit, config and the cpu_baseline / e2e objects the
driver reads, for every configuration (1, the default; 2, growing; 3, no-grad rollouts; 4, the 256 x 256 shard)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize('config,metric,hw', [(1, 'cell-updates/s fwd+bwd, 64-step rollout', 128),
                                              (2, 'cell-updates/s fwd+bwd, 80-step rollout', 72),
                                              (3, 'cell-updates/s no-grad, 128-step rollout', 256),
                                              (4, 'cell-updates/s fwd+bwd, 96-step rollout', 256)])
def test_reference_arm_prints_one_contract_line(config, metric, hw):
    out = subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--impl', 'reference', '--steps', '1',
                          '--warmup', '0', '--config', str(config)], capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, RANK='0'))
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d['impl'] == 'reference' and d['metric'] == metric and d['unit'] == 'cell-updates/s'
    assert d['higher_is_better'] is True and d['value'] > 0 and d['steps'] == 1 and d['warmup'] == 0
    assert d['config']['H'] == hw and d['config']['W'] == hw
    assert d['cpu_baseline']['value'] == d['value'] and d['cpu_baseline']['cores'] >= 1
    assert d['e2e'] == {'value': d['value'], 'unit': d['unit'], 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}
