"""The CPU reference runner (`oracle/ref_cpu.py`) that the benchmark's reference arm times: the reference's own
`LeanGemma4.prepare` / `run` with torch-eager stand-ins for its three Triton kernels reproduces the probabilities
recorded with the real Triton kernels (interpreted), on every recorded case; and the timed 3-layer cut stamps each
layer. Needs the reference package installed under `baseline/_ref` (skipped otherwise)."""
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), 'baseline', '_ref')

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, 'aleria_judge')),
                                reason='reference package not installed under baseline/_ref')


def test_eager_standins_reproduce_the_reference_fixtures():
    out = subprocess.run([sys.executable, os.path.join(HERE, 'ref_cpu_check.py')], capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res['cases'] == 7 and res['max_abs'] < 2e-3, res


def test_timed_reference_stamps_every_layer_and_loads_no_native_library():
    code = r'''
import json, sys
sys.path.insert(0, %r)
from morj_b200 import workloads
from oracle.ref_cpu import TimedReference
top = dict(workloads.tiny_config())
cfg = dict(top['text_config'], layer_types=['sliding_attention'] * 5 + ['full_attention'], num_hidden_layers=6)
tr = TimedReference(dict(top, text_config=cfg), workloads.tiny_tree(0))
r = tr.sample()
plan = tr.plan_of_last_request()
maps = open('/proc/self/maps').read()
print(json.dumps(dict(r=r, extra=tr.extrapolate(r), steps=len(plan['steps']), native='_morj_b200' in maps)))
''' % os.path.dirname(HERE)
    out = subprocess.run([sys.executable, '-c', code], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    r = res['r']
    assert r['tokens'] == 128 + 4 * 24 and res['steps'] == 1 and not res['native']
    assert min(r['setup'], r['sliding'], r['global_'], r['last']) > 0
    want = r['setup'] + 5 * r['sliding'] + r['last']  # 5 sliding layers, then the pruned global last layer
    assert abs(res['extra'] - want) < 1e-9
