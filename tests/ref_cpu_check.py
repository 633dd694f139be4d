"""Run the reference's own lean path on the CPU with the torch-eager stand-ins of its Triton kernels
(`oracle/ref_cpu.py`) over the recorded tiny cases, and print the largest difference from the fixtures (which were
recorded with the real Triton kernels in Triton's interpreter). Runs in its own process: it replaces FlashInfer and
`torch.cuda.Event` for the whole interpreter.

    python tests/ref_cpu_check.py [reference source dir]
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(HERE, 'golden')]


def main():
    from morj_b200 import workloads
    from morj_b200.checkpoint import random_state
    from oracle.ref_cpu import load_reference, reference_model
    lean_core = load_reference(sys.argv[1] if len(sys.argv) > 1 else None, eager=True)
    assert lean_core._qkv_post.__class__.__name__ == '_Launchable'
    with open(os.path.join(HERE, 'golden', 'forward_tiny.json')) as f:
        cases = json.load(f)['cases']
    top = workloads.tiny_config()
    state = random_state(top, seed=0)
    worst = 0.0
    for c in cases:
        m = reference_model(lean_core, top, state, c['single_max'], c['step_tokens'])
        if c['retain_budget'] is not None:
            m.retain_budget = c['retain_budget']
        images = None
        if c['images']:
            from make_forward_golden import tiny_images
            images = tiny_images(top)
        req = m.prepare(c['seqs'], c['label_ids'], retain=c['retain'], images=images)
        assert (bool(req.retain), bool(req.pinned)) == (c['retained'], c['pinned']), c['name']
        for p, ref in zip(c['passes'], c['reference']):
            got = m.run(req, list(p))
            err = max(np.abs(np.asarray(a) - np.asarray(b)).max() for a, b in zip(got, ref))
            worst = max(worst, float(err))
    print(json.dumps({'cases': len(cases), 'max_abs': worst}))


if __name__ == '__main__':
    main()
