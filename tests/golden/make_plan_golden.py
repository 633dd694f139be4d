"""Record the reference planner's outputs as fixtures (run in a container that holds the reference source).

    python tests/golden/make_plan_golden.py /path/to/reference

Imports `aleria_judge.lean_core` from the reference tree (torch and triton must import; nothing runs on a GPU),
drives its `Tree` through seeded random requests and the benchmark-shaped trees (`morj_b200.workloads`), and writes
`tests/golden/plans.json.gz`. The engine's planner (`morj_b200.tree.Tree`) must reproduce every record exactly.
"""
import gzip
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from plan_io import plan_record, random_case, simulate_passes, tree_record  # noqa: E402


def reference_lean_core(ref_root):
    sys.path.insert(0, ref_root)
    from aleria_judge import lean_core
    return lean_core


def record(tree_cls, case):
    try:
        tree, passes = simulate_passes(tree_cls, case['seqs'], case['passes'], case['window'], case['single_max'],
                                       case['step_tokens'], case['mode'], case.get('head', ()),
                                       case.get('bidir_pick', ()))
    except (ValueError, AssertionError) as error:
        return dict(error=type(error).__name__)
    return dict(tree=tree_record(tree), passes=passes)


def workload_cases():
    from morj_b200 import workloads as w
    out = []
    t = w.tiny_tree(0)
    out.append(dict(name='tiny', seqs=t['seqs'], passes=[list(range(4))], window=64, single_max=16384,
                    step_tokens=8192, mode='none'))
    t = w.text_tree(0)
    out.append(dict(name='text31b', seqs=t['seqs'], passes=[list(range(9))], window=1024, single_max=16384,
                    step_tokens=8192, mode='none'))
    # the same tree in multi-step passes (liveness allocator), two passes with pinned and whole retention
    out.append(dict(name='text31b-steps', seqs=t['seqs'], passes=[list(range(9))], window=1024, single_max=1000,
                    step_tokens=512, mode='none'))
    out.append(dict(name='text31b-pinned', seqs=t['seqs'], passes=[[0, 3, 6], [1, 2, 4, 5, 7, 8]], window=1024,
                    single_max=800, step_tokens=400, mode='pinned'))
    out.append(dict(name='text31b-identity', seqs=t['seqs'], passes=[[0, 1, 2], [3, 4, 5, 6, 7, 8]], window=1024,
                    single_max=16384, step_tokens=8192, mode='identity'))
    t = w.latency_tree(0)
    out.append(dict(name='latency', seqs=t['seqs'], passes=[list(range(8))], window=1024, single_max=16384,
                    step_tokens=8192, mode='none'))
    return out


def multimodal_cases(lean_core):
    """The multimodal tree goes through the reference `prepare` (placeholder expansion, node splits at image
    blocks, bidirectional image nodes), on CPU with a model object that skips the CUDA-only constructor."""
    import numpy as np
    from morj_b200 import workloads as w
    cfg = w.gemma31b_config()
    m = lean_core.LeanGemma4.__new__(lean_core.LeanGemma4)
    m.image_id, m.boi_id, m.eoi_id = cfg['image_token_id'], cfg['boi_token_id'], cfg['eoi_token_id']
    m.shared, m.shared_kv, m.device = None, None, 'cpu'
    m.free_bytes, m.kv_bytes, m.retain_budget, m.single_max, m.act_bytes = 1 << 50, 1, 1 << 50, 16384, 1
    out = []
    for name, kw, single_max, step in (('mm31b', {}, 16384, 8192), ('mm31b-steps', {}, 3000, 1024),
                                       ('mm-small', dict(hidden=8, blocks=3, soft=5, text=7, branch=4), 16384, 8192),
                                       ('mm-small-steps', dict(hidden=8, blocks=3, soft=5, text=7, branch=4), 9, 4)):
        t = w.multimodal_tree(0, **kw)
        req = m.prepare(t['seqs'], t['label_ids'], retain=False, images=t['images'])
        seqs = list(range(req.n_real))
        tree = req.tree
        need = tree.pass_nodes(seqs, set())
        plan = tree.plan_pass(need, seqs, 1024 if name.startswith('mm31b') else 3, single_max, step, False,
                              bidir=req.bidir)
        out.append(dict(name=name, kw=kw, single_max=single_max, step_tokens=step,
                        expanded=[list(map(int, s)) for s in tree.seqs], bidir=sorted(int(n) for n in req.bidir),
                        blob_start=np.asarray(req.blob_start).tolist(), blob_end=np.asarray(req.blob_end).tolist(),
                        blob_off=np.asarray(req.blob_off).tolist(), n_real=int(req.n_real),
                        tree=tree_record(tree), need=list(map(int, need)), plan=plan_record(plan)))
    return out


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else '/root/reference'
    lean_core = reference_lean_core(ref_root)
    rng = random.Random(20261201)
    cases = []
    for i in range(400):
        c = random_case(rng)
        c['name'] = f'random-{i}'
        cases.append(c)
    cases += workload_cases()
    for c in cases:
        c['expect'] = record(lean_core.Tree, c)
    mm = multimodal_cases(lean_core)
    path = os.path.join(HERE, 'plans.json.gz')
    with gzip.open(path, 'wt') as f:
        json.dump(dict(source='aleria_judge/lean_core.py Tree (reference planner)', cases=cases, multimodal=mm), f)
    print('wrote', path, os.path.getsize(path), 'bytes,', len(cases), 'cases +', len(mm), 'multimodal')


if __name__ == '__main__':
    main()
