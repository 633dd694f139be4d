"""`bench.py`'s contract on the CPU: both arms describe a run with the same `config`, the reference arm's FLOP count
comes from the reference planner's plan and equals the engine planner's, and without the reference installed the
reference arm prints an `unavailable` line and exits cleanly."""
import argparse
import io
import json
import os
import sys
from contextlib import redirect_stdout

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def args(**kw):
    base = dict(gpus=1, steps=2, warmup=1, impl='reference', workload='text', layers=0, tp_comm='peer',
                mode='replicas')
    base.update(kw)
    return argparse.Namespace(**base)


@pytest.mark.parametrize('world,mode', [(1, 'replicas'), (4, 'replicas'), (2, 'tp')])
def test_both_arms_build_the_same_config(world, mode):
    a = args(mode=mode)
    desc = bench.workload('text', 0)[1]
    cfg = bench.bench_config(a, world, desc, 2040, 102.23e12)  # (the one builder both arms call)
    assert cfg['tokens'] == 2040 and cfg['tflops_per_tree_specified'] == 102.23
    assert ('tensor parallel' in cfg['parallelism']) == (mode == 'tp' and world > 1)


def test_tree_flops_of_the_engine_plan_is_the_specified_workload():
    from morj_b200 import workloads as w
    from morj_b200.tree import Tree
    top = w.gemma31b_config()
    t = w.text_tree(0)
    tree = Tree(t['seqs'])
    seqs = list(range(len(t['seqs'])))
    plan = tree.plan_pass(tree.pass_nodes(seqs, set()), seqs, 1024, 16384, 8192, False)
    flops = bench.tree_flops(top, plan, tree.num_tokens)
    assert abs(flops / 1e12 - 102.2) < 0.1  # 100.62 TF linear + 1.60 TF attention


def test_reference_arm_without_the_reference_prints_unavailable(monkeypatch, tmp_path):
    import oracle.ref_cpu as rc
    monkeypatch.setattr(rc, 'INSTALL', str(tmp_path / 'nothing'))
    out = io.StringIO()
    with redirect_stdout(out):
        bench.reference_arm(args(), 0, 1)
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    assert line['impl'] == 'reference' and 'unavailable' in line


def test_reference_arm_prints_nothing_on_other_ranks():
    out = io.StringIO()
    with redirect_stdout(out):
        bench.reference_arm(args(gpus=2), 1, 2)
    assert out.getvalue() == ''
