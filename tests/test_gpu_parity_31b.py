"""Parity at the configuration the headline is quoted on: the whole 60-layer 31B-class model (hidden 5376, 32 / 16
heads of 128, GeGLU 21504, vocabulary 262144, 5 sliding-1024 : 1 global layers) on the GPU against the CPU oracle
run layer by layer on the engine's own weights (copied to the host one layer at a time).

* the bench's text tree (1500-token prefix, 3 questions x 3 rotations x 60 tokens, 5 labels per question), 60 layers;
* the multimodal tree (8 image blocks of 560 soft tokens + 300 text tokens, 2 questions x 4 rotations x 40 tokens, a
  255-label and a 2-label question), 60 layers;
* the latency tree (8192-token prefix, 8 branches of 64) over the first 6 layers (one full 5 : 1 layer pattern).

Bar: per-question option probabilities within 1e-2 absolute of the oracle (the reference's BF16 lean path,
`aleria_judge/lean_core.py:599-737`, readout `558-561`). The measured error is printed with `-s`.
"""
import json
import os

import numpy as np
import pytest
import torch

from morj_b200 import workloads

pytestmark = pytest.mark.gpu

TOL = 1e-2
HERE = os.path.dirname(os.path.abspath(__file__))


def flat(rows):
    return np.concatenate([np.asarray(r, dtype=np.float64) for r in rows])


@pytest.fixture(scope='module')
def model():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    torch.set_num_threads(os.cpu_count())
    from morj_b200.lean_core import LeanGemma4
    m = LeanGemma4.random_init(workloads.gemma31b_config(), seed=0, device='cuda')
    yield m
    del m
    torch.cuda.empty_cache()


def run_engine(m, tree_in):
    images = [f.cuda() for f in tree_in['images']] if tree_in['images'] else None
    req = m.prepare(tree_in['seqs'], tree_in['label_ids'], images=images)
    return m.run(req, list(range(len(tree_in['seqs']))))


def oracle_on(m, top, tree_in):
    from make_oracle_31b import engine_fetch, oracle_probs
    from morj_b200.lean_core import expand_images
    from oracle.lean_oracle import OracleModel
    embed, norm, fetch = engine_fetch(m)
    return oracle_probs(OracleModel.streamed(top, embed, norm, fetch), tree_in, expand=expand_images)


def test_text_tree_60_layers_matches_oracle(model):
    top = workloads.gemma31b_config()
    tree_in = workloads.text_tree(seed=0)
    got = flat(run_engine(model, tree_in))
    ref = flat(oracle_on(model, top, tree_in))
    err = np.abs(got - ref).max()
    print(f'\n31B text tree, 60 layers: max |engine - oracle| = {err:.3e} over {len(got)} probabilities')
    assert err <= TOL, err
    # the record bench.py compares its own tree against is this oracle on these weights
    with open(os.path.join(HERE, 'golden', 'oracle_31b_text.json')) as f:
        stored = flat(json.load(f)['probs'])
    assert np.abs(stored - ref).max() <= 1e-6


def test_multimodal_tree_60_layers_matches_oracle(model):
    top = workloads.gemma31b_config()
    tree_in = workloads.multimodal_tree(seed=0)
    got_rows = run_engine(model, tree_in)
    ref_rows = oracle_on(model, top, tree_in)
    assert [len(r) for r in got_rows] == [255] * 4 + [2] * 4
    got, ref = flat(got_rows), flat(ref_rows)
    err = np.abs(got - ref).max()
    print(f'\n31B multimodal tree, 60 layers: max |engine - oracle| = {err:.3e} over {len(got)} probabilities')
    assert err <= TOL, err


def test_latency_tree_one_layer_pattern_matches_oracle(model):
    """8,704 tokens through the first 6 layers (5 sliding + 1 global) of the same weights."""
    from morj_b200.lean_core import LeanGemma4
    top = workloads.reduced_config(workloads.gemma31b_config(), 6)
    m6 = LeanGemma4.random_init(top, seed=0, device='cuda')  # checkpoint order: the full model's first 6 layers
    try:
        assert torch.equal(m6.layers[5]['down'], model.layers[5]['down'])
        tree_in = workloads.latency_tree(seed=0)
        got = flat(run_engine(m6, tree_in))
        ref = flat(oracle_on(m6, top, tree_in))
    finally:
        del m6
        torch.cuda.empty_cache()
    err = np.abs(got - ref).max()
    print(f'\n31B latency tree, 6 layers: max |engine - oracle| = {err:.3e} over {len(got)} probabilities')
    assert err <= TOL, err
