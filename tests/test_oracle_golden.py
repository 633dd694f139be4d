"""Pin the CPU oracle before trusting it: against probabilities recorded from the reference's own lean path run on
the CPU (`tests/golden/make_forward_golden.py`), and against transformers' Gemma4ForCausalLM in FP32."""
import json
import os

import numpy as np
import pytest
import torch

from morj_b200 import workloads
from morj_b200.checkpoint import random_state
from morj_b200.lean_core import expand_images
from morj_b200.tree import Tree
from oracle.lean_oracle import OracleModel

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'forward_tiny.json')
with open(GOLDEN) as _f:
    DATA = json.load(_f)
CASES = {c['name']: c for c in DATA['cases']}


@pytest.fixture(scope='module')
def model():
    top = workloads.tiny_config()
    state = random_state(top, seed=0)
    checksum = float(sum(v.float().double().abs().sum().item() for v in state.values()))
    assert checksum == pytest.approx(DATA['weight_checksum'], rel=1e-12), 'seeded weights drifted'
    return OracleModel(top, state)


def flat(rows):
    return np.concatenate([np.asarray(r, dtype=np.float64) for r in rows])


@pytest.mark.parametrize('name', ['tiny', 'tiny-nested', 'tiny-steps'])
def test_bf16_tree_oracle_reproduces_reference_lean_path(model, name):
    c = CASES[name]
    got = model.forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16', c['single_max'], c['step_tokens'])
    ref = c['reference'][0]
    # same rounding points and the same CPU BF16 matmuls: only FP32 summation-order noise remains
    assert np.abs(flat(got) - flat(ref)).max() < 2e-3


def test_bf16_tree_oracle_with_image_blocks_reproduces_reference(model):
    from make_forward_golden import tiny_images
    c = CASES['tiny-images']
    images = tiny_images(model.top)
    got = model.forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16', images=images, expand=expand_images)
    assert np.abs(flat(got) - flat(c['reference'][0])).max() < 2e-3


@pytest.mark.parametrize('name', ['tiny', 'tiny-nested'])
def test_fp32_oracles_reproduce_transformers(model, name):
    c = CASES[name]
    tf = flat(c['transformers_fp32'])
    branches = flat(model.forward_branches(c['seqs'], c['label_ids'], 'fp32'))
    tree = flat(model.forward_tree(Tree, c['seqs'], c['label_ids'], 'fp32'))
    # transformers scales embeddings by the FP32 sqrt(hidden); the tiny config's sqrt(256) = 16 is exact in BF16
    assert np.abs(branches - tf).max() < 1e-4
    assert np.abs(tree - tf).max() < 1e-4


def test_reference_bf16_path_is_within_its_own_tolerance_of_fp32(model):
    # the reference BF16 lean path vs the FP32 model: the budget the B200 path is held to (1e-2) is of this order
    c = CASES['tiny']
    assert np.abs(flat(c['reference'][0]) - flat(c['transformers_fp32'])).max() < 1e-2


def test_planted_mistake_in_the_oracle_is_caught(model, monkeypatch):
    """A wrong rounding point planted in the oracle must move the probabilities past the parity budget."""
    import oracle.lean_oracle as lo
    c = CASES['tiny']
    real = lo.attn_epilogue

    def skip_post_norm(o, x, w_post, w_pre, eps, bf16=True):
        return real(o, x, torch.ones_like(w_post), w_pre, eps, bf16)
    monkeypatch.setattr(lo, 'attn_epilogue', skip_post_norm)
    got = flat(model.forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16'))
    assert np.abs(got - flat(c['reference'][0])).max() > 2e-3


def test_streamed_oracle_equals_the_resident_one(model):
    """The layer-streamed form (used at the 60-layer 31B width) computes exactly what the resident form does, and
    the dense attention's query blocking changes nothing."""
    import oracle.lean_oracle as lo
    c = CASES['tiny-nested']
    top = model.top
    state = random_state(top, seed=0)
    fetched = []

    def fetch(i):
        fetched.append(i)
        return lo.layer_from_state(lambda k: state[k], i, top['text_config']['layer_types'][i])
    streamed = OracleModel.streamed(top, model.embed, model.norm, fetch)
    want = flat(model.forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16'))
    assert np.array_equal(flat(streamed.forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16')), want)
    assert fetched == [0, 1]
    lo.QUERY_BLOCK, saved = 7, lo.QUERY_BLOCK
    try:
        blocked = flat(model.forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16'))
    finally:
        lo.QUERY_BLOCK = saved
    assert np.abs(blocked - want).max() < 1e-6
