"""The whole engine on the GPU against the reference lean path: label probabilities within 1e-2 absolute of the
probabilities recorded from the reference's own `LeanGemma4` (`tests/golden/forward_tiny.json`) and of the CPU
oracle, on the tiny seeded model; one-step, multi-step, two-pass retained, two-pass pinned, nested-branch and
image-block requests; the shared head, poison mode and the checkpoint loader."""
import json
import os

import numpy as np
import pytest
import torch

from morj_b200 import workloads
from morj_b200.checkpoint import random_state, write_checkpoint

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'forward_tiny.json')
with open(GOLDEN) as _f:
    DATA = json.load(_f)
CASES = {c['name']: c for c in DATA['cases']}
TOL = 1e-2


@pytest.fixture(scope='module')
def state():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    top = workloads.tiny_config()
    return top, random_state(top, seed=0)


def engine(state, **kw):
    from morj_b200.lean_core import LeanGemma4
    top, st = state
    budget = kw.pop('retain_budget', None)
    m = LeanGemma4.from_state(top, st, device='cuda', **kw)
    if budget is not None:
        m.retain_budget = budget
    return m


def flat(rows):
    return np.concatenate([np.asarray(r, dtype=np.float64) for r in rows])


def check_contract(probs, labels):
    """The method.py contract: one row per sequence, its labels' length, finite, in [0, 1], summing to 1."""
    assert len(probs) == len(labels)
    for p, ids in zip(probs, labels):
        assert isinstance(p, list) and len(p) == len(ids)
        assert all(np.isfinite(p)) and min(p) >= 0 and max(p) <= 1 and abs(sum(p) - 1) <= 1e-3


@pytest.mark.parametrize('name', ['tiny', 'tiny-steps', 'tiny-nested', 'tiny-retain-two-pass',
                                  'tiny-pinned-two-pass', 'tiny-images', 'tiny-images-steps'])
def test_engine_matches_reference_lean_path(state, name):
    c = CASES[name]
    m = engine(state, single_max=c['single_max'], step_tokens=c['step_tokens'], retain_budget=c['retain_budget'])
    images = None
    if c['images']:
        from make_forward_golden import tiny_images
        images = [f.cuda() for f in tiny_images(state[0])]
    req = m.prepare(c['seqs'], c['label_ids'], retain=c['retain'], images=images)
    assert (req.retain, req.pinned) == (c['retained'], c['pinned'])
    for p, ref in zip(c['passes'], c['reference']):
        got = m.run(req, list(p))
        check_contract(got, [c['label_ids'][b] for b in p])
        err = np.abs(flat(got) - flat(ref)).max()
        assert err <= TOL, (name, err)
    if len(c['passes']) > 1:
        # the second pass computed fewer tokens than the whole tree: the first pass's K/V were kept
        assert m.timing['tokens'] < req.tree.num_tokens


def test_engine_matches_oracle_and_transformers(state):
    from morj_b200.tree import Tree
    from oracle.lean_oracle import OracleModel
    c = CASES['tiny-nested']
    m = engine(state)
    got = flat(m.forward_tree(Tree(c['seqs']), c['label_ids']))
    oracle = flat(OracleModel(*state).forward_tree(Tree, c['seqs'], c['label_ids'], 'bf16'))
    assert np.abs(got - oracle).max() <= TOL
    assert np.abs(got - flat(c['transformers_fp32'])).max() <= 2 * TOL


def test_shared_head_is_reused_not_recomputed(state):
    c = CASES['tiny']
    head = c['seqs'][0][:40]
    m = engine(state)
    m.set_shared_prefix(head)
    req = m.prepare(c['seqs'], c['label_ids'])
    assert req.head_nodes
    got = m.run(req, [0, 1, 2, 3])
    head_tokens = sum(req.tree.nodes[n][2] - req.tree.nodes[n][1] for n in req.head_nodes)
    assert head_tokens == 40 and not set(req.head_nodes) & set(m.last_need)
    assert np.abs(flat(got) - flat(c['reference'][0])).max() <= TOL


def test_poisoned_pools_read_no_unwritten_slot(state, monkeypatch):
    """Every K/V pool starts as NaN: any read of a slot no pass wrote would turn the probabilities into NaN."""
    import morj_b200.lean_core as lc
    monkeypatch.setattr(lc, 'POISON', True)
    for name in ('tiny-steps', 'tiny-pinned-two-pass', 'tiny-images-steps'):
        c = CASES[name]
        m = engine(state, single_max=c['single_max'], step_tokens=c['step_tokens'], retain_budget=c['retain_budget'])
        images = None
        if c['images']:
            from make_forward_golden import tiny_images
            images = [f.cuda() for f in tiny_images(state[0])]
        req = m.prepare(c['seqs'], c['label_ids'], retain=c['retain'], images=images)
        for p, ref in zip(c['passes'], c['reference']):
            got = m.run(req, list(p))
            assert np.isfinite(flat(got)).all(), name
            assert np.abs(flat(got) - flat(ref)).max() <= TOL


def test_checkpoint_directory_loads_like_the_reference(state, tmp_path):
    from morj_b200.lean_core import LeanGemma4
    top, st = state
    write_checkpoint(str(tmp_path), top, st)
    m = LeanGemma4(str(tmp_path), device='cuda')
    c = CASES['tiny']
    req = m.prepare(c['seqs'], c['label_ids'])
    got = m.run(req, [0, 1, 2, 3])
    assert np.abs(flat(got) - flat(c['reference'][0])).max() <= TOL
    assert m.timing['steps'] == 1 and m.timing['tokens'] == req.tree.num_tokens and m.gpu_ms > 0


def test_a_pass_too_large_for_the_budget_raises_memory_error(state):
    m = engine(state)
    c = CASES['tiny']
    req = m.prepare(c['seqs'], c['label_ids'])
    with pytest.raises(MemoryError):
        m.run(req, [0, 1, 2, 3], available=1)


def full_width_model(vocab=4096):
    """The 31B-class layer dimensions (hidden 5376, 32 / 16 heads of 128, GeGLU 21504, window 1024) with two layers
    (one sliding, one global) and a small vocabulary: full-size kernels, an oracle run of seconds."""
    top = workloads.gemma31b_config()
    cfg = dict(top['text_config'], layer_types=['sliding_attention', 'full_attention'], num_hidden_layers=2,
               vocab_size=vocab)
    top = dict(top, text_config=cfg, image_token_id=vocab - 1, boi_token_id=vocab - 2, eoi_token_id=vocab - 3)
    state = {k: v.cpu() for k, v in random_state(top, seed=11, device='cuda').items()}
    return top, state


@pytest.mark.parametrize('kind', ['text', 'images'])
def test_full_width_layers_match_oracle(kind):
    """Parity at the 31B layer width on the text-tree shape (1500-token prefix, 9 branches of 60), and with two image
    blocks (560 soft tokens, and 1100 > the 1024 window: the explicit-mask path) in the shared prefix."""
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from morj_b200.lean_core import LeanGemma4, expand_images
    from morj_b200.tree import Tree
    from oracle.lean_oracle import OracleModel
    top, state = full_width_model()
    images = None
    if kind == 'text':
        t = workloads.text_tree(3, vocab=4096)
        seqs, labels = t['seqs'], t['label_ids']
    else:
        rng = np.random.default_rng(4)
        img = top['image_token_id']
        head = [int(v) for v in rng.integers(0, 4000, 20)] + [img] + [int(v) for v in rng.integers(0, 4000, 30)] + [img]
        seqs = [head + [int(v) for v in rng.integers(0, 4000, n)] for n in (40, 25, 60)]
        labels = [[5, 6, 7], [5, 6, 7], list(range(100, 355))]
        g = torch.Generator().manual_seed(5)
        images = [(torch.randn(n, 5376, generator=g) / 5376 ** 0.5).to(torch.bfloat16) for n in (560, 1100)]
    m = LeanGemma4.from_state(top, state, device='cuda')
    req = m.prepare(seqs, labels, images=[f.cuda() for f in images] if images else None)
    got = flat(m.run(req, list(range(len(seqs)))))
    oracle = flat(OracleModel(top, state).forward_tree(Tree, seqs, labels, 'bf16', images=images,
                                                       expand=expand_images))
    assert np.abs(got - oracle).max() <= TOL, np.abs(got - oracle).max()
