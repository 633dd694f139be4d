"""The drop-in, exercised: the reference's own adapter `aleria_judge.lean_engine.LeanEngine` (unmodified, from the
offline install beside the repository) drives `morj_b200.lean_core.LeanGemma4` after the one-line swap of the model
class it imports (`lean_engine.py:20`). Everything above the model is the reference's code: the worker thread,
`score_request` / `_score_pass` (`lean_engine.py:52-149`) with gated `future` orders (a retained first pass, then a
second pass over the kept K/V), `release`, the evict-and-retry ladder on `MemoryError`, the shared head, and the
prompt / cached token statistics. Probabilities are compared with the reference lean path's recorded ones
(`tests/golden/forward_tiny.json`) within 1e-2 absolute; the statistics with the values the adapter's formula
(`lean_engine.py:139-149`) gives for the tree."""
import asyncio
import json
import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from morj_b200 import workloads
from morj_b200.checkpoint import random_state, write_checkpoint

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), 'baseline', '_ref')
TOL = 1e-2
PREFIX = 128  # the tiny tree: a 128-token prefix, then 24-token branches
with open(os.path.join(HERE, 'golden', 'forward_tiny.json')) as _f:
    CASES = {c['name']: c for c in json.load(_f)['cases']}


@pytest.fixture(scope='module')
def adapter(tmp_path_factory):
    """The reference's `lean_engine` module with its model class swapped for this engine's."""
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    if not os.path.isdir(os.path.join(REF, 'aleria_judge')):
        pytest.skip('the reference package is not installed under baseline/_ref')
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from aleria_judge import lean_engine
    from morj_b200.lean_core import LeanGemma4
    swapped = lean_engine.LeanGemma4
    lean_engine.LeanGemma4 = LeanGemma4  # the one-line swap of `lean_engine.py:20`
    path = tmp_path_factory.mktemp('tiny_ckpt')
    top = workloads.tiny_config()
    write_checkpoint(str(path), top, random_state(top, seed=0))
    yield lean_engine, str(path)
    lean_engine.LeanGemma4 = swapped


def branches(seqs, labels, which):
    """Judge's scoring branches (`question`, `kind`, `order` make the adapter's key) for sequences `which`."""
    return [SimpleNamespace(question=f'q{i}', kind='answer', order=(i,), input_ids=list(seqs[i]),
                            label_ids=tuple(labels[i])) for i in which]


def flat(rows):
    return np.concatenate([np.asarray(r, dtype=np.float64) for r in rows])


def test_gated_second_pass_reuses_the_first_pass_kv_through_the_reference_adapter(adapter):
    lean_engine, ckpt = adapter
    c = CASES['tiny-retain-two-pass']  # passes [0, 2] then [1, 3], retained
    seqs, labels = c['seqs'], c['label_ids']
    engine = lean_engine.LeanEngine(ckpt, retain_budget_gb=1.0)
    try:
        from morj_b200.lean_core import LeanGemma4
        assert isinstance(engine.model, LeanGemma4)
        first, second = branches(seqs, labels, c['passes'][0]), branches(seqs, labels, c['passes'][1])
        probs, stats = asyncio.run(engine.score_request(first, salt='s', future=second))
        assert np.abs(flat(probs) - flat(c['reference'][0])).max() <= TOL
        req, _ = engine.requests['s']
        assert req.retain and req.pools is not None
        assert stats['prompt_tokens'] == [len(seqs[i]) for i in c['passes'][0]]
        assert stats['cached_tokens'] == [0, PREFIX]
        assert engine.model.timing['tokens'] == req.tree.num_tokens - sum(len(seqs[i]) - PREFIX
                                                                          for i in c['passes'][1])
        probs2, stats2 = asyncio.run(engine.score_request(second, salt='s'))
        assert np.abs(flat(probs2) - flat(c['reference'][1])).max() <= TOL
        # the second pass computed only the gated orders' own tokens against the kept K/V
        assert engine.model.timing['tokens'] == sum(len(seqs[i]) - PREFIX for i in c['passes'][1])
        assert stats2['cached_tokens'] == [PREFIX, PREFIX]
        assert engine._kept_bytes(exclude=None) == req.tree.num_tokens * engine.model.kv_bytes
        engine.release('s')
        assert 's' not in engine.requests and engine._kept_bytes(exclude=None) == 0
    finally:
        engine.close()


def test_memory_error_evicts_other_requests_and_retries_through_the_reference_adapter(adapter):
    lean_engine, ckpt = adapter
    c = CASES['tiny']
    seqs, labels = c['seqs'], c['label_ids']
    engine = lean_engine.LeanEngine(ckpt, retain_budget_gb=1.0)
    try:
        m = engine.model
        need = (PREFIX + 2 * 24) * m.act_bytes  # one step's activations: what the planner checks for a one-step pass
        # another request holds K/V; with it kept the pass does not fit, without it it does
        kept = torch.empty(need // 2, dtype=torch.uint8)
        engine.requests['other'] = (SimpleNamespace(pools=[(kept, kept[:0])]), {})
        m.free_bytes = need + need // 4
        probs, stats = asyncio.run(engine.score_request(branches(seqs, labels, [0, 1]), salt='s'))
        assert 'other' not in engine.requests  # evicted by the ladder's second attempt
        assert np.abs(flat(probs) - flat(c['reference'][0][:2])).max() <= TOL
        assert stats['cached_tokens'] == [0, PREFIX]
        # a pass too large on its own is the request's MemoryError (the service's 413)
        m.free_bytes = need // 2
        with pytest.raises(MemoryError):
            asyncio.run(engine.score_request(branches(seqs, labels, [0, 1]), salt='t'))
        assert not engine.requests
    finally:
        engine.close()


def test_shared_head_through_the_reference_adapter(adapter):
    lean_engine, ckpt = adapter
    c = CASES['tiny']
    seqs, labels = c['seqs'], c['label_ids']
    engine = lean_engine.LeanEngine(ckpt, shared_prefix=seqs[0][:40], retain_budget_gb=1.0)
    try:
        probs, stats = asyncio.run(engine.score_request(branches(seqs, labels, [0, 1, 2, 3]), salt='s'))
        assert np.abs(flat(probs) - flat(c['reference'][0])).max() <= TOL
        # the head's 40 tokens were copied, not computed: the first branch counts them as cached
        assert stats['cached_tokens'] == [40, PREFIX, PREFIX, PREFIX]
        assert engine.model.timing['tokens'] == PREFIX - 40 + 4 * 24
    finally:
        engine.close()
