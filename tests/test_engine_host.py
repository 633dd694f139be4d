"""Host-side engine behaviour that needs no GPU: the planner's memory-fit loop ends in MemoryError rather than
looping (reference `tests/test_lean.py:218-239`), the retention decision and image-block layout of `prepare`, the
GeGLU weight interleave, and the engine's native path failing loudly when the library is absent."""
import threading

import numpy as np
import pytest
import torch

from morj_b200 import lean_core
from morj_b200.lean_core import LeanGemma4, Request, interleave_glu
from morj_b200.tree import Tree


def bare_model(**kw):
    m = LeanGemma4.__new__(LeanGemma4)
    m.free_bytes, m.step_tokens, m.single_max, m.act_bytes, m.window = 2**34, 8192, 16384, 10**6, 1024
    m.geom = {'sliding_attention': (8, 256), 'full_attention': (4, 512)}
    m.types = ['sliding_attention', 'full_attention']
    m.kv_bytes = sum(2 * 2 * m.geom[k][0] * m.geom[k][1] for k in m.types)
    m.retain_budget = 10 * 2**30
    m.shared = None
    for k, v in kw.items():
        setattr(m, k, v)
    return m


def test_a_pass_that_does_not_fit_raises_instead_of_looping():
    model = bare_model()
    req = Request(Tree([list(range(1, 400))]), [[0]], False, [])
    outcome = []

    def run():
        try:
            model.plan(req, [0], available=1)
        except MemoryError as error:
            outcome.append(error)
    worker = threading.Thread(target=run, daemon=True)
    worker.start()
    worker.join(30)
    assert not worker.is_alive(), 'the planner loops forever'
    assert outcome and isinstance(outcome[0], MemoryError)


def test_a_large_pass_is_cut_into_steps_to_fit():
    """One step's activations do not fit: the planner drops `single_max`, then halves the step until the live pools
    plus one step's activations fit (reference `lean_core.py:509-529`)."""
    model = bare_model(act_bytes=20000, window=256)
    model.geom = {'sliding_attention': (8, 256), 'full_attention': (1, 64)}
    req = Request(Tree([list(range(1, 3000))]), [[0]], False, [])
    need, head, pinned, plan = model.plan(req, [0], available=20_000_000)
    per_token = {'s': 4 * 8 * 256, 'g': 4 * 64}
    largest = max(len(st['tokens']) for st in plan['steps'])
    assert len(plan['steps']) > 1 and largest <= 512
    assert sum(plan['cap'][k] * per_token[k] for k in 'gs') + largest * 20000 <= 20_000_000
    assert plan['cap']['s'] < 3000  # sliding slots are freed as the pass moves on


def test_prepare_retains_only_within_budget():
    model = bare_model()
    model.device = torch.device('cpu')
    seqs = [list(range(1, 50)) + [7], list(range(1, 50)) + [8]]
    req = model.prepare(seqs, [[1, 2], [1, 2]], retain=False)
    assert not req.retain and not req.pinned and req.pools is None
    model.retain_budget = 10
    req = model.prepare(seqs, [[1, 2], [1, 2]], retain=True)
    assert not req.retain and req.pinned


def test_glu_interleave_puts_gate_and_up_blocks_side_by_side():
    F, H = 256, 8
    gate = torch.arange(F * H).reshape(F, H).float()
    up = -gate
    w = interleave_glu(gate, up)
    assert torch.equal(w[0:128], gate[0:128]) and torch.equal(w[128:256], up[0:128])
    assert torch.equal(w[256:384], gate[128:256]) and torch.equal(w[384:512], up[128:256])


def test_native_path_fails_loudly_without_the_library(monkeypatch, tmp_path):
    from morj_b200 import _native
    monkeypatch.setattr(_native, '_lib', None)
    monkeypatch.setattr(_native, 'LIB_PATH', str(tmp_path / 'missing.so'))
    with pytest.raises(ImportError, match='not built'):
        _native.lib()
