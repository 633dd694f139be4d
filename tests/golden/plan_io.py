"""Serialisation and pass bookkeeping shared by the planner fixture generator and the planner tests.

`simulate_passes` drives a `Tree` class through a request's passes the way the engine's `run` does
(reference `aleria_judge/lean_core.py:495-576`: cached nodes, pinned offsets for later passes, slot tables carried
between passes) and records every planner output in plain lists, so two implementations can be compared exactly.
"""
import numpy as np


def _l(a):
    return np.asarray(a).astype(np.int64).tolist()


def tree_record(tree):
    return dict(nodes=[list(map(int, n)) for n in tree.nodes], paths=[list(map(int, p)) for p in tree.paths],
                offsets=_l(tree.offsets), num_tokens=int(tree.num_tokens), prompt_tokens=int(tree.prompt_tokens),
                node_path=sorted([int(k), list(map(int, v))] for k, v in tree.node_path.items()),
                readout=[list(tree.readout_slot(b)) if len(tree.seqs[b]) else None for b in range(len(tree.seqs))])


def plan_record(plan):
    steps = []
    for st in plan['steps']:
        d = dict(segs=[list(map(int, s)) for s in st['segs']], own=_l(st['own']), positions=_l(st['positions']),
                 tokens=_l(st['tokens']), n_bidir=int(st['n_bidir']), qo_indptr=_l(st['qo_indptr']))
        for k in 'gs':
            d['slots_' + k] = _l(st['slots'][k])
            d['kv_indptr_' + k] = _l(st['kv_indptr_' + k])
            d['kv_indices_' + k] = _l(st['kv_indices_' + k])
        steps.append(d)
    return dict(steps=steps, cap={k: int(v) for k, v in plan['cap'].items()},
                slot_of={k: _l(v) for k, v in plan['slot_of'].items()},
                readout=[list(map(int, r)) for r in plan['readout']])


def simulate_passes(tree_cls, seqs, passes, window, single_max, step_tokens, mode, head=(), bidir_pick=()):
    """Plan every pass of a request over `seqs` (+ an optional shared `head` sequence) in retention `mode`
    ('none', 'identity' or 'pinned'); returns the tree and per-pass records."""
    tree = tree_cls(list(seqs) + ([list(head)] if len(head) else []))
    head_nodes = tree.paths[-1] if len(head) else []
    head_off = np.concatenate([tree.slots(n) for n in head_nodes]) if len(head) else np.zeros(0, np.int64)
    bidir = frozenset(int(tree.paths[0][i]) for i in bidir_pick if i < len(tree.paths[0])) if len(seqs) else frozenset()
    computed, read, tables = set(head_nodes), set(), None
    identity = mode == 'identity'
    out = []
    for pas in passes:
        if not pas:
            continue
        cached = computed if mode != 'none' else set(head_nodes)
        need = tree.pass_nodes(pas, cached)
        pinned = None
        if mode == 'pinned':
            future = [b for b in range(len(tree.seqs)) if b not in read and b not in set(pas)]
            pinned = tree.pinned_for(cached | set(need), future, window)
        plan = tree.plan_pass(need, pas, window, single_max, step_tokens, identity,
                              prealloc=() if identity else head_off, initial=tables, pinned=pinned, bidir=bidir)
        rec = dict(pas=list(pas), need=list(map(int, need)), plan=plan_record(plan),
                   pinned=None if pinned is None else {k: _l(v) for k, v in pinned.items()})
        out.append(rec)
        read |= set(pas)
        if mode != 'none':
            computed |= set(need)
        if mode == 'pinned':
            tables = {}
            for kk in 'gs':
                t = np.full(tree.num_tokens, -1)
                t[pinned[kk]] = plan['slot_of'][kk][pinned[kk]]
                tables[kk] = t
    return tree, out


def random_case(rng):
    """A seeded random request: sequences over a small alphabet sharing prefixes, passes, window, step sizes and
    retention mode (in the spirit of the reference's planner property test, `tests/lean_tree_check.py:108-126`)."""
    trunk = [rng.randint(0, 4) for _ in range(rng.randint(1, 26))]
    seqs = []
    for _ in range(rng.randint(1, 7)):
        cut = rng.randint(0, len(trunk))
        seqs.append(trunk[:cut] + [rng.randint(0, 3) for _ in range(rng.randint(0 if cut else 1, 10))])
        if rng.random() < .35:
            trunk = seqs[-1]
    head = []
    if rng.random() < .4:
        head = [7, 7, 6]
        seqs = [head + s for s in seqs]
    n = len(seqs)
    order = rng.sample(range(n), n)
    split = rng.randint(1, n)
    passes = [list(range(n))] if rng.random() < .4 else [order[:split], order[split:]]
    kw = dict(window=rng.choice([1, 2, 3, 5, 10**9]), single_max=rng.choice([2, 5, 9, 10**9]),
              step_tokens=rng.choice([1, 2, 4, 6]), mode=rng.choice(['none', 'identity', 'pinned']))
    bidir_pick = tuple(sorted(rng.sample(range(4), rng.randint(0, 2)))) if rng.random() < .3 else ()
    return dict(seqs=seqs, passes=passes, head=head, bidir_pick=list(bidir_pick), **kw)
