"""Token-tree layout and pass planner for the tree-prefill engine (host side, numpy).

A request's sequences (branches) share prefixes. The tree stores every distinct prefix token once: node `i` covers
depths `[start, end)` of the sequence that first produced them, and owns the tree offsets
`offsets[i]:offsets[i + 1]`. Nodes are ordered by start depth (ties by creation order), so a parent always precedes
its children. A pass plan cuts the nodes to compute into steps and gives, per step and per attention kind
('g' = full attention, 's' = sliding window):

* `slots[kind]`    pool slot of each token computed in the step (K/V are written there),
* `kv_indptr_<k>`, `kv_indices_<k>`   CSR lists: segment `s` attends over the pool slots
  `kv_indices[kv_indptr[s]:kv_indptr[s + 1]]` (page size 1), which are its path's tokens in depth order (only the
  last `window` before the segment's first query for sliding layers), bottom-right aligned with its queries.

The plan is bit-exact with the reference planner (`aleria_judge/lean_core.py:34-231`, `Tree`): the same node ids,
offsets, step cuts, readout rows and slot numbers, because the K/V pools and tree tables it produces are the
contract the kernels and the request-level retention modes read. The code here is an independent implementation
of those published rules; `tests/test_tree_golden.py` compares it with fixtures recorded from the reference.
"""
from __future__ import annotations

import numpy as np

KINDS = ('g', 's')


def _common_prefix(a: np.ndarray, b: np.ndarray) -> int:
    """Length of the longest common prefix of two int64 arrays."""
    n = min(len(a), len(b))
    if n == 0:
        return 0
    neq = a[:n] != b[:n]
    k = int(np.argmax(neq))
    return n if not neq[k] else k


class Tree:
    """Radix layout of token sequences (reference: `lean_core.py:34-83`).

    Attributes (names and types as in the reference, since the engine adapter reads them):
    `seqs` (list of int64 arrays), `nodes` (list of `[owner sequence, start depth, end depth]`), `paths` (per
    sequence, node ids from the root), `offsets` (int64 prefix sums of node lengths), `num_tokens`,
    `prompt_tokens`, `node_path` (node id -> node ids from the root to it, inclusive).
    """

    def __init__(self, seqs):
        self.seqs = [np.asarray(s, dtype=np.int64) for s in seqs]
        raw: list[list[int]] = []        # creation order: [owner, start, end]
        members: list[list[int]] = []    # per sequence: creation ids from the root
        for b, seq in enumerate(self.seqs):
            # the earlier sequence sharing the longest prefix (first one on ties) and that length
            donor, shared = -1, 0
            for j in range(b):
                c = _common_prefix(seq, self.seqs[j])
                if c > shared:
                    donor, shared = j, c
            route: list[int] = []
            if donor >= 0:
                for nid in list(members[donor]):
                    owner, start, end = raw[nid]
                    if end <= shared:
                        route.append(nid)
                        continue
                    if start < shared:
                        # the branch point falls inside this node: keep [start, shared) here and move the rest to a
                        # new node, which follows it on every path through it
                        raw.append([owner, shared, end])
                        tail = len(raw) - 1
                        raw[nid][2] = shared
                        for m in members:
                            if nid in m:
                                m.insert(m.index(nid) + 1, tail)
                        route.append(nid)
                    break
            if shared < len(seq):
                raw.append([b, shared, len(seq)])
                route.append(len(raw) - 1)
            members.append(route)
        order = sorted(range(len(raw)), key=lambda i: (raw[i][1], i))
        new_id = np.empty(len(raw), dtype=np.int64)
        new_id[np.asarray(order, dtype=np.int64)] = np.arange(len(raw))
        self.nodes = [raw[i] for i in order]
        self.paths = [[int(new_id[n]) for n in m] for m in members]
        lengths = [e - s for _, s, e in self.nodes]
        self.offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
        self.num_tokens = int(self.offsets[-1])
        self.prompt_tokens = sum(len(s) for s in self.seqs)
        self.node_path = {}
        for p in self.paths:
            for i, nid in enumerate(p):
                if nid not in self.node_path:
                    self.node_path[nid] = p[:i + 1]

    # ---- lookups --------------------------------------------------------------------------------------------------
    def slots(self, nid):
        """Tree offsets of node `nid` (reference `lean_core.py:85-86`)."""
        return np.arange(self.offsets[nid], self.offsets[nid + 1])

    def span(self, nid):
        return self.nodes[nid][2] - self.nodes[nid][1]

    def readout_slot(self, b):
        """(node, tree offset) of sequence `b`'s last token (reference `lean_core.py:88-94`)."""
        last = len(self.seqs[b]) - 1
        for nid in self.paths[b]:
            _, s, e = self.nodes[nid]
            if s <= last < e:
                return nid, int(self.offsets[nid] + last - s)
        raise ValueError('empty sequence')

    def pass_nodes(self, seqs, cached):
        """Nodes a pass over `seqs` computes: uncached path nodes plus every readout node, whose hidden state is not
        kept and is computed again (reference `lean_core.py:96-101`)."""
        need = set()
        for b in seqs:
            need.update(self.paths[b])
        need.difference_update(cached)
        for b in seqs:
            need.add(self.readout_slot(b)[0])
        return sorted(need)

    def pinned_for(self, done, future, window):
        """Offsets a later pass over `future` reads once this pass has computed `done`: per future path, every token
        before its first node that is not done (or its readout node, always recomputed); all of them for full layers
        ('g'), the last `window` before that point for sliding layers ('s') (reference `lean_core.py:103-118`)."""
        keep = {'g': [], 's': []}
        for f in future:
            path = self.paths[f]
            ro = self.readout_slot(f)[0]
            j = len(path)
            for i, n in enumerate(path):
                if n not in done or n == ro:
                    j = i
                    break
            if j == 0:
                continue
            before = np.concatenate([self.slots(n) for n in path[:j]])
            d0 = self.nodes[path[j]][1] if j < len(path) else self.nodes[path[-1]][2]
            keep['g'].append(before)
            keep['s'].append(before[max(0, d0 - window + 1):])
        return {k: (np.unique(np.concatenate(v)) if v else np.zeros(0, np.int64)) for k, v in keep.items()}

    # ---- planning -------------------------------------------------------------------------------------------------
    def _depth_first(self, compute):
        """`compute` in depth-first pre-order over the sub-forest it spans, children in ascending id order."""
        todo = set(compute)
        kids: dict[int, list[int]] = {}
        for n in compute:
            np_ = self.node_path[n]
            parent = np_[-2] if len(np_) > 1 else -1
            kids.setdefault(parent if parent in todo else -1, []).append(n)
        out, stack = [], sorted(kids.get(-1, []), reverse=True)
        while stack:
            n = stack.pop()
            out.append(n)
            stack.extend(sorted(kids.get(n, []), reverse=True))
        return out

    def _cut(self, compute, budget, bidir):
        """Cut the node list into steps of at most `budget` tokens; image blocks (`bidir`) are never split."""
        steps, cur, room = [], [], budget
        for n in compute:
            a, end = self.nodes[n][1], self.nodes[n][2]
            whole = n in bidir
            if whole and end - a > room and cur:
                steps.append(cur)
                cur, room = [], budget
            while a < end:
                take = end - a if whole else min(end - a, room)
                cur.append((n, a, a + take))
                a += take
                room -= take
                if room <= 0:
                    steps.append(cur)
                    cur, room = [], budget
        if cur:
            steps.append(cur)
        # image blocks lead their step: their queries attend without the causal mask in sliding layers
        return [[s for s in st if s[0] in bidir] + [s for s in st if s[0] not in bidir] for st in steps]

    def plan_pass(self, compute, readout_seqs, window, single_max, step_tokens, identity, prealloc=(), initial=None,
                  pinned=None, bidir=frozenset()):
        """Plan one pass over the nodes `compute` (reference `lean_core.py:120-231`; same arguments and result).

        Returns `dict(steps=[...], cap={kind: slots}, slot_of={kind: offset -> slot}, readout=[(step, row)])`; each
        step is a dict with `segs, own, positions, tokens, n_bidir, qo_indptr, slots, kv_indptr_g, kv_indices_g,
        kv_indptr_s, kv_indices_s`."""
        compute = list(compute)
        total = sum(self.span(n) for n in compute)
        if total > single_max:
            budget = step_tokens
            compute = self._depth_first(compute)
        else:
            budget = total
        cuts = self._cut(compute, budget, bidir)

        # readout rows: tree offset -> indices into readout_seqs
        want: dict[int, list[int]] = {}
        for i, b in enumerate(readout_seqs):
            want.setdefault(self.readout_slot(b)[1], []).append(i)
        readout = [None] * len(readout_seqs)

        last_read = {k: np.full(self.num_tokens, -1) for k in KINDS}
        steps = []
        for k, segs in enumerate(cuts):
            own, pos, toks, lists = [], [], [], {'g': [], 's': []}
            for n, a, b in segs:
                owner, sn, _ = self.nodes[n]
                base = self.offsets[n]
                ancestors = [self.slots(p) for p in self.node_path[n][:-1]]
                path = np.concatenate(ancestors + [base + np.arange(0, b - sn)])
                lists['g'].append(path)
                lists['s'].append(path[max(0, a - window + 1):])
                for kind in KINDS:
                    last_read[kind][lists[kind][-1]] = k
                own.append(base + np.arange(a - sn, b - sn))
                pos.append(np.arange(a, b))
                toks.append(self.seqs[owner][a:b])
            own = np.concatenate(own)
            hits = np.flatnonzero(np.isin(own, list(want)))
            for r in hits:
                for i in want[int(own[r])]:
                    readout[i] = (k, int(r))
            steps.append(dict(segs=segs, own=own, kv=lists, positions=np.concatenate(pos),
                              tokens=np.concatenate(toks), n_bidir=sum(1 for s in segs if s[0] in bidir),
                              qo_indptr=np.concatenate([[0], np.cumsum([b - a for _, a, b in segs])])))
        if any(r is None for r in readout):
            raise ValueError('a readout token is not computed in this pass')

        slot_of, cap = {}, {}
        for kind in KINDS:
            if identity:
                slot_of[kind], cap[kind] = np.arange(self.num_tokens), self.num_tokens
                continue
            slot_of[kind], cap[kind] = self._allocate(kind, steps, last_read[kind], prealloc, initial, pinned)
        for st in steps:
            st['slots'] = {kind: slot_of[kind][st['own']] for kind in KINDS}
            for kind in KINDS:
                idx = [slot_of[kind][x] for x in st['kv'][kind]]
                for i in idx:
                    if (i < 0).any():
                        raise AssertionError('a segment reads a token that has no slot')
                st['kv_indptr_' + kind] = np.concatenate([[0], np.cumsum([len(i) for i in idx])])
                st['kv_indices_' + kind] = np.concatenate(idx)
            del st['kv']
        return dict(steps=steps, cap=cap, slot_of=slot_of, readout=readout)

    def _allocate(self, kind, steps, last_read, prealloc, initial, pinned):
        """Liveness slot allocator for one kind: computed tokens take the lowest free slots (then new ones on top);
        with several steps, a slot is freed after the last step that reads its token. Resident tokens (`initial`, or
        the `prealloc` head) keep their slots; `pinned` offsets are never freed (reference `lean_core.py:198-222`)."""
        if initial is not None:
            table = initial[kind].copy()
        else:
            table = np.full(self.num_tokens, -1)
            table[np.asarray(prealloc, dtype=np.int64)] = np.arange(len(prealloc))
        last = last_read
        if pinned is not None:
            last[pinned[kind]] = len(steps)
        resident = table >= 0
        top = int(table.max()) + 1 if resident.any() else 0
        taken = np.zeros(top, dtype=bool)
        taken[table[resident]] = True
        free = sorted(np.flatnonzero(~taken).tolist(), reverse=True)   # pop() gives the lowest free slot
        multi = len(steps) > 1
        for k, st in enumerate(steps):
            own = st['own']
            reuse = min(len(free), len(own))
            got = [free.pop() for _ in range(reuse)]
            fresh = top + np.arange(len(own) - reuse)
            table[own] = np.concatenate([np.asarray(got, dtype=np.int64), fresh])
            top += len(own) - reuse
            resident[own] = True
            if multi:
                gone = np.flatnonzero(resident & (last <= k))
                resident[gone] = False
                free.extend(table[gone].tolist())
                free.sort(reverse=True)
        return table, top
