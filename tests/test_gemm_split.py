"""The split schedule of the SM-pair GEMM kernel on the CPU (`morj_gemm_split_walk`, the same host/device code the
kernel walks): every k-block of every tile is computed exactly once, a cut tile is shared by two neighbouring pairs
(head on pair p, tail on pair p + 1), a pair waits only on a lower pair, and the pairs' k-block counts differ by at
most one."""
import numpy as np
import pytest

from morj_b200 import _native as nat

WHOLE, HEAD, TAIL = 0, 1, 2


def walks(tiles, pairs, kb):
    return [nat.split_walk(tiles, pairs, kb, p) for p in range(pairs)]


@pytest.mark.parametrize('tiles,pairs,kb', [
    (168, 74, 336),    # 2040 x 5376 x 21504 at 256-wide tiles (the down projection)
    (168, 74, 64),     # 2040 x 5376 x 4096 (the O projection)
    (1344, 74, 84),    # 2040 x 43008 x 5376 (gate / up)
    (256, 74, 84),     # 2040 x 8192 x 5376 (QKV, pair kernel)
    (75, 74, 1), (75, 74, 2), (147, 74, 3), (149, 74, 7), (10, 4, 5), (5, 4, 1), (7, 2, 9), (3, 2, 1000),
    (148, 74, 5), (74, 74, 5), (20, 74, 5), (1, 1, 3), (9, 1, 4),
])
def test_every_k_block_once_and_balanced(tiles, pairs, kb):
    cover = np.zeros((tiles, kb), dtype=np.int32)
    owner_head, owner_tail = {}, {}
    per_pair = []
    split = tiles > pairs and tiles % pairs != 0 and pairs > 1
    for p, items in enumerate(walks(tiles, pairs, kb)):
        kinds = items[:, 3].tolist()
        assert kinds.count(HEAD) <= 1 and kinds.count(TAIL) <= 1
        done = 0
        for tile, k0, k1, kind in items.tolist():
            assert 0 <= tile < tiles and 0 <= k0 < k1 <= kb
            assert kind == (TAIL if k0 > 0 else HEAD if k1 < kb else WHOLE)
            cover[tile, k0:k1] += 1
            done += k1 - k0
            if kind == HEAD:
                owner_head[tile] = p
            elif kind == TAIL:
                owner_tail[tile] = p
        if HEAD in kinds:   # the head piece comes first among the pair's split items (written early) ...
            dp_tiles = (tiles // pairs - 1) * pairs
            assert kinds.index(HEAD) == int((items[:, 0] < dp_tiles).sum())
        if TAIL in kinds:   # ... the tail piece last (it waits for the lower pair's head)
            assert kinds.index(TAIL) == len(kinds) - 1
        per_pair.append(done)
    assert (cover == 1).all()
    assert owner_head.keys() == owner_tail.keys()
    for tile, p in owner_head.items():
        assert owner_tail[tile] == p + 1
    if split:
        assert max(per_pair) - min(per_pair) <= 1
    else:
        assert not owner_head


def test_bad_arguments():
    with pytest.raises(ValueError):
        nat.split_walk(10, 4, 0, 0)
    with pytest.raises(ValueError):
        nat.split_walk(10, 4, 5, 4)


@pytest.mark.parametrize('tiles,kb,ctas', [
    (42, 336, 148),    # 9 x 5376 x 21504 (the last layer's down projection)
    (42, 64, 148),     # 9 x 5376 x 4096 (O)
    (336, 84, 148),    # 9 x 43008 x 5376 (gate / up)
    (2, 65, 130), (1, 1, 1), (208, 9, 148), (5, 3, 15), (3, 1000, 7), (148, 1, 148),
])
def test_skinny_schedule_covers_every_k_block_once(tiles, kb, ctas):
    """`morj_gemm_skinny_walk` (the weight-streaming kernel's schedule, same host/device code): every k-block of every
    tile once; a tile's pieces are consecutive CTAs in k order, numbered 0.. on each and counted the same by all; the
    CTAs' k-block counts differ by at most one."""
    cover = np.zeros((tiles, kb), dtype=np.int32)
    pieces = {}
    per_cta = []
    for c in range(ctas):
        items = nat.skinny_walk(tiles, kb, ctas, c)
        assert len(items) >= 1
        per_cta.append(int(sum(k1 - k0 for _, k0, k1, _, _ in items)))
        for t, k0, k1, piece, n in items:
            assert 0 <= k0 < k1 <= kb
            cover[t, k0:k1] += 1
            pieces.setdefault(t, []).append((k0, c, piece, n))
    assert (cover == 1).all()
    assert max(per_cta) - min(per_cta) <= 1
    for t, ps in pieces.items():
        ps.sort()
        assert [p for _, _, p, _ in ps] == list(range(len(ps)))
        assert all(n == len(ps) for _, _, _, n in ps)
        assert [c for _, c, _, _ in ps] == list(range(ps[0][1], ps[0][1] + len(ps)))


def test_skinny_walk_rejects_bad_arguments():
    with pytest.raises(ValueError):
        nat.skinny_walk(2, 3, 7, 0)  # more CTAs than units
    with pytest.raises(ValueError):
        nat.skinny_walk(2, 3, 3, 3)  # no such CTA
