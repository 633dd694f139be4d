"""The peer-memory exchange of tensor parallelism, on the CPU: buffer layout, the counting rules of the kernels
against the host's cumulative targets, and the handle swap over a 2-rank gloo group (`morj_b200.tp`)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from morj_b200.tp import BLOCK, exchange_layout, owner, partial_target, row_target


@pytest.mark.parametrize('world', [1, 2, 3, 4, 8])
@pytest.mark.parametrize('hidden,max_rows', [(256, 1), (256, 1000), (5376, 16384), (5376, 16385)])
def test_exchange_layout(world, hidden, max_rows):
    lay = exchange_layout(world, hidden, max_rows)
    mb = lay['max_blocks']
    assert mb * BLOCK >= max_rows
    regions = sorted(lay['regions'].values())
    for (o1, s1), (o2, _) in zip(regions, regions[1:]):
        assert o1 % 256 == 0 and o1 + s1 <= o2
    assert regions[-1][0] + regions[-1][1] <= lay['nbytes']
    assert lay['regions']['part'][1] == lay['regions']['x'][1] == lay['regions']['h'][1] == mb * BLOCK * hidden * 2
    assert lay['regions']['partials'][1] == mb * 8 == lay['regions']['rows'][1]


def _simulate_site(partials, rows, world, hidden, n, max_blocks, bn, rng):
    """One site, by the kernels' counting rules: `gemm_sm100.cu` epilogue_peer (every epilogue warp of every tile of
    a row block below ceil(n/128) counts that tile's columns on the owner's counter), `tp_peer.cu` reduce_kernel
    (one CTA per owned row below ceil(n/128) * 128 counts 1 row on every rank; the last CTA pads both counters
    for the blocks past n). The order of arrivals is shuffled: counters are sums."""
    n_blocks = -(-n // BLOCK)
    events = []
    for r in range(world):
        for b in range(n_blocks):
            for t in range(-(-hidden // bn)):
                cols = min(hidden, (t + 1) * bn) - t * bn
                events += [('p', owner(b, world), b, cols)] * 4
        for b in range(n_blocks, max_blocks):
            events.append(('p', owner(b, world), b, 4 * hidden))
            if owner(b, world) == r:
                events += [('r', q, b, 128) for q in range(world)]
        for b in range(r, n_blocks, world):
            events += [('r', q, b, 1) for q in range(world)] * 128
    for i in rng.permutation(len(events)):
        kind, rank, b, v = events[i]
        (partials if kind == 'p' else rows)[rank][b] += v


@pytest.mark.parametrize('world', [1, 2, 3, 4, 8])
def test_counters_reach_the_targets_on_every_block_at_every_site(world):
    hidden, max_rows = 328, 3000
    mb = exchange_layout(world, hidden, max_rows)['max_blocks']
    rng = np.random.default_rng(world)
    partials = np.zeros((world, mb), dtype=np.int64)
    rows = np.zeros((world, mb), dtype=np.int64)
    sizes = [1, 127, 128, 129, 3000, 2999, 640, 1, 1700]
    for site, n in enumerate(sizes, 1):
        _simulate_site(partials, rows, world, hidden, n, mb, int(rng.choice([128, 192, 208, 256])), rng)
        # the owner's counter of every block holds the cumulative target (other ranks' copies stay zero)
        for b in range(mb):
            assert partials[owner(b, world), b] == partial_target(site, world, hidden)
            assert (rows[:, b] == row_target(site)).all()
        assert partials.sum() == mb * partial_target(site, world, hidden)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from morj_b200.tp import gather_handles
        out[rank] = gather_handles(dist.group.WORLD, bytes([rank]) * 72)
    finally:
        dist.destroy_process_group()


def test_handles_are_swapped_in_rank_order_over_gloo():
    world = 2
    out = mp.Manager().dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True, start_method='spawn')
    for r in range(world):
        assert out[r] == [bytes([q]) * 72 for q in range(world)]


def _protocol_rank(rank, world, port, out):
    """One rank of a pass sequence in which rank 1 reaches pass 1 three seconds late and reports a device error
    (0x104, a peer wait that ran out) in pass 2."""
    import time

    import torch
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from morj_b200.tp import PassProtocol
        proto = PassProtocol(dist.group.WORLD)
        counters = torch.full((4,), 7, dtype=torch.int64)  # stand-in for the rank's counter regions
        sites = [5]

        def clear():
            counters.zero_()
            sites[0] = 0
        log = []
        for pas in (1, 2, 3):
            if pas == 1 and rank == 1:
                time.sleep(3.0)
            t0 = time.time()
            proto.begin()
            log.append(('begin', pas, t0, time.time()))
            code = proto.agree(0x104 if (pas == 2 and rank == 1) else 0)
            if code:
                proto.recover(clear)
            log.append(('end', pas, code, int(counters.sum()), sites[0]))
        out[rank] = log
    finally:
        dist.destroy_process_group()


def test_pass_protocol_holds_an_early_rank_and_shares_a_failure_over_gloo():
    """A rank that reaches a pass late holds the others at the pass barrier (so no kernel waits on it against its
    bound), and a device failure on one rank is seen by all, which all zero their counters and go on in step."""
    world = 2
    out = mp.Manager().dict()
    mp.start_processes(_protocol_rank, args=(world, _free_port(), out), nprocs=world, join=True, start_method='spawn')
    r0, r1 = out[0], out[1]
    begin0 = [e for e in r0 if e[0] == 'begin' and e[1] == 1][0]
    begin1 = [e for e in r1 if e[0] == 'begin' and e[1] == 1][0]
    assert begin0[3] >= begin1[2] - 0.05  # rank 0 left the first barrier only once the late rank reached it
    assert begin0[3] - begin0[2] > 2.0
    for log in (r0, r1):
        ends = {e[1]: e for e in log if e[0] == 'end'}
        assert ends[1][2] == 0 and ends[3][2] == 0
        assert ends[2][2] == 0x104  # both ranks see rank 1's failure
        assert ends[2][3] == 0 and ends[2][4] == 0  # and both cleared their counters and the site count
