"""Tensor parallelism on 2 GPUs, with the row-parallel reductions over peer memory and over NCCL: the sharded
engine's label probabilities match the reference lean path's recorded probabilities, every rank computes the same
ones, and the two exchanges agree bit for bit. Runs as two spawned processes, one per GPU (NVLS off); skipped with
fewer than two GPUs."""
import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), 'golden', 'forward_tiny.json')


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, device_id=torch.device('cuda', rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        from morj_b200 import workloads
        from morj_b200.checkpoint import random_state
        from morj_b200.lean_core import LeanGemma4
        with open(GOLDEN) as f:
            cases = {c['name']: c for c in json.load(f)['cases']}
        top = workloads.tiny_config()
        res = {}
        for comm in ('peer', 'nccl'):
            model = LeanGemma4.from_state(top, random_state(top, seed=0), device=f'cuda:{rank}',
                                          tp_group=dist.group.WORLD, tp_comm=comm)
            for name in ('tiny', 'tiny-nested', 'tiny-steps', 'tiny-images'):
                c = cases[name]
                model.single_max, model.step_tokens = c['single_max'], c['step_tokens']
                images = None
                if c['images']:
                    from make_forward_golden import tiny_images
                    images = [f.to(f'cuda:{rank}') for f in tiny_images(top)]
                req = model.prepare(c['seqs'], c['label_ids'], images=images)
                res[(comm, name)] = np.concatenate(model.run(req, list(range(len(c['seqs'])))))
            if model.peer is not None:
                model.peer.close()
        out[rank] = res
    finally:
        dist.destroy_process_group()


def test_two_gpu_tensor_parallel_matches_reference():
    if torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    world = 2
    out = mp.get_context('spawn').Manager().dict()
    mp.start_processes(_rank, args=(world, _port(), out), nprocs=world, join=True, start_method='spawn')
    with open(GOLDEN) as f:
        cases = {c['name']: c for c in json.load(f)['cases']}
    for (comm, name), got in out[0].items():
        ref = np.concatenate([np.asarray(r) for r in cases[name]['reference'][0]])
        assert np.abs(got - ref).max() <= 1e-2, (comm, name)
        assert np.array_equal(got, out[1][(comm, name)])  # every rank computes the same probabilities
        # two ranks: the peer exchange's FP32 sum of the two BF16 partials is NCCL's BF16 sum, bit for bit
        assert np.array_equal(got, out[0][('nccl', name)]), name
