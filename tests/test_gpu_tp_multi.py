"""Tensor parallelism on every GPU of the box (2, 4 or 8 ranks), peer exchange and NCCL: a 2-layer model whose
heads and intermediate size divide by 8 (hidden 512, 16 query / 8 KV heads of 64, GeGLU 2048) sharded over all
ranks gives the label probabilities of the same model on one GPU (within 1e-2; two layers leave no depth for BF16
roundings to accumulate), every rank the same ones, on a 301- and a 2,151-row request. Child processes, one per
GPU, NVLS off; skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def config():
    from morj_b200 import workloads
    cfg = workloads.text_config(2, 512, 16, 8, 64, 2048, 4096, 64, 2)
    return dict(text_config=cfg, image_token_id=4095, boi_token_id=4094, eoi_token_id=4093)


def request(prefix=150):
    """4 branches over a shared prefix (150 or 2,000 tokens: 301 or 2,151 rows, 2 or 17 row blocks of 128)."""
    rng = np.random.default_rng(3)
    head = [int(v) for v in rng.integers(0, 4000, prefix)]
    seqs = [head + [int(v) for v in rng.integers(0, 4000, n)] for n in (30, 45, 12, 64)]
    labels = [[7, 8, 9], [7, 8, 9], [10, 11], list(range(100, 140))]
    return seqs, labels


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
        from morj_b200.checkpoint import random_state
        from morj_b200.lean_core import LeanGemma4
        top = config()
        res = {}
        for comm in ('peer', 'nccl'):
            model = LeanGemma4.from_state(top, random_state(top, seed=5), device=f'cuda:{rank}',
                                          tp_group=dist.group.WORLD, tp_comm=comm)
            for prefix in (150, 2000):
                seqs, labels = request(prefix)
                for steps in ((16384, 8192), (96, 64)):  # one step, and a pass cut into steps
                    model.single_max, model.step_tokens = steps
                    req = model.prepare(seqs, labels)
                    res[(comm, prefix, steps)] = np.concatenate(model.run(req, list(range(len(seqs)))))
            if model.peer is not None:
                dist.barrier()
                model.peer.close()
                dist.barrier()
        out[rank] = res
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_on_every_gpu_matches_one_gpu():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip('needs 2 or more GPUs')
    world = 8 if world >= 8 else 4 if world >= 4 else 2
    # the ranks first (spawned, before this process touches CUDA), then the one-GPU run here
    out = mp.get_context('spawn').Manager().dict()
    mp.start_processes(_rank, args=(world, _port(), out), nprocs=world, join=True, start_method='spawn')
    from morj_b200.checkpoint import random_state
    from morj_b200.lean_core import LeanGemma4
    top = config()
    one = LeanGemma4.from_state(top, random_state(top, seed=5), device='cuda:0')
    want = {}
    for prefix in (150, 2000):
        seqs, labels = request(prefix)
        want[prefix] = np.concatenate(one.run(one.prepare(seqs, labels), list(range(len(seqs)))))
    for key, got in out[0].items():
        err = np.abs(got - want[key[1]]).max()
        print(f'\n{world} ranks {key}: max |TP - one GPU| = {err:.2e}')
        assert err <= 1e-2, (world, key, err)
        for r in range(1, world):
            assert np.array_equal(got, out[r][key])  # every rank computes the same probabilities
