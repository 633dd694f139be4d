"""Tensor-parallel sharding on the CPU (gloo, 2 ranks): the oracle run on each rank's shard, with its two
row-parallel projections summed over ranks, reproduces the unsharded model (`morj_b200.tp`)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from morj_b200 import workloads
        from morj_b200.checkpoint import random_state
        from morj_b200.tp import shard_config, shard_getter
        from morj_b200.tree import Tree
        from oracle.lean_oracle import OracleModel
        top = workloads.tiny_config()
        state = random_state(top, seed=0)
        get = shard_getter(top, state.__getitem__, rank, world)
        local_top = shard_config(top, world)
        local = {k: get(k) for k in state}
        model = OracleModel(local_top, local)

        def reduce(t):
            t = t.contiguous().clone()
            dist.all_reduce(t)
            return t
        model.reduce = reduce
        t = workloads.tiny_tree(0)
        probs = model.forward_tree(Tree, t['seqs'], t['label_ids'], 'fp32')
        out[rank] = np.concatenate(probs)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_forward_matches_the_whole_model():
    from morj_b200 import workloads
    from morj_b200.checkpoint import random_state
    from morj_b200.tree import Tree
    from oracle.lean_oracle import OracleModel
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True, start_method='spawn')
    top = workloads.tiny_config()
    t = workloads.tiny_tree(0)
    whole = np.concatenate(OracleModel(top, random_state(top, seed=0)).forward_tree(Tree, t['seqs'], t['label_ids'],
                                                                                   'fp32'))
    for r in range(world):
        assert np.abs(out[r] - whole).max() < 1e-5


def test_shard_shapes_and_divisibility():
    from morj_b200 import workloads
    from morj_b200.checkpoint import PREFIX, tensor_shapes
    from morj_b200.tp import shard_config, shard_getter
    top = workloads.gemma31b_config()
    for world in (2, 4, 8):
        local = shard_config(top, world)['text_config']
        assert (local['num_attention_heads'], local['num_key_value_heads'], local['intermediate_size']) == \
            (32 // world, 16 // world, 21504 // world)
    small = workloads.tiny_config()
    shapes = dict(tensor_shapes(small))
    fake = {k: torch.zeros(s) for k, s in shapes.items()}
    g = shard_getter(small, fake.__getitem__, 1, 2)
    assert g(PREFIX + 'layers.0.self_attn.q_proj.weight').shape == (128, 256)
    assert g(PREFIX + 'layers.0.self_attn.o_proj.weight').shape == (256, 128)
    assert g(PREFIX + 'layers.1.mlp.down_proj.weight').shape == (256, 512)
    assert g(PREFIX + 'embed_tokens.weight').shape == (4096, 256)
    with pytest.raises(ValueError, match='divisible'):
        shard_config(top, 3)
