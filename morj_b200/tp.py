"""Tensor-parallel sharding of the decoder for single-tree latency (T = 2, 4 or 8 GPUs, one process per GPU).

Rank r of T holds:
  * q heads [r * hq/T, (r+1) * hq/T) and KV heads [r * hk/T, (r+1) * hk/T) of every layer (column-parallel QKV;
    a query head's KV head h // (hq/hk) stays on the same rank), and the K/V pools of its KV heads;
  * the matching columns of the O projection (row-parallel): its partial [n, hidden] output is summed over ranks
    (all-reduce) before the post-attention norms;
  * intermediate slice [r * F/T, (r+1) * F/T) of the gate and up projections (column-parallel) and the matching
    columns of the down projection (row-parallel, all-reduced before the post-MLP norms);
  * the embedding, norms, layer scalars and the label head whole (replicated; every rank computes the same
    probabilities).
The tree plan is deterministic, so every rank plans the same steps on the host.
"""
from .checkpoint import PREFIX, layer_geometry


def shard_config(top, world):
    """The per-rank config: local head counts and intermediate size."""
    cfg = dict(top['text_config'])
    hq = cfg['num_attention_heads']
    for key in ('num_attention_heads', 'num_key_value_heads', 'num_global_key_value_heads', 'intermediate_size'):
        if cfg[key] % world:
            raise ValueError(f'{key} = {cfg[key]} is not divisible by {world} ranks')
    if (cfg['intermediate_size'] // world) % 128:
        raise ValueError('each rank needs a multiple of 128 intermediate rows (GeGLU tile layout)')
    for kind in ('sliding_attention', 'full_attention'):
        hk, _ = layer_geometry(cfg, kind)
        if (hq // world) % (hk // world) and (hk // world) % (hq // world):
            raise ValueError('query heads per KV head must stay on one rank')
    cfg['num_attention_heads'] = hq // world
    cfg['num_key_value_heads'] //= world
    cfg['num_global_key_value_heads'] //= world
    cfg['intermediate_size'] //= world
    return dict(top, text_config=cfg)


def shard_getter(top, get, rank, world):
    """`get(key)` for rank `rank`: the full tensor's shard (a contiguous copy), replicated tensors unchanged."""
    cfg = top['text_config']
    hq, F = cfg['num_attention_heads'], cfg['intermediate_size']

    def rows(t, n, width=1):
        per = n // world
        return t[rank * per * width:(rank + 1) * per * width].contiguous()

    def cols(t, n, width=1):
        per = n // world
        return t[:, rank * per * width:(rank + 1) * per * width].contiguous()

    def g(key):
        t = get(key)
        if not key.startswith(PREFIX + 'layers.'):
            return t
        i = int(key[len(PREFIX + 'layers.'):].split('.')[0])
        kind = cfg['layer_types'][i]
        hk, d = layer_geometry(cfg, kind)
        if key.endswith('self_attn.q_proj.weight'):
            return rows(t, hq, d)
        if key.endswith(('self_attn.k_proj.weight', 'self_attn.v_proj.weight')):
            return rows(t, hk, d)
        if key.endswith('self_attn.o_proj.weight'):
            return cols(t, hq, d)
        if key.endswith(('mlp.gate_proj.weight', 'mlp.up_proj.weight')):
            return rows(t, F)
        if key.endswith('mlp.down_proj.weight'):
            return cols(t, F)
        return t
    return g
