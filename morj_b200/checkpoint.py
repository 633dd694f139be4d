"""Checkpoint layout, seeded random-init weights and safetensors I/O for the Gemma-style text decoder.

Keys and shapes follow the checkpoint the reference engine loads (`aleria_judge/lean_core.py:360-382`: prefix
`model.language_model.`, fused at load into `qkv` and `gate/up`), so the same directory loads into either engine.
Random init (no real weights exist offline): linear and embedding weights N(0, std); RMSNorm weights and the
per-layer scalar 1 + N(0, norm_std) (non-trivial, so a kernel that ignored them would fail parity). The q and k norm
weights are further scaled by head_dim^-1/4: the model attends with scale 1.0 (its q/k norms carry the scale), so
unit q/k norm weights would give logits of standard deviation sqrt(head_dim) and a near one-hot, chaotic attention
that no trained checkpoint has; scaled, the logits have unit variance.
"""
import json
import os

import torch

PREFIX = 'model.language_model.'


def layer_geometry(cfg, kind):
    if kind == 'sliding_attention':
        return cfg['num_key_value_heads'], cfg['head_dim']
    return cfg['num_global_key_value_heads'], cfg['global_head_dim']


def tensor_shapes(top):
    """Ordered (key, shape) list of every tensor the engine loads."""
    cfg = top['text_config']
    H, F, V, hq = cfg['hidden_size'], cfg['intermediate_size'], cfg['vocab_size'], cfg['num_attention_heads']
    out = [(PREFIX + 'embed_tokens.weight', (V, H)), (PREFIX + 'norm.weight', (H,))]
    for i, kind in enumerate(cfg['layer_types']):
        hk, d = layer_geometry(cfg, kind)
        p = f'{PREFIX}layers.{i}.'
        a = p + 'self_attn.'
        out += [(a + 'q_proj.weight', (hq * d, H)), (a + 'k_proj.weight', (hk * d, H))]
        if kind == 'sliding_attention':
            out.append((a + 'v_proj.weight', (hk * d, H)))
        out += [(a + 'o_proj.weight', (H, hq * d)), (a + 'q_norm.weight', (d,)), (a + 'k_norm.weight', (d,)),
                (p + 'mlp.gate_proj.weight', (F, H)), (p + 'mlp.up_proj.weight', (F, H)),
                (p + 'mlp.down_proj.weight', (H, F)),
                (p + 'input_layernorm.weight', (H,)), (p + 'post_attention_layernorm.weight', (H,)),
                (p + 'pre_feedforward_layernorm.weight', (H,)), (p + 'post_feedforward_layernorm.weight', (H,)),
                (p + 'layer_scalar', (1,))]
    return out


def random_tensor(shape, gen, device, std=0.02, norm_std=0.1, key=''):
    if len(shape) == 1:  # norm weights and layer scalars
        t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * norm_std + 1.0
        if key.endswith(('q_norm.weight', 'k_norm.weight')):
            t = t * shape[0] ** -0.25
    else:
        t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std
    return t.to(torch.bfloat16)


def random_state(top, seed=0, std=0.02, norm_std=0.1, device='cpu'):
    """Every tensor of `tensor_shapes(top)`, drawn in order from one seeded generator on `device`."""
    gen = torch.Generator(device=device).manual_seed(seed)
    return {k: random_tensor(s, gen, device, std, norm_std, k) for k, s in tensor_shapes(top)}


def iter_random_state(top, seed=0, std=0.02, norm_std=0.1, device='cuda'):
    """Like `random_state` but one tensor at a time, large matrices drawn in row blocks (bounded FP32 temporaries),
    for full-size models generated straight on the GPU."""
    gen = torch.Generator(device=device).manual_seed(seed)
    for k, s in tensor_shapes(top):
        if len(s) == 2 and s[0] * s[1] > (1 << 28):
            t = torch.empty(s, dtype=torch.bfloat16, device=device)
            step = max(1, (1 << 27) // s[1])
            for r in range(0, s[0], step):
                e = min(s[0], r + step)
                t[r:e] = (torch.randn((e - r, s[1]), generator=gen, device=device) * std).to(torch.bfloat16)
            yield k, t
        else:
            yield k, random_tensor(s, gen, device, std, norm_std, k)


def write_checkpoint(model_dir, top, state):
    """config.json (`text_config` + image token ids), model.safetensors and its index, as the engine loads them."""
    from safetensors.torch import save_file
    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, 'config.json'), 'w') as f:
        json.dump(top, f, indent=1)
    save_file({k: v.contiguous().cpu() for k, v in state.items()}, os.path.join(model_dir, 'model.safetensors'))
    with open(os.path.join(model_dir, 'model.safetensors.index.json'), 'w') as f:
        json.dump({'weight_map': {k: 'model.safetensors' for k in state}}, f)


def open_checkpoint(model_dir, device):
    """(top-level config, get(key) -> tensor on `device`) for a safetensors checkpoint directory."""
    from safetensors import safe_open
    with open(os.path.join(model_dir, 'config.json')) as f:
        top = json.load(f)
    with open(os.path.join(model_dir, 'model.safetensors.index.json')) as f:
        index = json.load(f)['weight_map']
    handles = {fn: safe_open(os.path.join(model_dir, fn), 'pt', device=str(device)) for fn in sorted(set(index.values()))}
    return top, (lambda k: handles[index[k]].get_tensor(k))
