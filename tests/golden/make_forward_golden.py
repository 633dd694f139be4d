"""Record the reference lean path's label probabilities on the tiny random-init model (run where the reference
source is available; nothing here runs on a GPU):

    python tests/golden/make_forward_golden.py /path/to/reference

The reference's own `LeanGemma4.prepare` / `run` / `_step` / `_last_layer` (`aleria_judge/lean_core.py:428-737`) run
on the CPU with: its Triton kernels in Triton's interpreter (TRITON_INTERPRET=1, with FP32 -> BF16 conversions
rounded to nearest even as the compiled kernels do), and stand-ins for the GPU-only
FlashInfer calls written here from FlashInfer's documented semantics (paged prefill over page-size-1 pages with the
bottom-right causal mask, `window_left`, `custom_mask`, GQA and `sm_scale`; `rmsnorm`; `gelu_tanh_and_mul`). The
same weights also go through transformers' `Gemma4ForCausalLM` in FP32, one branch at a time.

Writes `tests/golden/forward_tiny.json`: per case the request, the reference's probabilities, and (text cases) the
transformers FP32 probabilities, plus a checksum of the seeded weights so a test can tell if they drifted.
"""
import json
import math
import os
import sys
import types

os.environ['TRITON_INTERPRET'] = '1'

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from morj_b200 import workloads  # noqa: E402
from morj_b200.checkpoint import PREFIX, random_state  # noqa: E402


# ---- FlashInfer stand-in (third-party GPU library; semantics restated from its documentation) ---------------------
class PagedPrefill:
    def __init__(self, workspace, layout):
        assert layout == 'NHD'

    def plan(self, qo_indptr, kv_indptr, kv_indices, last_page_len, num_qo_heads, num_kv_heads, head_dim, page_size,
             causal=False, sm_scale=None, window_left=-1, custom_mask=None, q_data_type=None, kv_data_type=None):
        assert page_size == 1
        self.qo = np.asarray(qo_indptr.cpu() if hasattr(qo_indptr, 'cpu') else qo_indptr, dtype=np.int64)
        self.kp = np.asarray(kv_indptr.cpu() if hasattr(kv_indptr, 'cpu') else kv_indptr, dtype=np.int64)
        self.ki = np.asarray(kv_indices.cpu(), dtype=np.int64)
        self.causal, self.scale, self.window_left = causal, sm_scale, window_left
        self.mask = None if custom_mask is None else custom_mask.cpu().numpy().astype(bool)
        self.hq, self.hk = num_qo_heads, num_kv_heads

    def run(self, q, kv, out=None):
        k_pool, v_pool = kv
        k_pool = k_pool[:, 0].float()
        v_pool = v_pool[:, 0].float()
        res = torch.zeros(q.shape, dtype=torch.float32)
        g = self.hq // self.hk
        moff = 0
        for s in range(len(self.qo) - 1):
            q0, q1 = int(self.qo[s]), int(self.qo[s + 1])
            idx = torch.as_tensor(self.ki[self.kp[s]:self.kp[s + 1]])
            ql, kl = q1 - q0, len(idx)
            qi = np.arange(ql)[:, None]
            ki = np.arange(kl)[None, :]
            if self.mask is not None:
                vis = self.mask[moff:moff + ql * kl].reshape(ql, kl)
                moff += ql * kl
            else:
                vis = np.ones((ql, kl), dtype=bool)
                if self.causal:
                    vis &= ki <= qi + kl - ql
                if self.window_left >= 0:
                    vis &= ki + ql + self.window_left >= kl + qi
            K = k_pool[idx].repeat_interleave(g, 1)
            V = v_pool[idx].repeat_interleave(g, 1)
            S = torch.einsum('qhd,khd->hqk', q[q0:q1].float(), K) * self.scale
            S = S.masked_fill(~torch.as_tensor(vis)[None], float('-inf'))
            res[q0:q1] = torch.einsum('hqk,khd->qhd', torch.softmax(S, -1), V)
        res = res.to(q.dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res


def fi_rmsnorm(x, w, eps):
    xf = x.float()
    return (xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def fi_gelu_tanh_and_mul(x):
    F = x.shape[-1] // 2
    a = x[..., :F].float()
    g = 0.5 * a * (1 + torch.tanh(math.sqrt(2 / math.pi) * (a + 0.044715 * a ** 3)))
    return (g * x[..., F:].float()).to(x.dtype)


def install_flashinfer_standin():
    fi = types.ModuleType('flashinfer')
    fi.BatchPrefillWithPagedKVCacheWrapper = PagedPrefill
    fi.rmsnorm = fi_rmsnorm
    act = types.ModuleType('flashinfer.activation')
    act.gelu_tanh_and_mul = fi_gelu_tanh_and_mul
    fi.activation = act
    sys.modules['flashinfer'] = fi
    sys.modules['flashinfer.activation'] = act
    return fi


class _Event:
    def __init__(self, **kw):
        pass

    def record(self):
        pass

    def elapsed_time(self, other):
        return 0.0


def reference_model(lean_core, top, state, single_max=16384, step_tokens=8192):
    """A reference LeanGemma4 on the CPU: the fields its constructor sets (`lean_core.py:342-416`), built without
    the CUDA-only parts."""
    cfg = top['text_config']
    m = lean_core.LeanGemma4.__new__(lean_core.LeanGemma4)
    m.fi = sys.modules['flashinfer']
    m.image_id, m.boi_id, m.eoi_id = top['image_token_id'], top['boi_token_id'], top['eoi_token_id']
    m.cfg, m.hidden, m.eps, m.softcap = cfg, cfg['hidden_size'], cfg['rms_norm_eps'], cfg['final_logit_softcapping']
    m.types, m.window, m.hq = cfg['layer_types'], cfg['sliding_window'], cfg['num_attention_heads']
    m.geom = {'sliding_attention': (cfg['num_key_value_heads'], cfg['head_dim']),
              'full_attention': (cfg['num_global_key_value_heads'], cfg['global_head_dim'])}
    m.device = 'cpu'
    get = lambda k: state[k].clone()
    m.embed, m.norm = get(PREFIX + 'embed_tokens.weight'), get(PREFIX + 'norm.weight')
    m.embed_scale = torch.tensor(m.hidden ** 0.5, dtype=torch.bfloat16)
    m.layers = []
    for i, kind in enumerate(m.types):
        p = f'{PREFIX}layers.{i}.'
        a = p + 'self_attn.'
        parts = [get(a + 'q_proj.weight'), get(a + 'k_proj.weight')]
        if kind == 'sliding_attention':
            parts.append(get(a + 'v_proj.weight'))
        m.layers.append(dict(kind=kind, qkv=torch.cat(parts, 0), o=get(a + 'o_proj.weight'),
                             gu=torch.cat([get(p + 'mlp.gate_proj.weight'), get(p + 'mlp.up_proj.weight')], 0),
                             down=get(p + 'mlp.down_proj.weight'), q_norm=get(a + 'q_norm.weight'),
                             k_norm=get(a + 'k_norm.weight'), in_ln=get(p + 'input_layernorm.weight'),
                             post_attn=get(p + 'post_attention_layernorm.weight'),
                             pre_ff=get(p + 'pre_feedforward_layernorm.weight'),
                             post_ff=get(p + 'post_feedforward_layernorm.weight'),
                             scalar=get(p + 'layer_scalar').to(torch.bfloat16)))
    rp = cfg['rope_parameters']
    d = cfg['head_dim']
    m.inv_freq = {'sliding_attention': 1.0 / (rp['sliding_attention']['rope_theta'] ** (
        torch.arange(0, d, 2, dtype=torch.int64).float() / d))}
    gd = cfg['global_head_dim']
    angles = int(rp['full_attention'].get('partial_rotary_factor', 1.0) * gd // 2)
    rot = 1.0 / (rp['full_attention']['rope_theta'] ** (torch.arange(0, 2 * angles, 2, dtype=torch.int64).float() / gd))
    m.inv_freq['full_attention'] = torch.cat([rot, torch.zeros(gd // 2 - angles)])
    m.wrappers = {k: PagedPrefill(None, 'NHD') for k in ('sliding_attention', 'full_attention', 'bidir')}
    m.last_wrapper = PagedPrefill(None, 'NHD')
    m.prune_last = True
    import triton
    m.H_BLOCK = triton.next_power_of_2(m.hidden)
    m.kv_bytes = sum(2 * 2 * m.geom[k][0] * m.geom[k][1] for k in m.types)
    m.retain_budget = 10 * 2**30
    m.shared, m.shared_kv = None, None
    m.single_max, m.step_tokens = single_max, step_tokens
    m.timing = {}
    m.free_bytes = 1 << 40
    hd = max(dd for _, dd in m.geom.values())
    m.act_bytes = 2 * (4 * m.hidden + max(l['qkv'].shape[0] for l in m.layers) + 2 * m.hq * hd
                       + 3 * m.layers[0]['gu'].shape[0] // 2)
    return m


def transformers_probs(top, state, seqs, label_ids):
    """transformers Gemma4ForCausalLM in FP32, each branch alone; softmax over the branch's labels of the final
    (softcapped) logits at its last token."""
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    cfg = dict(top['text_config'])
    conf = Gemma4TextConfig(**cfg)
    conf._attn_implementation = 'eager'
    model = Gemma4ForCausalLM(conf).float().eval()
    sd = {'model.' + k[len(PREFIX):]: v.float() for k, v in state.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [k for k in missing if k != 'lm_head.weight']
    assert not missing and not unexpected, (missing[:5], unexpected[:5])
    out = []
    with torch.no_grad():
        for seq, ids in zip(seqs, label_ids):
            logits = model(input_ids=torch.as_tensor([seq])).logits[0, -1]
            out.append(torch.softmax(logits[torch.as_tensor(ids)].float(), -1).double().tolist())
    return out


def round_bf16_like_the_gpu():
    """Triton's CPU interpreter converts FP32 to BF16 by truncating the mantissa, whereas the compiled kernels the
    reference runs on the GPU round to nearest even. Route the interpreter's FP32 -> BF16 conversion through torch's
    round-to-nearest-even so the recorded numbers are the GPU kernels' numbers."""
    from triton.runtime import interpreter as tri
    import triton.language as tl
    plain = tri._convert_float

    def convert(input, input_dtype, output_dtype, rounding_mode):
        if input_dtype == tl.float32 and output_dtype == tl.bfloat16:
            f = torch.from_numpy(np.frombuffer(input.tobytes(), dtype=np.float32).copy())
            return f.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).reshape(np.shape(input))
        return plain(input, input_dtype, output_dtype, rounding_mode)
    tri._convert_float = convert


def weight_checksum(state):
    return float(sum(v.float().double().abs().sum().item() for v in state.values()))


def tiny_images(top):
    """Two image blocks for the tiny model: 80 soft tokens (longer than the 64-token window: explicit mask path) and
    16 (shorter: windowed non-causal path); features N(0,1)/16, seed 3."""
    g = torch.Generator().manual_seed(3)
    return [(torch.randn(n, top['text_config']['hidden_size'], generator=g) / 16.0).to(torch.bfloat16)
            for n in (80, 16)]


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else '/root/reference'
    install_flashinfer_standin()
    sys.path.insert(0, ref_root)
    torch.cuda.Event = _Event
    torch.cuda.current_stream = lambda *a: types.SimpleNamespace(synchronize=lambda: None)
    round_bf16_like_the_gpu()
    from aleria_judge import lean_core
    top = workloads.tiny_config()
    state = random_state(top, seed=0)
    t = workloads.tiny_tree(0)
    cases = []

    def run_case(name, seqs, labels, passes, retain=False, single_max=16384, step_tokens=8192, images=None,
                 with_transformers=False, retain_budget=None):
        m = reference_model(lean_core, top, state, single_max, step_tokens)
        if retain_budget is not None:
            m.retain_budget = retain_budget
        req = m.prepare(seqs, labels, retain=retain, images=images)
        probs = [m.run(req, list(p)) for p in passes]
        rec = dict(name=name, seqs=seqs, label_ids=labels, passes=passes, retain=retain, single_max=single_max,
                   step_tokens=step_tokens, retain_budget=retain_budget, images=images is not None,
                   reference=probs, retained=bool(req.retain), pinned=bool(req.pinned))
        if with_transformers:
            rec['transformers_fp32'] = transformers_probs(top, state, seqs, labels)
        cases.append(rec)
        print(name, 'retain', req.retain, 'pinned', req.pinned, probs[0][0][:3])

    run_case('tiny', t['seqs'], t['label_ids'], [[0, 1, 2, 3]], with_transformers=True)
    run_case('tiny-steps', t['seqs'], t['label_ids'], [[0, 1, 2, 3]], single_max=64, step_tokens=48)
    run_case('tiny-retain-two-pass', t['seqs'], t['label_ids'], [[0, 2], [1, 3]], retain=True)
    # pinned: a retained request whose whole pool does not fit the budget keeps only what the second pass reads
    run_case('tiny-pinned-two-pass', t['seqs'], t['label_ids'], [[1, 3], [0, 2]], retain=True, single_max=80,
             step_tokens=40, retain_budget=100 * 1024)
    # deeper tree: branches sharing question blocks, ragged labels
    rng = np.random.default_rng(1)
    head = [int(v) for v in rng.integers(0, 4000, 40)]
    qa, qb = [int(v) for v in rng.integers(0, 4000, 20)], [int(v) for v in rng.integers(0, 4000, 30)]
    seqs = [head + qa + [int(v) for v in rng.integers(0, 4000, n)] for n in (5, 9)] + \
           [head + qb + [int(v) for v in rng.integers(0, 4000, n)] for n in (1, 70)]
    labels = [[11, 12], [13, 14, 15], [16, 17, 18, 19, 20], [21, 22, 23]]
    run_case('tiny-nested', seqs, labels, [[0, 1, 2, 3]], with_transformers=True)
    images = tiny_images(top)
    pre = [int(v) for v in rng.integers(0, 4000, 6)]
    mid = [int(v) for v in rng.integers(0, 4000, 10)]
    img = top['image_token_id']
    img_seqs = [pre + [img] + mid + [img] + [int(v) for v in rng.integers(0, 4000, n)] for n in (12, 20, 7)]
    img_labels = [[31, 32, 33], [31, 32, 33], [40, 41]]
    run_case('tiny-images', img_seqs, img_labels, [[0, 1, 2]], images=images)
    run_case('tiny-images-steps', img_seqs, img_labels, [[0, 1, 2]], images=images, single_max=100, step_tokens=50)
    path = os.path.join(HERE, 'forward_tiny.json')
    with open(path, 'w') as f:
        json.dump(dict(source='aleria_judge/lean_core.py LeanGemma4 on CPU (Triton interpreter, FlashInfer stand-in)',
                       config=top, seed=0, weight_checksum=weight_checksum(state), cases=cases), f)
    print('wrote', path, os.path.getsize(path), 'bytes')


if __name__ == '__main__':
    main()
