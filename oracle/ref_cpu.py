"""The reference's own lean path (`aleria_judge/lean_core.py`) run on the host CPU. TEST AND BASELINE INFRASTRUCTURE.

Only `tests/`, `tests/golden/` generators and `bench.py`'s CPU-baseline / reference arm use this module; the engine
(`morj_b200`) never imports it. Nothing here loads the B200 library.

The reference's forward needs a GPU for three third-party pieces. They are replaced, and nothing else is:

* FlashInfer's `BatchPrefillWithPagedKVCacheWrapper` (`lean_core.py:397,402`; `plan`/`run` at `609-635,677-681,
  723-728`), `flashinfer.rmsnorm` (`653,692,736`) and `flashinfer.activation.gelu_tanh_and_mul` (`685,733`): dense
  torch stand-ins written from FlashInfer's documented semantics (page size 1, bottom-right causal mask,
  `window_left`, `custom_mask`, GQA, `sm_scale`).
* The reference's three Triton kernels `_qkv_post`, `_attn_epilogue`, `_mlp_epilogue` (`lean_core.py:234-320`):
  `EAGER_KERNELS`, torch restatements that take the same launch (`kernel[grid](*args, num_warps=...)`) and compute the
  same values with the same BF16 rounding points (used for timing; the golden fixtures instead run the real Triton
  code in Triton's interpreter, see `tests/golden/make_forward_golden.py`).
* `torch.cuda.Event` and `torch.cuda.current_stream` (`lean_core.py:551-556`): host no-ops.

`reference_model` builds a `LeanGemma4` on the CPU with the fields its CUDA-only constructor sets
(`lean_core.py:342-416`); `prepare`, `run`, `_step`, `_last_layer` and the planner `Tree` are the reference's, unchanged.
"""
import math
import os
import sys
import time
import types

import numpy as np
import torch

PREFIX = 'model.language_model.'
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
# where the unmodified reference package is found: the offline install beside the repository (it travels with the
# repository to the benchmark machine), or a source checkout named by the caller
INSTALL = os.path.join(ROOT, 'baseline', '_ref')


# ---- FlashInfer stand-in (third-party GPU library; semantics restated from its documentation) ---------------------
class PagedPrefill:
    """Paged prefill attention over page-size-1 pages: per segment, queries attend to their `kv_indices` keys with
    the bottom-right-aligned causal mask and `window_left` (or an explicit `custom_mask`), in FP32, output in q's
    dtype."""

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


def install_cuda_standins():
    """`run`'s CUDA events and stream sync become host no-ops (everything runs synchronously on the CPU)."""
    torch.cuda.Event = _Event
    torch.cuda.current_stream = lambda *a: types.SimpleNamespace(synchronize=lambda: None)


# ---- torch-eager restatements of the reference's Triton kernels -------------------------------------------------
def _bf(x):
    return x.to(torch.bfloat16).float()


def _inv_rms(x, n, eps):
    """1 / sqrt(sum(x^2) / n + eps) per row, FP32, as the kernels compute it."""
    return 1.0 / torch.sqrt((x * x).sum(-1, keepdim=True) / n + eps)


def eager_qkv_post(grid, qkv, q_out, k_pool, v_pool, slots, qw, kw, cos, sin, stride_tok, HQ, HK, HAS_V, D, HALF, BH,
                   eps, **launch):
    """`_qkv_post` (`lean_core.py:234-277`) over `grid[0]` tokens: per head RMSNorm (q with `qw`, k with `kw`, v
    unweighted), BF16 rounding, rotate-half RoPE on q and k (v passes through), q to `q_out`, k/v to each token's
    pool slot. V reads the K columns when `HAS_V` is 0."""
    n = grid[0]
    x = torch.as_strided(qkv, (n, qkv.shape[-1]), (stride_tok, 1)).float()
    c, s = cos[:n].float()[:, None, :], sin[:n].float()[:, None, :]

    def head_out(cols, heads, w, rope):
        t = x[:, cols:cols + heads * D].reshape(n, heads, D)
        y = t * _inv_rms(t, D, eps)
        y = _bf(y * w.float() if w is not None else y)
        if not rope:
            return y.to(torch.bfloat16)
        y1, y2 = y[..., :HALF], y[..., HALF:]
        return torch.cat([y1 * c - y2 * s, y2 * c + y1 * s], -1).to(torch.bfloat16)
    if HQ:
        q_out.view(-1, HQ, D)[:n] = head_out(0, HQ, qw, True)
    if HK:
        idx = slots[:n].long()
        k_pool.view(-1, HK, D)[idx] = head_out(HQ * D, HK, kw, True)
        v_pool.view(-1, HK, D)[idx] = head_out((HQ + HAS_V * HK) * D, HK, None, False)


def eager_attn_epilogue(grid, o, x, h_out, w_post, w_pre, H, eps, BLOCK, **launch):
    """`_attn_epilogue` (`lean_core.py:290-302`): x += bf16(rms(o) * w_post) rounded to BF16; h = bf16(rms(x) *
    w_pre), over `grid[0]` rows."""
    n = grid[0]
    ov = o.reshape(-1, H)[:n].float()
    on = _bf(ov * _inv_rms(ov, H, eps) * w_post.float())
    xv = x.view(-1, H)
    xn = _bf(xv[:n].float() + on)
    xv[:n] = xn.to(torch.bfloat16)
    h_out.view(-1, H)[:n] = (xn * _inv_rms(xn, H, eps) * w_pre.float()).to(torch.bfloat16)


def eager_mlp_epilogue(grid, d, x, h_out, w_post, scale, w_next, H, eps, HAS_NEXT, BLOCK, **launch):
    """`_mlp_epilogue` (`lean_core.py:305-320`): x = bf16(bf16(x + bf16(rms(d) * w_post)) * layer_scalar); with
    `HAS_NEXT`, h = bf16(rms(x) * w_next), over `grid[0]` rows."""
    n = grid[0]
    dv = d.reshape(-1, H)[:n].float()
    dn = _bf(dv * _inv_rms(dv, H, eps) * w_post.float())
    xv = x.view(-1, H)
    xa = _bf(xv[:n].float() + dn)
    xs = _bf(xa * scale.float())
    xv[:n] = xs.to(torch.bfloat16)
    if HAS_NEXT:
        h_out.view(-1, H)[:n] = (xs * _inv_rms(xs, H, eps) * w_next.float()).to(torch.bfloat16)


class _Launchable:
    """`kernel[grid](*args, **launch)` as the reference launches its Triton kernels."""

    def __init__(self, fn):
        self.fn = fn

    def __getitem__(self, grid):
        return lambda *args, **kw: self.fn(tuple(grid), *args, **kw)


EAGER_KERNELS = {'_qkv_post': _Launchable(eager_qkv_post), '_attn_epilogue': _Launchable(eager_attn_epilogue),
                 '_mlp_epilogue': _Launchable(eager_mlp_epilogue)}


# ---- the reference package ----------------------------------------------------------------------------------------
def load_reference(source=None, eager=True):
    """Import the unmodified reference `aleria_judge.lean_core` for CPU use: FlashInfer and CUDA events replaced as
    above, and (with `eager`) its Triton kernels swapped for `EAGER_KERNELS` on the imported module. `source`: a
    directory holding the `aleria_judge` package; default the offline install (`baseline/_ref`). Raises ImportError
    when no reference is available."""
    path = source or INSTALL
    if not os.path.isdir(os.path.join(path, 'aleria_judge')):
        raise ImportError(f'no reference package under {path}')
    install_flashinfer_standin()
    install_cuda_standins()
    if path not in sys.path:
        sys.path.insert(0, path)
    from aleria_judge import lean_core
    if eager:
        for name, k in EAGER_KERNELS.items():
            setattr(lean_core, name, k)
    return lean_core


def reference_model(lean_core, top, state, single_max=16384, step_tokens=8192):
    """A reference `LeanGemma4` on the CPU: the fields its constructor sets (`lean_core.py:342-416`), built without
    the CUDA-only parts. `state`: tensors in the checkpoint key layout."""
    cfg = top['text_config']
    m = lean_core.LeanGemma4.__new__(lean_core.LeanGemma4)
    m.fi = sys.modules['flashinfer']
    m.image_id, m.boi_id, m.eoi_id = top['image_token_id'], top['boi_token_id'], top['eoi_token_id']
    m.cfg, m.hidden, m.eps, m.softcap = cfg, cfg['hidden_size'], cfg['rms_norm_eps'], cfg['final_logit_softcapping']
    m.types, m.window, m.hq = cfg['layer_types'], cfg['sliding_window'], cfg['num_attention_heads']
    m.geom = {'sliding_attention': (cfg['num_key_value_heads'], cfg['head_dim']),
              'full_attention': (cfg['num_global_key_value_heads'], cfg['global_head_dim'])}
    m.device = 'cpu'
    get = lambda k: state[k]
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
    m.H_BLOCK = 1 << (m.hidden - 1).bit_length()
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


# ---- timing the reference on the host CPU (the benchmark's reference arm and CPU baseline) -------------------------
class StampedLayers(list):
    """A model's layer list that records the time each layer starts when `_step`'s layer loop iterates it
    (`lean_core.py:655`); indexing and `len` are a list's."""

    def __iter__(self):
        for layer in list.__iter__(self):
            self.stamps.append(time.perf_counter())
            yield layer


def checkpoint_shapes(top):
    """(key, shape) of every tensor the reference loads (`lean_core.py:362-382`)."""
    cfg = top['text_config']
    H, F, V, hq = cfg['hidden_size'], cfg['intermediate_size'], cfg['vocab_size'], cfg['num_attention_heads']
    out = [(PREFIX + 'embed_tokens.weight', (V, H)), (PREFIX + 'norm.weight', (H,))]
    for i, kind in enumerate(cfg['layer_types']):
        hk, d = ((cfg['num_key_value_heads'], cfg['head_dim']) if kind == 'sliding_attention' else
                 (cfg['num_global_key_value_heads'], cfg['global_head_dim']))
        a, p = f'{PREFIX}layers.{i}.self_attn.', f'{PREFIX}layers.{i}.'
        out += [(a + 'q_proj.weight', (hq * d, H)), (a + 'k_proj.weight', (hk * d, H)),
                (a + 'o_proj.weight', (H, hq * d)), (a + 'q_norm.weight', (d,)), (a + 'k_norm.weight', (d,)),
                (p + 'mlp.gate_proj.weight', (F, H)), (p + 'mlp.up_proj.weight', (F, H)),
                (p + 'mlp.down_proj.weight', (H, F)), (p + 'input_layernorm.weight', (H,)),
                (p + 'post_attention_layernorm.weight', (H,)), (p + 'pre_feedforward_layernorm.weight', (H,)),
                (p + 'post_feedforward_layernorm.weight', (H,)), (p + 'layer_scalar', (1,))]
        if kind == 'sliding_attention':
            out.append((a + 'v_proj.weight', (hk * d, H)))
    return out


def timing_state(top, seed=0, std=0.02):
    """Weights for timing only, in the checkpoint key layout: every matrix is a seeded N(0, std) block tiled to its
    shape (the values do not change the work), norm weights and layer scalars 1."""
    block = (torch.randn(1 << 22, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16)
    state = {}
    for k, shape in checkpoint_shapes(top):
        n = int(np.prod(shape))
        if len(shape) == 1:
            state[k] = torch.ones(shape, dtype=torch.bfloat16)
        else:
            state[k] = block.repeat(-(-n // block.numel()))[:n].reshape(shape).clone()
    return state


class TimedReference:
    """The reference's own `LeanGemma4.prepare` + `run` (`lean_core.py:428-576`) on the host CPU over a 3-layer cut of
    a model (one sliding layer, one global layer, and the pruned global last layer `_last_layer`, as the 31B-class
    model's layer 59 is), on a full-size request tree. One `sample()` times one request end to end and each layer
    inside it; `extrapolate` scales the per-layer times to the full layer pattern:
    setup (prepare, planning, embedding) + n_sliding x sliding + n_global x global + the last layer and readout."""

    CUT = ['sliding_attention', 'full_attention', 'full_attention']

    def __init__(self, top, tree_in, source=None):
        self.lean_core = load_reference(source, eager=True)
        self.full_types = list(top['text_config']['layer_types'])
        if self.full_types[-1] != 'full_attention':
            raise ValueError('the 3-layer cut times a global last layer')
        cfg = dict(top['text_config'], layer_types=list(self.CUT), num_hidden_layers=len(self.CUT))
        cut = dict(top, text_config=cfg)
        self.m = reference_model(self.lean_core, cut, timing_state(cut))
        self.m.layers = StampedLayers(self.m.layers)
        self.tree_in = tree_in

    def sample(self):
        t = self.tree_in
        self.m.layers.stamps = []
        t0 = time.perf_counter()
        req = self.m.prepare(t['seqs'], t['label_ids'], images=t.get('images') or None)
        probs = self.m.run(req, list(range(len(t['seqs']))))
        t1 = time.perf_counter()
        self.last_req = req
        s = self.m.layers.stamps
        assert len(s) == 3 and len(probs) == len(t['seqs'])
        return dict(seconds=t1 - t0, setup=s[0] - t0, sliding=s[1] - s[0], global_=s[2] - s[1], last=t1 - s[2],
                    tokens=int(self.m.timing['tokens']))

    def plan_of_last_request(self):
        """The reference planner's pass plan for the last sampled request (every sequence, nothing cached)."""
        req, m = self.last_req, self.m
        seqs = list(range(len(self.tree_in['seqs'])))
        need = req.tree.pass_nodes(seqs, set(req.head_nodes))
        return req.tree.plan_pass(need, seqs, m.window, m.single_max, m.step_tokens, False, bidir=req.bidir)

    def extrapolate(self, r):
        """Seconds for the full layer pattern from one sample's per-layer times."""
        body = self.full_types[:-1]
        n_s = sum(1 for k in body if k == 'sliding_attention')
        return r['setup'] + n_s * r['sliding'] + (len(body) - n_s) * r['global_'] + r['last']
