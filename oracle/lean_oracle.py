"""CPU oracle of the lean tree-prefill forward. TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm import this module, and only
as the checker or the timed CPU baseline. The engine (`morj_b200`) never imports it.

Two forms, both plain torch on the CPU:

* `forward_tree` restates the reference's `LeanGemma4._step` / `_last_layer` / readout (`aleria_judge/lean_core.py:
  599-737`, `558-561`) over a pass plan (the planner tables of `Tree.plan_pass`), with dense stand-ins for the
  third-party pieces: FlashInfer's paged prefill (page size 1, bottom-right causal mask, `window_left`, the image
  blocks' non-causal mask, `sm_scale`, GQA; used at `lean_core.py:609-635,677-681,723-728`), FlashInfer `rmsnorm` and
  `activation.gelu_tanh_and_mul`. With `precision='bf16'` it rounds to BF16 exactly where the reference path rounds
  (the reference's three Triton kernels `lean_core.py:234-320`, cuBLAS BF16 outputs, FlashInfer BF16 outputs); with
  `precision='fp32'` nothing is rounded (the "fp32 tree-mask path").
* `forward_branches` computes every branch as its own causal sequence (no tree, no plan): an independent statement
  of the same model (transformers' `modeling_gemma4` numerics, which the reference follows, `lean_core.py:15-17`).

Pins (`tests/test_oracle_golden.py`): `forward_tree(bf16)` reproduces probabilities recorded by running the
reference's own `_step` on CPU (`tests/golden/make_forward_golden.py`), and `forward_branches(fp32)` /
`forward_tree(fp32)` reproduce transformers' `Gemma4ForCausalLM` in FP32 on the same random-init weights.
"""
import math

import numpy as np
import torch

PREFIX = 'model.language_model.'
BF = torch.bfloat16
QUERY_BLOCK = 1024  # query rows per dense score block in `tree_attention`


def _r(x, bf16):
    """Round to BF16 (and back to FP32) in the BF16 path; identity in the FP32 path."""
    return x.to(BF).float() if bf16 else x


def rmsnorm(x, w, eps):
    """x * rsqrt(mean(x^2) + eps) * w in FP32 (plain weights; reference `lean_core.py:254,297`)."""
    x = x.float()
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * (w.float() if w is not None else 1.0)


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


def rope_tables(positions, inv_freq):
    """cos/sin of positions * inv_freq in FP32 (reference `lean_core.py:636-640`)."""
    pos = torch.as_tensor(np.asarray(positions), dtype=torch.float32, device=inv_freq.device)
    f = pos[:, None] * inv_freq[None, :]
    return f.cos(), f.sin()


def inv_freqs(cfg):
    """RoPE inverse frequencies per layer kind (reference `lean_core.py:386-394`)."""
    rp = cfg['rope_parameters']
    d = cfg['head_dim']
    out = {'sliding_attention': 1.0 / (rp['sliding_attention']['rope_theta'] ** (
        torch.arange(0, d, 2, dtype=torch.int64).float() / d))}
    gd = cfg['global_head_dim']
    angles = int(rp['full_attention'].get('partial_rotary_factor', 1.0) * gd // 2)
    rot = 1.0 / (rp['full_attention']['rope_theta'] ** (torch.arange(0, 2 * angles, 2, dtype=torch.int64).float() / gd))
    out['full_attention'] = torch.cat([rot, torch.zeros(gd // 2 - angles)])
    return out


def qkv_post(qkv, hq, hk, has_v, d, q_norm, k_norm, cos, sin, eps, bf16=True):
    """Per head: RMSNorm (q, k weighted; v unweighted), rounding, rotate-half RoPE on q and k
    (reference `_qkv_post`, `lean_core.py:234-277`). Returns q [n,hq,d], k [n,hk,d], v [n,hk,d] (FP32 values)."""
    n = qkv.shape[0]
    x = qkv.float()
    half = d // 2
    q = x[:, :hq * d].reshape(n, hq, d)
    k = x[:, hq * d:(hq + hk) * d].reshape(n, hk, d)
    v = (x[:, (hq + hk) * d:(hq + 2 * hk) * d] if has_v else x[:, hq * d:(hq + hk) * d]).reshape(n, hk, d)

    def norm_rope(t, w, rope):
        y = _r(rmsnorm(t, w, eps), bf16)
        if not rope:
            return y
        y1, y2 = y[..., :half], y[..., half:]
        c, s = cos[:, None, :], sin[:, None, :]
        return _r(torch.cat([y1 * c - y2 * s, y2 * c + y1 * s], -1), bf16)
    return norm_rope(q, q_norm, True), norm_rope(k, k_norm, True), norm_rope(v, None, False)


def segment_mask(q_len, kv_len, window, bidir, device=None):
    """[q_len, kv_len] visibility of a segment's keys (bottom-right aligned): causal, with the sliding window when
    window > 0; an image block (bidir) drops the causal bound and keeps its own block plus the window before each
    query (reference `lean_core.py:612-629` with FlashInfer's mask rules)."""
    j = torch.arange(q_len, device=device)[:, None]
    t = torch.arange(kv_len, device=device)[None, :]
    diag = kv_len - q_len
    if bidir:
        lo = diag + torch.clamp(j - (window - 1), max=0) if window > 0 else torch.zeros_like(j)
        return (t >= lo).expand(q_len, kv_len)
    hi = diag + j
    m = t <= hi
    if window > 0:
        m &= t >= hi - (window - 1)
    return m


def tree_attention(q, k_pool, v_pool, qo_indptr, kv_indptr, kv_indices, n_bidir, window, sm_scale, page_size=1,
                   kv_last_page_len=None):
    """Dense statement of the paged prefill attention over a tree plan. q [n, hq, d]; pools [slots, hk, d]. FP32."""
    n, hq, d = q.shape
    hk = k_pool.shape[1]
    G = hq // hk
    out = torch.zeros(n, hq, d, dtype=torch.float32, device=q.device)
    qo = np.asarray(qo_indptr)
    kp = np.asarray(kv_indptr)
    ki = np.asarray(kv_indices)
    for s in range(len(qo) - 1):
        q0, q1 = int(qo[s]), int(qo[s + 1])
        if q1 == q0:
            continue
        pages = ki[kp[s]:kp[s + 1]]
        if page_size == 1:
            slots = pages
        else:
            last = page_size if kv_last_page_len is None else int(kv_last_page_len[s])
            slots = np.concatenate([p * page_size + np.arange(page_size if i < len(pages) - 1 else last)
                                    for i, p in enumerate(pages)])
        idx = torch.as_tensor(np.asarray(slots, dtype=np.int64), device=k_pool.device)
        K = k_pool[idx].float()
        V = v_pool[idx].float()
        mask = segment_mask(q1 - q0, len(slots), window, s < n_bidir, q.device)
        Kg = K.repeat_interleave(G, dim=1)
        Vg = V.repeat_interleave(G, dim=1)
        # query blocks bound the score matrix (an 8,192-token segment would need hq x 8192^2 FP32 at once); each
        # query row's softmax is over its own keys, so blocking changes nothing
        for b0 in range(0, q1 - q0, QUERY_BLOCK):
            b1 = min(q1 - q0, b0 + QUERY_BLOCK)
            S = torch.einsum('qhd,khd->hqk', q[q0 + b0:q0 + b1].float(), Kg) * sm_scale
            S = S.masked_fill(~mask[None, b0:b1], float('-inf'))
            out[q0 + b0:q0 + b1] = torch.einsum('hqk,khd->qhd', torch.softmax(S, -1), Vg)
    return out


def attn_epilogue(o, x, w_post, w_pre, eps, bf16=True):
    """x' = x + rms(o) * w_post; h = rms(x') * w_pre (reference `_attn_epilogue`, `lean_core.py:290-302`)."""
    on = _r(rmsnorm(o, w_post, eps), bf16)
    xn = _r(x.float() + on, bf16)
    return xn, _r(rmsnorm(xn, w_pre, eps), bf16)


def mlp_epilogue(dn, x, w_post, scalar, w_next, eps, bf16=True):
    """x' = (x + rms(d) * w_post) * scalar; h = rms(x') * w_next (reference `_mlp_epilogue`, `lean_core.py:305-320`)."""
    dd = _r(rmsnorm(dn, w_post, eps), bf16)
    xa = _r(x.float() + dd, bf16)
    xs = _r(xa * scalar.float(), bf16)
    return xs, (_r(rmsnorm(xs, w_next, eps), bf16) if w_next is not None else None)


def geglu(gu, bf16=True):
    """gelu_tanh(gate) * up over [gate | up] halves (FlashInfer `gelu_tanh_and_mul`, `lean_core.py:685`)."""
    F = gu.shape[-1] // 2
    g = gu.float()
    return _r(gelu_tanh(g[..., :F]) * g[..., F:], bf16)


def matmul(a, w, bf16=True):
    """a @ w^T: BF16 inputs with FP32 accumulation rounded to BF16 (the cuBLAS call), or FP32."""
    if bf16:
        return (a.to(BF) @ w.to(BF).T).float()
    return a.float() @ w.float().T


def label_probs(rows, norm_w, embed, labels, softcap, eps, bf16=True):
    """Final norm, label-row logits in FP32, softcap, softmax per sequence (reference `lean_core.py:558-561,692`)."""
    out = []
    for r, ids in zip(rows, labels):
        normed = _r(rmsnorm(r[None], norm_w, eps), bf16)[0]
        logits = normed.float() @ embed[torch.as_tensor(ids, device=embed.device)].float().T
        logits = softcap * torch.tanh(logits / softcap)
        out.append(torch.softmax(logits, -1).double().tolist())
    return out


def layer_from_state(g, i, kind):
    """Layer i's weights in the reference's fused load layout (`lean_core.py:368-382`): `qkv` = [q; k(; v)], `gu` =
    [gate; up], the layer scalar in BF16. `g(key)` returns a checkpoint tensor."""
    p = f'{PREFIX}layers.{i}.'
    a = p + 'self_attn.'
    parts = [g(a + 'q_proj.weight'), g(a + 'k_proj.weight')]
    if kind == 'sliding_attention':
        parts.append(g(a + 'v_proj.weight'))
    return dict(
        kind=kind, qkv=torch.cat(parts, 0), o=g(a + 'o_proj.weight'),
        gu=torch.cat([g(p + 'mlp.gate_proj.weight'), g(p + 'mlp.up_proj.weight')], 0),
        down=g(p + 'mlp.down_proj.weight'), q_norm=g(a + 'q_norm.weight'), k_norm=g(a + 'k_norm.weight'),
        in_ln=g(p + 'input_layernorm.weight'), post_attn=g(p + 'post_attention_layernorm.weight'),
        pre_ff=g(p + 'pre_feedforward_layernorm.weight'), post_ff=g(p + 'post_feedforward_layernorm.weight'),
        scalar=g(p + 'layer_scalar').to(BF))


class StreamedLayers:
    """A read-only list of layers fetched on demand, keeping only the two most recently used (a layer reads its own
    weights and the next layer's input norm)."""

    def __init__(self, n, fetch):
        self.n, self.fetch, self.cache = n, fetch, {}

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        if i < 0:
            i += self.n
        if not 0 <= i < self.n:
            raise IndexError(i)
        if i not in self.cache:
            if len(self.cache) >= 2:
                del self.cache[max(self.cache, key=lambda j: abs(j - i))]  # the farthest from i
            self.cache[i] = self.fetch(i)
        return self.cache[i]


class OracleModel:
    """The decoder's weights from a state dict in the checkpoint key layout (`model.language_model.*`), on `device`
    (the CPU by default; the same torch code runs on a CUDA device for full-size checks, where it goes through torch's
    own library kernels, never this repository's)."""

    def __init__(self, top, state, device='cpu'):
        cfg = top['text_config']
        self.top, self.cfg = top, cfg
        self.H, self.eps, self.softcap = cfg['hidden_size'], cfg['rms_norm_eps'], cfg['final_logit_softcapping']
        self.hq, self.window, self.types = cfg['num_attention_heads'], cfg['sliding_window'], cfg['layer_types']
        self.geom = {'sliding_attention': (cfg['num_key_value_heads'], cfg['head_dim']),
                     'full_attention': (cfg['num_global_key_value_heads'], cfg['global_head_dim'])}
        self.image_id = top.get('image_token_id')
        self.device = torch.device(device)
        if state is None:  # `streamed`: the caller sets embed, norm and layers
            self.embed = self.norm = self.layers = None
        else:
            g = lambda k: state[k].to(self.device)
            self.embed, self.norm = g(PREFIX + 'embed_tokens.weight'), g(PREFIX + 'norm.weight')
            self.layers = [layer_from_state(g, i, kind) for i, kind in enumerate(self.types)]
        self.inv = {k: v.to(self.device) for k, v in inv_freqs(cfg).items()}
        # tensor-parallel check only: sums a row-parallel projection's partial output over ranks (None: one device)
        self.reduce = None

    @classmethod
    def streamed(cls, top, embed, norm, fetch, device='cpu'):
        """An oracle whose layers are fetched one at a time (`fetch(i)` -> the layer dict `layer_from_state` builds,
        CPU tensors) and dropped after use: host memory holds the embedding and two layers, so a 60-layer 31B-class
        forward fits in a few GB."""
        self = cls(top, None, device)
        self.embed, self.norm = embed.to(self.device), norm.to(self.device)
        self.layers = StreamedLayers(len(self.types), lambda i: {k: (v.to(self.device) if torch.is_tensor(v) else v)
                                                                 for k, v in fetch(i).items()})
        return self

    def embed_rows(self, tokens, feature_rows=None, features=None, bf16=True):
        """embed[tok] * bf16(sqrt(H)) in BF16 (reference `lean_core.py:366,641`), or * sqrt(H) in FP32; image rows
        take their feature rows (reference `lean_core.py:642-650`)."""
        scale = float(torch.tensor(self.H ** 0.5, dtype=BF)) if bf16 else self.H ** 0.5
        x = _r(self.embed[torch.as_tensor(np.asarray(tokens), dtype=torch.int64, device=self.device)].float() * scale,
               bf16)
        if feature_rows is not None:
            fr = np.asarray(feature_rows)
            rows = np.flatnonzero(fr >= 0)
            if len(rows):
                x[torch.as_tensor(rows, device=self.device)] = features.to(self.device)[
                    torch.as_tensor(fr[rows], device=self.device)].float()
        return x

    def layer(self, i, x, h, st, cap, rope, pools=None, precision='bf16'):
        """One decoder layer over a planned step (reference `lean_core.py:655-689`); returns (x, h, attention out)."""
        bf16 = precision == 'bf16'
        eps, hq = self.eps, self.hq
        layer = self.layers[i]
        kind = layer['kind']
        hk, d = self.geom[kind]
        kk = 's' if kind == 'sliding_attention' else 'g'
        has_v = kind == 'sliding_attention'
        n = x.shape[0]
        if pools is not None and pools[i] is not None:
            k_pool, v_pool = pools[i]
        else:
            k_pool = torch.zeros(cap[kk], hk, d, device=self.device)
            v_pool = torch.zeros(cap[kk], hk, d, device=self.device)
            if pools is not None:
                pools[i] = (k_pool, v_pool)
        cos, sin = rope[kind]
        qkv = _r(matmul(h, layer['qkv'], bf16), bf16)
        q, k, v = qkv_post(qkv, hq, hk, has_v, d, layer['q_norm'], layer['k_norm'], cos, sin, eps, bf16)
        sl = torch.as_tensor(np.asarray(st['slots'][kk], dtype=np.int64), device=self.device)
        k_pool[sl] = k
        v_pool[sl] = v
        window = self.window if kind == 'sliding_attention' else 0
        nb = int(st['n_bidir']) if kind == 'sliding_attention' else 0
        attn = tree_attention(q, k_pool, v_pool, st['qo_indptr'], st['kv_indptr_' + kk], st['kv_indices_' + kk],
                              nb, window, 1.0)
        attn = _r(attn, bf16).reshape(n, hq * d)
        o = _r(matmul(attn, layer['o'], bf16), bf16)
        if self.reduce is not None:
            o = self.reduce(o)
        x, h2 = attn_epilogue(o, x, layer['post_attn'], layer['pre_ff'], eps, bf16)
        gu = _r(matmul(h2, layer['gu'], bf16), bf16)
        act = geglu(gu, bf16)
        dn = _r(matmul(act, layer['down'], bf16), bf16)
        if self.reduce is not None:
            dn = self.reduce(dn)
        nxt = self.layers[i + 1]['in_ln'] if i + 1 < len(self.layers) else None
        x, h = mlp_epilogue(dn, x, layer['post_ff'], layer['scalar'], nxt, eps, bf16)
        return x, h, attn

    def forward_step(self, st, cap, readout_rows, pools=None, feature_rows=None, features=None, precision='bf16'):
        """One planned step through every layer; returns {row: final residual x of that readout row (FP32)}.
        `pools`: per layer (K, V) FP32 tensors [slots, hk, d] shared across steps (created when None entries)."""
        bf16 = precision == 'bf16'
        x = self.embed_rows(st['tokens'], feature_rows, features, bf16)
        h = _r(rmsnorm(x, self.layers[0]['in_ln'], self.eps), bf16)
        rope = {k: rope_tables(st['positions'], v) for k, v in self.inv.items()}
        for i in range(len(self.layers)):
            x, h, _ = self.layer(i, x, h, st, cap, rope, pools, precision)
        return {r: x[r].clone() for r in readout_rows}

    def forward_tree(self, tree_cls, seqs, label_ids, precision='bf16', single_max=16384, step_tokens=8192,
                     images=None, expand=None):
        """Plan one pass over every sequence with `tree_cls` (a planner bit-exact with the reference's) and run it;
        returns per-sequence label probabilities. `expand`: the engine's image layout (`ImageBlocks`: placeholder
        expansion, block bounds and splits, reference `lean_core.py:433-462`) when images are given."""
        bf16 = precision == 'bf16'
        splits, layout, feats = [], None, None
        seqs = [list(s) for s in seqs]
        if images:
            layout = expand(seqs, images, self.image_id, self.top['boi_token_id'], self.top['eoi_token_id'])
            seqs, splits = layout.seqs, layout.splits
            feats = torch.cat([f.float() for f in images])
        tree = tree_cls(seqs + splits)
        bidir = layout.bidir_nodes(tree) if layout else frozenset()
        idx = list(range(len(seqs)))
        need = tree.pass_nodes(idx, set())
        plan = tree.plan_pass(need, idx, self.window, single_max, step_tokens, False, bidir=bidir)
        pools = [None] * len(self.layers)
        finals = []
        for k, st in enumerate(plan['steps']):
            rows = sorted({r for kk, r in plan['readout'] if kk == k})
            fr = None
            if layout is not None:
                fr = np.full(len(st['tokens']), -1)
                im = np.flatnonzero(st['tokens'] == self.image_id)
                depth = st['positions'][im]
                kb = np.searchsorted(layout.start, depth, side='right') - 1
                fr[im] = layout.off[kb] + depth - layout.start[kb]
            finals.append(self.forward_step(st, plan['cap'], rows, pools if len(plan['steps']) > 1 else None, fr,
                                            feats, precision))
        rows = [finals[k][r] for k, r in plan['readout']]
        return label_probs(rows, self.norm, self.embed, label_ids, self.softcap, self.eps, bf16)

    def forward_branches(self, seqs, label_ids, precision='fp32'):
        """Each sequence as its own causal forward (text only); its last token's label distribution."""
        bf16 = precision == 'bf16'
        out = []
        for seq, ids in zip(seqs, label_ids):
            L = len(seq)
            ar = np.arange(L)
            st = dict(tokens=np.asarray(seq), positions=ar, n_bidir=0, qo_indptr=np.array([0, L]),
                      slots={'g': ar, 's': ar}, kv_indptr_g=np.array([0, L]), kv_indices_g=ar,
                      kv_indptr_s=np.array([0, L]), kv_indices_s=ar)
            x = self.forward_step(st, {'g': L, 's': L}, [L - 1], precision=precision)[L - 1]
            out.append(label_probs([x], self.norm, self.embed, [ids], self.softcap, self.eps, bf16)[0])
        return out
