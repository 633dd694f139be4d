"""The image path of a request on the B200 kernels: Gemma 4's vision tower and the projection of its soft tokens into the
text model's embedding space, in place of the reference's `VisionEncoder` (`aleria_judge/lean_core.py:745-781`),
which runs transformers' `Gemma4VisionModel` + `Gemma4MultimodalEmbedder` in BF16.

`VisionEncoder(model_dir, device='cuda', batch=2)` keeps the reference's interface: `encode(images, soft_tokens=None)`
returns one tensor (soft tokens x text hidden, BF16) per image, the image processor (transformers, on the host)
fixing each image's soft-token count. Everything after the processor runs on this library's kernels:

  pixels -> BF16 rescale to [-1, 1] (`morj_vision_patch_prologue`) -> patch projection (GEMM) -> + x and y position
  rows (`morj_vision_position_add`) -> per layer: input norm, QKV GEMM, per-head norm + 2-D rotary embedding
  (`morj_vision_head_epilogue`), attention (the tree attention kernel, each image one bidirectional segment over its
  real patches), O GEMM, post-attention residual + pre-MLP norm (`morj_attn_epilogue`), gate/up GEMM with the GeGLU
  epilogue, down GEMM, post-MLP residual + the next layer's input norm (`morj_mlp_epilogue`, layer scalar 1) ->
  average over each k x k cell of patches x sqrt(hidden) (`morj_vision_pool`) -> unweighted RMSNorm
  (`morj_rmsnorm_rows`) -> projection to the text hidden size (GEMM).

Unsupported checkpoint options are refused at load: clipped linears (`use_clipped_linears`) and feature
standardization (`standardize`).
"""
import numpy as np
import torch

from . import _native as nat
from .lean_core import _Tables, interleave_glu

TOWER = 'model.vision_tower.'
EMBED = 'model.embed_vision.'


def pool_cells(position_ids, length, k):
    """Host side of the pooler (transformers' `Gemma4VisionPooler._avg_pool_by_positions`): for one image's patch
    positions [P, 2] (-1 for padding), the cells of the k x k grid its pooled output keeps, in cell order, each with
    the patch rows (real patches only) it averages. A cell is kept when any patch, padding included (which sits in
    cell 0), falls in it; padding patches add nothing to the average. Returns (cell ids, CSR indptr, patch rows)."""
    pos = np.asarray(position_ids, dtype=np.int64)
    real = ~(pos == -1).all(-1)
    clamped = np.maximum(pos, 0)
    max_x = int(clamped[:, 0].max()) + 1 if len(pos) else 1
    cell = clamped[:, 0] // k + (max_x // k) * (clamped[:, 1] // k)
    if (cell >= length).any():
        raise ValueError(f'a patch position falls outside the {length} pooled cells')
    kept = np.unique(cell)
    rows = [np.flatnonzero((cell == c) & real) for c in kept]
    indptr = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int64)
    return kept, indptr, (np.concatenate(rows) if rows else np.zeros(0, np.int64))


class VisionTower:
    """Gemma 4's vision tower and multimodal embedder over this library's kernels, from a `vision_config` dict, the
    text hidden size and `get(key)` returning checkpoint tensors (keys `model.vision_tower.*`,
    `model.embed_vision.*`)."""

    def __init__(self, vcfg, text_hidden, get, device='cuda'):
        if vcfg.get('use_clipped_linears'):
            raise ValueError('unsupported vision checkpoint: clipped linears')
        if vcfg.get('standardize'):
            raise ValueError('unsupported vision checkpoint: feature standardization')
        self.device = torch.device(device)
        if self.device.type == 'cuda' and self.device.index is None:
            self.device = torch.device('cuda', torch.cuda.current_device())
        self.H = vcfg['hidden_size']
        self.heads = vcfg['num_attention_heads']
        self.d = vcfg.get('head_dim') or self.H // self.heads
        if vcfg.get('num_key_value_heads', self.heads) != self.heads:
            raise ValueError('unsupported vision checkpoint: grouped K/V heads')
        self.eps = vcfg['rms_norm_eps']
        self.k = vcfg['pooling_kernel_size']
        self.text_hidden = text_hidden
        theta = vcfg.get('rope_parameters', {}).get('rope_theta', 100.0)
        spatial = self.d // 2  # each spatial dimension rotates half of the head dims
        self.inv_freq = (1.0 / (theta ** (torch.arange(0, spatial, 2, dtype=torch.int64).float() / spatial))).to(
            self.device)
        bf = torch.bfloat16
        g = lambda k: get(k).to(self.device, bf).contiguous()
        self.proj_in = g(TOWER + 'patch_embedder.input_proj.weight')
        self.pos_table = g(TOWER + 'patch_embedder.position_embedding_table')
        self.layers = []
        for i in range(vcfg['num_hidden_layers']):
            p = f'{TOWER}encoder.layers.{i}.'
            a = p + 'self_attn.'
            qkv = torch.cat([g(a + f'{n}_proj.linear.weight') for n in 'qkv']).contiguous()
            gu = interleave_glu(g(p + 'mlp.gate_proj.linear.weight'), g(p + 'mlp.up_proj.linear.weight'))
            self.layers.append(dict(
                qkv=qkv, o=g(a + 'o_proj.linear.weight'), gu=gu.contiguous(), down=g(p + 'mlp.down_proj.linear.weight'),
                q_norm=g(a + 'q_norm.weight'), k_norm=g(a + 'k_norm.weight'), in_ln=g(p + 'input_layernorm.weight'),
                post_attn=g(p + 'post_attention_layernorm.weight'),
                pre_ff=g(p + 'pre_feedforward_layernorm.weight'),
                post_ff=g(p + 'post_feedforward_layernorm.weight')))
        self.proj_out = g(EMBED + 'embedding_projection.weight')
        self.one = torch.ones(1, dtype=bf, device=self.device)  # the residual's layer scalar (none in the tower)
        self.scale = float(self.H ** 0.5)

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def _gemm(self, a, w, out, epi=nat.EPI_STORE):
        nat.call('morj_gemm_bf16', a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                 out.stride(0), a.shape[0], w.shape[0], a.shape[1], epi, self._stream())

    @torch.inference_mode()
    def forward(self, pixel_values, position_ids):
        """Soft tokens in the text embedding space, [kept cells of every image in order, text hidden] BF16, for a
        processed batch: `pixel_values` [B, P, 3 x patch^2] in [0, 1] (padding rows anything), `position_ids`
        [B, P, 2] patch (x, y), -1 for padding. Also returns the number of soft tokens per image."""
        B, P, C = pixel_values.shape
        n = B * P
        H, d, heads, s = self.H, self.d, self.heads, self._stream()
        dev, bf = self.device, torch.bfloat16
        length = P // (self.k * self.k)
        pos_host = np.asarray(position_ids.cpu() if torch.is_tensor(position_ids) else position_ids, np.int64)
        # host tables: positions, the attention segments (one per image: every patch queries the image's real
        # patches), the pooled cells
        t = _Tables(dev)
        t.add('pos', pos_host.reshape(n, 2))
        real = [np.flatnonzero(~(pos_host[b] == -1).all(-1)) + b * P for b in range(B)]
        t.add('qo', np.arange(B + 1) * P)
        t.add('kv_indptr', np.concatenate([[0], np.cumsum([len(r) for r in real])]))
        t.add('kv_indices', np.concatenate(real) if real else np.zeros(0, np.int64))
        work = nat.attention_work(np.arange(B + 1) * P, np.concatenate([[0], np.cumsum([len(r) for r in real])]),
                                  B, heads, heads, 0)
        t.add('work', work)
        cell_indptr, cell_rows, counts = [0], [], []
        for b in range(B):
            kept, indptr, prow = pool_cells(pos_host[b], length, self.k)
            counts.append(len(kept))
            cell_indptr += (indptr[1:] + cell_indptr[-1]).tolist()
            cell_rows.append(prow + b * P)
        t.add('cell_indptr', cell_indptr)
        t.add('cell_rows', np.concatenate(cell_rows))
        t.upload()
        # patch embedding
        x = pixel_values.reshape(n, C).to(dev, bf).contiguous()
        nat.call('morj_vision_patch_prologue', x.data_ptr(), x.numel(), s)
        h0 = torch.empty(n, H, dtype=bf, device=dev)
        self._gemm(x, self.proj_in, h0)
        nat.call('morj_vision_position_add', h0.data_ptr(), t.ptr('pos'), self.pos_table.data_ptr(),
                 self.pos_table.shape[1], n, H, s)
        x = h0
        h = torch.empty(n, H, dtype=bf, device=dev)
        nat.call('morj_rmsnorm_rows', x.data_ptr(), self.layers[0]['in_ln'].data_ptr(), n, H, self.eps, h.data_ptr(),
                 s)
        qkv = torch.empty(n, 3 * heads * d, dtype=bf, device=dev)
        q = torch.empty(n, heads, d, dtype=bf, device=dev)
        kp = torch.empty(n, heads, d, dtype=bf, device=dev)
        vp = torch.empty(n, heads, d, dtype=bf, device=dev)
        attn = torch.empty(n, heads * d, dtype=bf, device=dev)
        o = torch.empty(n, H, dtype=bf, device=dev)
        act = torch.empty(n, self.layers[0]['gu'].shape[0] // 2, dtype=bf, device=dev)
        last = len(self.layers) - 1
        for i, L in enumerate(self.layers):
            self._gemm(h, L['qkv'], qkv)
            nat.call('morj_vision_head_epilogue', qkv.data_ptr(), qkv.stride(0), n, heads, d, L['q_norm'].data_ptr(),
                     L['k_norm'].data_ptr(), t.ptr('pos'), self.inv_freq.data_ptr(), self.eps, q.data_ptr(),
                     kp.data_ptr(), vp.data_ptr(), s)
            nat.call('morj_tree_attention', q.data_ptr(), n, kp.data_ptr(), vp.data_ptr(), n, attn.data_ptr(),
                     t.ptr('qo'), t.ptr('kv_indptr'), t.ptr('kv_indices'), None, B, B, heads, heads, d, 1, 0, 1.0,
                     t.ptr('work'), len(work) // 2, s)
            self._gemm(attn, L['o'], o)
            nat.call('morj_attn_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), L['post_attn'].data_ptr(),
                     L['pre_ff'].data_ptr(), n, H, self.eps, s)
            self._gemm(h, L['gu'], act, nat.EPI_GEGLU)
            self._gemm(act, L['down'], o)
            nxt = self.layers[i + 1]['in_ln'] if i < last else L['in_ln']
            nat.call('morj_mlp_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), L['post_ff'].data_ptr(),
                     self.one.data_ptr(), nxt.data_ptr(), n, H, self.eps, int(i < last), s)
        # pooling, the embedder's unweighted norm and projection
        n_cells = len(cell_indptr) - 1
        pooled = torch.empty(n_cells, H, dtype=bf, device=dev)
        nat.call('morj_vision_pool', x.data_ptr(), H, t.ptr('cell_indptr'), t.ptr('cell_rows'), n_cells,
                 1.0 / (self.k * self.k), self.scale, pooled.data_ptr(), s)
        normed = torch.empty_like(pooled)
        nat.call('morj_rmsnorm_rows', pooled.data_ptr(), None, n_cells, H, self.eps, normed.data_ptr(), s)
        out = torch.empty(n_cells, self.text_hidden, dtype=bf, device=dev)
        self._gemm(normed, self.proj_out, out)
        code = nat.device_error(s)
        if code:
            raise nat.NativeFailure(f'a kernel reported device error 0x{code:x}')
        return out, counts


class VisionEncoder:
    """Drop-in for the reference's `VisionEncoder` (`lean_core.py:745-781`): the checkpoint's image processor on the
    host, then `VisionTower` on the GPU; `encode` returns one tensor (soft tokens x text hidden) per image."""

    def __init__(self, model_dir, device='cuda', batch=2):
        from transformers import AutoProcessor
        from .checkpoint import open_checkpoint
        top, get = open_checkpoint(model_dir, 'cpu')
        self.processor = AutoProcessor.from_pretrained(model_dir).image_processor
        self.tower = VisionTower(top['vision_config'], top['text_config']['hidden_size'], get, device)
        self.device, self.batch = self.tower.device, batch

    @classmethod
    def from_parts(cls, processor, tower, batch=2):
        self = cls.__new__(cls)
        self.processor, self.tower, self.device, self.batch = processor, tower, tower.device, batch
        return self

    def encode(self, images, soft_tokens=None):
        out = []
        kw = {'max_soft_tokens': soft_tokens} if soft_tokens else {}
        for i in range(0, len(images), self.batch):  # a few images per call bounds the activations
            p = self.processor(list(images[i:i + self.batch]), return_tensors='pt', **kw)
            feats, counts = self.tower.forward(p['pixel_values'], p['image_position_ids'])
            want = p['num_soft_tokens_per_image'].tolist()
            if counts != want:
                raise ValueError(f'pooled soft tokens {counts} differ from the processor\'s {want}')
            out += list(torch.split(feats, counts))
        return out
