"""B200-native tree-prefill engine: a drop-in for the reference lean engine's model (`ENGINE=lean`).

`LeanGemma4` keeps the interface `aleria_judge/lean_engine.py` drives (reference `aleria_judge/lean_core.py:339-742`):
the constructor arguments, `free_bytes`, `kv_bytes`, `act_bytes`, `last_need`, `timing`, `gpu_ms`, `enqueued`,
`set_shared_prefix`, `prepare`, `run`, `forward_tree`, and `Request` with its `tree`, `retain`, `pinned`, `pools`,
`computed`, `read`, `tables`. `run` returns, per requested sequence in order, the softmax over that sequence's label
ids (the `method.py` contract). The host planner (`morj_b200.tree`) is bit-exact with the reference's; every device
operation of the forward is a hand-written sm_100a kernel reached through the C-ABI library (`morj_b200._native`):
no cuBLAS, FlashInfer or Triton, and no CPU fallback.

Forward per step (one pass may need several steps; see `Tree.plan_pass`):
  embed + input norm -> per layer: QKV GEMM with head norm + RoPE + pool scatter fused -> tree attention -> O GEMM ->
  residual + norms -> gate/up GEMM with GeGLU epilogue -> down GEMM -> residual * scalar + next input norm;
  the last layer computes K/V for every token and the rest only for readout rows; the label head reads them.
Numerics follow the reference path: FP32 norms and softmax, BF16 rounding where it rounds, attention scale 1.0,
V = K projection on full-attention layers, proportional partial RoPE there, BF16 embedding scale.
"""
import os
import time

import numpy as np
import torch

from . import _native as nat
from .checkpoint import PREFIX, iter_random_state, layer_geometry, open_checkpoint
from .tree import Tree

# Test only (JUDGE_LEAN_POISON=1): new K/V pools are filled with NaN, so a read of a slot no pass wrote shows up
# as NaN probabilities (reference `lean_core.py:29-31`).
POISON = os.environ.get('JUDGE_LEAN_POISON') == '1'

KINDS = {'sliding_attention': 's', 'full_attention': 'g'}
GLU_BLOCK = 128  # gate/up rows are interleaved in blocks of this many rows for the fused GeGLU epilogue
MAX_LABELS = 8192  # labels per sequence the label-head kernel holds in shared memory


class Request:
    """State of one scoring request across its passes. The attribute names are the ones `LeanEngine` and its stats
    read (reference `lean_core.py:323-336`): `tree`, `label_ids` (per tree sequence; shape-only sequences get a dummy
    label), `retain` (whole K/V kept for later passes), `pinned` (only the K/V later passes read kept), `head_nodes`
    (nodes filled from the shared head, never computed), `computed` (nodes whose K/V are in the pools), `read`
    (sequences already scored), `tables` (pinned mode: per kind, tree offset -> pool slot, -1 where dropped), `pools`
    (per layer (K, V) while kept), `n_real` (the caller's sequences come first in the tree), `features` and
    `bidir` (image blocks)."""

    def __init__(self, tree, label_ids, retain, head_nodes, pinned=False):
        self.tree, self.label_ids = tree, label_ids
        self.retain, self.pinned = retain, pinned
        self.head_nodes = head_nodes
        self.computed = set(head_nodes)
        self.read = set()
        self.tables = self.pools = self.features = None
        self.n_real = len(tree.seqs)
        self.bidir = frozenset()
        self.blocks = None


class ImageBlocks:
    """Where a request's images sit. Every image placeholder token becomes BOI, one image token per soft token, EOI
    (the layout of reference `lean_core.py:433-444,471-484`); the blocks must lie in the prefix every sequence shares.

    `seqs`: the expanded sequences; `splits`: prefixes of the first sequence ending at each block's first and last
    token, which give every block its own tree nodes; `start`, `end`: each block's depth range; `off`: each block's
    first row in the concatenated features."""

    def __init__(self, seqs, images, image_id, boi_id, eoi_id):
        sizes = np.asarray([len(f) for f in images], dtype=np.int64)
        self.seqs = []
        for seq in seqs:
            arr = np.asarray(seq, dtype=np.int64)
            marks = np.flatnonzero(arr == image_id)
            if len(marks) != len(sizes):
                raise ValueError(f'{len(sizes)} images but {len(marks)} image placeholders in a sequence')
            pieces = np.split(arr, marks + 1)  # each piece but the last ends with its placeholder
            out = []
            for piece, n in zip(pieces, sizes):
                out += piece[:-1].tolist() + [boi_id] + [image_id] * int(n) + [eoi_id]
            out += pieces[-1].tolist()
            self.seqs.append(out)
        marks0 = np.flatnonzero(np.asarray(seqs[0]) == image_id)
        # block k starts after its BOI; every earlier placeholder grew by its soft tokens + 1 (BOI and EOI replace it)
        self.start = marks0 + 1 + np.concatenate([[0], np.cumsum(sizes + 1)[:-1]]).astype(np.int64)
        self.end = self.start + sizes
        self.off = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
        last = int(self.end[-1])
        first = self.seqs[0]
        if any(len(x) <= last or x[:last] != first[:last] for x in self.seqs):
            raise ValueError('every branch must hold the same images in its shared prefix')
        self.splits = [first[:int(e)] for pair in zip(self.start, self.end) for e in pair]

    def bidir_nodes(self, tree):
        """Nodes of the shared prefix that lie inside one image block (attended without the causal mask in sliding
        layers)."""
        inside = lambda s, e: bool(np.any((self.start <= s) & (e <= self.end)))
        return frozenset(n for n in tree.paths[0] if inside(tree.nodes[n][1], tree.nodes[n][2]))

    def feature_rows(self, tokens, positions, image_id):
        """Per step token: its row in the concatenated image features, -1 for text tokens."""
        rows = np.full(len(tokens), -1, np.int64)
        img = np.flatnonzero(np.asarray(tokens) == image_id)
        if len(img):
            depth = np.asarray(positions)[img]
            k = np.searchsorted(self.start, depth, side='right') - 1
            if (k < 0).any() or (depth >= self.end[k]).any():
                raise ValueError('image placeholder outside an image block')
            rows[img] = self.off[k] + depth - self.start[k]
        return rows


def expand_images(seqs, images, image_id, boi_id, eoi_id):
    """The image layout of a request (see `ImageBlocks`)."""
    return ImageBlocks(seqs, images, image_id, boi_id, eoi_id)


def interleave_glu(gate, up, block=GLU_BLOCK):
    """[gate; up] rows reordered as (gate block 0, up block 0, gate block 1, ...) for the GeGLU GEMM epilogue."""
    F, H = gate.shape
    if F % block:
        raise ValueError('intermediate size must be a multiple of 128')
    return torch.stack([gate.reshape(F // block, block, H), up.reshape(F // block, block, H)], 1).reshape(2 * F, H)


def _ptr(t):
    return t.data_ptr() if t is not None else None


class _Tables:
    """Per-step int32 tables packed into one pinned host buffer and copied to the device in one transfer."""

    def __init__(self, device):
        self.parts, self.offset, self.device = [], 0, device
        self.views = {}

    def add(self, name, arr):
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.int32).reshape(-1))
        self.views[name] = (self.offset, len(a))
        self.parts.append(a)
        pad = (-len(a)) % 4  # keep every table 16-byte aligned
        if pad:
            self.parts.append(np.zeros(pad, np.int32))
        self.offset += len(a) + pad
        return name

    def upload(self):
        host = torch.from_numpy(np.concatenate(self.parts) if self.parts else np.zeros(4, np.int32)).pin_memory()
        self.dev = host.to(self.device, non_blocking=True)
        self.host = host  # kept alive until the copy has run
        self.nbytes = host.numel() * 4
        return self

    def __getitem__(self, name):
        o, n = self.views[name]
        return self.dev[o:o + n]

    def ptr(self, name):
        return self[name].data_ptr()


class LeanGemma4:
    def __init__(self, model_dir, device='cuda', workspace_mb=512, retain_budget_gb=10.0, single_max=16384,
                 step_tokens=8192, *, tp_group=None, tp_comm='peer'):
        """Load a safetensors checkpoint (`config.json["text_config"]` + `model.language_model.*` tensors) as the
        reference does (`lean_core.py:340-416`). `workspace_mb` is accepted for interface compatibility; the tree
        attention kernel needs no workspace. `tp_group`: a torch.distributed process group (NCCL) to shard the model
        over for tensor parallelism (`morj_b200.tp`); None runs the whole model on this GPU. `tp_comm`: 'peer'
        reduces the row-parallel projections over peer memory fused with their epilogues (`tp.PeerExchange`),
        'nccl' with an NCCL all-reduce followed by the replicated epilogues."""
        top, get = open_checkpoint(model_dir, device)
        self._setup(top, get, device, retain_budget_gb, single_max, step_tokens, tp_group, tp_comm)

    @classmethod
    def from_state(cls, top, state, device='cuda', retain_budget_gb=10.0, single_max=16384, step_tokens=8192,
                   tp_group=None, tp_comm='peer'):
        """An engine over an in-memory state dict in the checkpoint's key layout (tensors on any device)."""
        self = cls.__new__(cls)
        self._setup(top, lambda k: state[k].to(device), device, retain_budget_gb, single_max, step_tokens, tp_group,
                    tp_comm)
        return self

    @classmethod
    def random_init(cls, top, seed=0, device='cuda', std=0.02, norm_std=0.1, retain_budget_gb=10.0,
                    single_max=16384, step_tokens=8192, tp_group=None, tp_comm='peer'):
        """An engine over seeded random-init weights generated on `device` (no checkpoint on disk); tensors are drawn
        in checkpoint order and handed over one at a time, so the peak memory is the model plus one layer."""
        gen = iter_random_state(top, seed=seed, std=std, norm_std=norm_std, device=device)
        cache = {}

        def get(key):
            while key not in cache:
                k, t = next(gen)
                cache[k] = t
            return cache.pop(key)
        self = cls.__new__(cls)
        self._setup(top, get, device, retain_budget_gb, single_max, step_tokens, tp_group, tp_comm)
        return self

    def _setup(self, top, get, device, retain_budget_gb, single_max, step_tokens, tp_group=None, tp_comm='peer'):
        if tp_comm not in ('peer', 'nccl'):
            raise ValueError(f"tp_comm must be 'peer' or 'nccl', not {tp_comm!r}")
        self.tp_group, self.tp_world, self.tp_rank = tp_group, 1, 0
        self.peer = None
        if tp_group is not None:
            import torch.distributed as dist
            from .tp import shard_config, shard_getter
            self.tp_world, self.tp_rank = dist.get_world_size(tp_group), dist.get_rank(tp_group)
            get = shard_getter(top, get, self.tp_rank, self.tp_world)
            top = shard_config(top, self.tp_world)
        cfg = top['text_config']
        self.image_id, self.boi_id, self.eoi_id = (top.get('image_token_id'), top.get('boi_token_id'),
                                                   top.get('eoi_token_id'))
        self.cfg = cfg
        self.hidden = cfg['hidden_size']
        self.eps = cfg['rms_norm_eps']
        self.softcap = cfg['final_logit_softcapping']
        self.types = cfg['layer_types']
        self.window = cfg['sliding_window']
        self.hq = cfg['num_attention_heads']
        self.geom = {k: layer_geometry(cfg, k) for k in ('sliding_attention', 'full_attention')}
        if not (cfg['attention_k_eq_v'] and not cfg['enable_moe_block'] and not cfg['hidden_size_per_layer_input']):
            raise ValueError('unsupported checkpoint: needs attention_k_eq_v, no MoE block, no per-layer input')
        if not (cfg['num_kv_shared_layers'] == 0 and cfg['tie_word_embeddings']):
            raise ValueError('unsupported checkpoint: needs no shared K/V layers and tied embeddings')
        self.device = torch.device(device)
        if self.device.type == 'cuda' and self.device.index is None:
            self.device = torch.device('cuda', torch.cuda.current_device())
        self.embed = get(PREFIX + 'embed_tokens.weight').contiguous()
        self.norm = get(PREFIX + 'norm.weight').contiguous()
        # the reference rounds sqrt(hidden) to BF16 (`lean_core.py:366`)
        self.embed_scale = float(torch.tensor(self.hidden ** 0.5, dtype=torch.bfloat16))
        self.layers = []
        for i, kind in enumerate(self.types):
            p = f'{PREFIX}layers.{i}.'
            a = p + 'self_attn.'
            parts = [get(a + 'q_proj.weight'), get(a + 'k_proj.weight')]
            if kind == 'sliding_attention':
                parts.append(get(a + 'v_proj.weight'))
            qkv = torch.cat(parts, 0).contiguous()
            del parts
            gu = interleave_glu(get(p + 'mlp.gate_proj.weight'), get(p + 'mlp.up_proj.weight')).contiguous()
            self.layers.append(dict(
                kind=kind, qkv=qkv, o=get(a + 'o_proj.weight').contiguous(), gu=gu,
                down=get(p + 'mlp.down_proj.weight').contiguous(),
                q_norm=get(a + 'q_norm.weight').contiguous(), k_norm=get(a + 'k_norm.weight').contiguous(),
                in_ln=get(p + 'input_layernorm.weight').contiguous(),
                post_attn=get(p + 'post_attention_layernorm.weight').contiguous(),
                pre_ff=get(p + 'pre_feedforward_layernorm.weight').contiguous(),
                post_ff=get(p + 'post_feedforward_layernorm.weight').contiguous(),
                scalar=get(p + 'layer_scalar').to(torch.bfloat16).contiguous()))
        # RoPE inverse frequencies (default for sliding layers, proportional partial for full attention), FP32, as
        # the reference computes them (`lean_core.py:386-394`)
        rp = cfg['rope_parameters']
        d = cfg['head_dim']
        self.inv_freq = {'sliding_attention': (1.0 / (rp['sliding_attention']['rope_theta'] ** (
            torch.arange(0, d, 2, dtype=torch.int64).float() / d))).float().to(self.device)}
        gd = cfg['global_head_dim']
        angles = int(rp['full_attention'].get('partial_rotary_factor', 1.0) * gd // 2)
        rot = 1.0 / (rp['full_attention']['rope_theta'] ** (
            torch.arange(0, 2 * angles, 2, dtype=torch.int64).float() / gd))
        self.inv_freq['full_attention'] = torch.cat([rot, torch.zeros(gd // 2 - angles)]).float().to(self.device)
        # (cos, sin) of position x inv_freq, by position, per kind: the reference's per-step tables
        # (`lean_core.py:636-640`), built once and grown with the longest position seen (`_rope`)
        self.rope = {}
        self.prune_last = True
        self.kv_bytes = sum(2 * 2 * self.geom[k][0] * self.geom[k][1] for k in self.types)
        self.retain_budget = retain_budget_gb * 2**30
        self.shared, self.shared_kv = None, None
        self.single_max, self.step_tokens = single_max, step_tokens
        self.timing = {}
        self.gpu_ms = 0.0
        self.last_need = []
        self.h2d_bytes = 0
        self.launches = 0
        self.trace = None
        # split-tile workspace of the pair GEMM kernel, registered for every stream the model launches on
        self.gemm_ws = nat.GemmWorkspace(self.device) if self.device.type == 'cuda' else None
        if tp_group is not None and tp_comm == 'peer':
            from .tp import PeerExchange
            self.peer = PeerExchange(tp_group, self.hidden, max(single_max, step_tokens), self.device)
        self.free_bytes = (torch.cuda.mem_get_info(self.device)[0] - (3 << 30)) if self.device.type == 'cuda' else 0
        hd = max(dd for _, dd in self.geom.values())
        qkv_rows = max(l['qkv'].shape[0] for l in self.layers)
        # activation bytes per token of a step, by the reference's formula (`lean_core.py:414-416`; the largest
        # QKV width over all layers, which is the reference's layer 0 / layer 5 maximum on its 6-layer pattern)
        self.act_bytes = 2 * (4 * self.hidden + qkv_rows + 2 * self.hq * hd + 3 * self.layers[0]['gu'].shape[0] // 2)

    # ---- requests -------------------------------------------------------------------------------------------------
    def set_shared_prefix(self, tokens):
        """Compute a prefix that many requests start with once, and keep its K/V: every later request whose sequences
        all start with it gets the K/V copied into its head slots instead of computed (`lean_core.py:419-426`)."""
        self.shared = self.shared_kv = None
        req = self.prepare([list(tokens)], [[0]], retain=True)
        self.run(req, [0])
        offsets = np.concatenate([req.tree.slots(n) for n in req.tree.paths[0]]).astype(np.int32)
        idx = torch.as_tensor(offsets, device=self.device)
        kv = [(self._gather(k, idx), self._gather(v, idx)) for k, v in req.pools]
        torch.cuda.current_stream(self.device).synchronize()
        self.shared, self.shared_kv = np.asarray(tokens, dtype=np.int64), kv

    def _starts_with_shared(self, seqs):
        n = 0 if self.shared is None else len(self.shared)
        return bool(n) and bool(seqs) and all(len(x) > n and np.array_equal(x[:n], self.shared) for x in seqs)

    def _retention(self, tokens, retain, available):
        """(keep whole, keep pinned) for a request of `tokens` tree tokens. A retained request keeps all its K/V when
        they fit both the retention budget and the memory left after one step's activations; otherwise it keeps only
        what its later passes read (the reference's rule, `lean_core.py:451-454`, which the adapter's OOM ladder
        relies on)."""
        if not retain:
            return False, False
        room = (self.free_bytes if available is None else available) - min(tokens, self.single_max) * self.act_bytes
        whole = tokens * self.kv_bytes <= min(self.retain_budget, room)
        return whole, not whole

    def prepare(self, seqs, label_ids, retain=False, images=None, available=None):
        """A request over `seqs`, every sequence it may score (`lean_core.py:428-469`): image placeholders expanded,
        the tree (with extra shape-only sequences: image-block bounds, the shared head), the retention decision, and
        for a request kept whole its pools with the shared head's K/V in place."""
        seqs = [list(x) for x in seqs]
        blocks = ImageBlocks(seqs, images, self.image_id, self.boi_id, self.eoi_id) if images else None
        if blocks is not None:
            seqs = blocks.seqs
        shared = self._starts_with_shared(seqs)
        shape_only = (blocks.splits if blocks is not None else []) + ([self.shared] if shared else [])
        tree = Tree(seqs + shape_only)
        whole, pinned = self._retention(tree.num_tokens, retain, available)
        req = Request(tree, list(label_ids) + [[0]] * len(shape_only), whole, tree.paths[-1] if shared else [],
                      pinned=pinned)
        req.n_real = len(seqs)
        if blocks is not None:
            req.blocks = blocks
            req.features = torch.cat([f.to(self.device, torch.bfloat16) for f in images]).contiguous()
            req.bidir = blocks.bidir_nodes(tree)
        if whole:
            req.pools = [self._kv_pool(kind, tree.num_tokens) for kind in self.types]
            if shared:
                self._copy_head(req.pools, None, np.concatenate([tree.slots(n) for n in req.head_nodes]))
        return req

    def _kv_pool(self, kind, slots):
        """A (K, V) pair of `slots` rows for one layer of `kind`. With POISON (tests) every row starts as NaN."""
        hk, d = self.geom[kind]
        shape = (max(slots, 1), hk, d)
        if POISON:
            return tuple(torch.full(shape, float('nan'), dtype=torch.bfloat16, device=self.device) for _ in 'kv')
        return tuple(torch.empty(shape, dtype=torch.bfloat16, device=self.device) for _ in 'kv')

    def _gather(self, src, idx):
        """Rows `idx` of a pool, as a new tensor (native row copy)."""
        width = src[0].numel()
        out = torch.empty((len(idx),) + tuple(src.shape[1:]), dtype=src.dtype, device=self.device)
        self._k('rows', 'morj_gather_rows', src.data_ptr(), width, idx.data_ptr(), len(idx), width, out.data_ptr(),
                width, self._stream())
        return out

    def _copy_head(self, pools, slot_of, head, layers=None):
        """The shared head's K/V into the pools of `layers` (default every layer, `pools[j]` for layer `layers[j]`),
        at the head's slots: the tree offsets `head` mapped through `slot_of` (per kind; None when slots are tree
        offsets) (`lean_core.py:594-597`)."""
        for (k, v), i in zip(pools, layers if layers is not None else range(len(self.types))):
            slots = head if slot_of is None else slot_of[KINDS[self.types[i]]][head]
            idx = torch.as_tensor(np.asarray(slots, dtype=np.int32), device=self.device)
            width = k[0].numel()
            for dst, src in zip((k, v), self.shared_kv[i]):
                nat.call('morj_scatter_rows', src.data_ptr(), width, idx.data_ptr(), len(idx), width, dst.data_ptr(),
                         width, self._stream())

    def _grow(self, req, cap):
        """A pinned request's pools, enlarged to at least `cap` slots per kind when a pass needs more; the rows held so
        far move to the same slots of the new pools (`lean_core.py:578-592`)."""
        old = req.pools
        short = old is None or any(old[i][0].shape[0] < cap[KINDS[kind]] for i, kind in enumerate(self.types))
        if not short:
            return old
        new = [self._kv_pool(kind, cap[KINDS[kind]]) for kind in self.types]
        if old is not None:
            for (k, v), (ok, ov) in zip(new, old):
                n = min(ok.shape[0], k.shape[0])
                idx = torch.arange(n, dtype=torch.int32, device=self.device)
                width = k[0].numel()
                for dst, src in ((k, ok), (v, ov)):
                    nat.call('morj_gather_rows', src.data_ptr(), width, idx.data_ptr(), n, width, dst.data_ptr(),
                             width, self._stream())
        req.pools = new
        return new

    def _stream(self):
        s = torch.cuda.current_stream(self.device).cuda_stream
        if self.gemm_ws is not None:
            self.gemm_ws.register(s)
        return s

    # ---- pass -----------------------------------------------------------------------------------------------------
    def _pass_bytes(self, plan, persistent):
        """Device bytes a planned pass needs: its largest step's activations, plus every layer's pools when they live
        for the whole pass (pinned requests, and multi-step passes of requests not kept whole)."""
        largest = max(len(st['tokens']) for st in plan['steps'])
        pools = sum(plan['cap'][KINDS[t]] * 4 * self.geom[t][0] * self.geom[t][1] for t in self.types)
        return (pools if persistent else 0) + largest * self.act_bytes

    def plan(self, req, seqs, available=None):
        """The planning half of `run` (`lean_core.py:497-529`): the nodes to compute, the head's tree offsets, the
        pinned offsets, and a plan whose memory fits `available` (default `free_bytes`).

        Fitting: the whole pass as one step first; then in steps of `step_tokens` (so a pass's sliding-window slots
        are reused as it moves on); then steps halved down to 512 tokens, below which the request does not fit and
        MemoryError is raised (the adapter then frees memory and retries)."""
        tree = req.tree
        cached = req.computed if (req.retain or req.pinned) else set(req.head_nodes)
        need = tree.pass_nodes(seqs, cached)
        head = (np.concatenate([tree.slots(n) for n in req.head_nodes]) if req.head_nodes
                else np.zeros(0, np.int64))
        pinned = None
        if req.pinned:
            later = [b for b in range(req.n_real) if b not in req.read and b not in set(seqs)]
            pinned = tree.pinned_for(cached | set(need), later, self.window)
        budget = self.free_bytes if available is None else available
        single, step = self.single_max, self.step_tokens
        while True:
            plan = tree.plan_pass(need, seqs, self.window, single, step, req.retain,
                                  prealloc=() if req.retain else head, initial=req.tables, pinned=pinned,
                                  bidir=req.bidir)
            one_step = len(plan['steps']) == 1
            cost = self._pass_bytes(plan, req.pinned or (not one_step and not req.retain))
            if cost <= budget:
                return need, head, pinned, plan
            if step <= 512:
                raise MemoryError(f'the pass needs {cost / 2**30:.2f} GiB at 512-token steps; '
                                  f'{budget / 2**30:.2f} GiB available')
            if one_step and single:
                single = 0
            else:
                step //= 2

    def _pass_pools(self, req, plan, head):
        """The pools a pass writes: the request's own (kept whole, or pinned and grown as needed), fresh pools for
        every layer when a pass of several steps must keep K/V between its steps, or None when one step runs with a
        temporary pool per layer kind. New pools get the shared head's K/V."""
        if req.retain:
            return req.pools
        if req.pinned:
            pools, fresh = self._grow(req, plan['cap']), req.tables is None
        elif len(plan['steps']) > 1:
            pools, fresh = [self._kv_pool(kind, plan['cap'][KINDS[kind]]) for kind in self.types], True
        else:
            return None
        if fresh and len(head):
            self._copy_head(pools, plan['slot_of'], head)
        return pools

    def prepare_pass(self, req, seqs, available=None):
        """Host half of `run`: plan (with the memory fit), the pools the pass writes, and every step's tables uploaded
        to the device. The result can be executed any number of times (`execute_pass`); each execution recomputes
        the same nodes into the same slots."""
        t0 = time.perf_counter()
        need, head, pinned, plan = self.plan(req, seqs, available)
        pools = self._pass_pools(req, plan, head)
        labels = [req.label_ids[b] for b in seqs]
        if any(len(ids) > MAX_LABELS for ids in labels):
            raise ValueError(f'at most {MAX_LABELS} labels per sequence')
        self.h2d_bytes = 0
        tables = [self._step_tables(k, st, plan, req) for k, st in enumerate(plan['steps'])]
        ro = self._readout_tables(plan, labels)
        return dict(req=req, seqs=list(seqs), need=need, head=head, pinned=pinned, plan=plan, pools=pools,
                    labels=labels, tables=tables, ro=ro, host_ms=1000 * (time.perf_counter() - t0),
                    h2d_bytes=self.h2d_bytes, tokens=sum(len(st['tokens']) for st in plan['steps']))

    def execute_pass(self, p):
        """Device half of `run`: every step's forward and the label head; returns the FP32 probabilities (device,
        CSR over the requested sequences' labels). Launches only; nothing waits for the GPU."""
        plan = p['plan']
        if self.peer is not None:
            self.peer.begin_pass()
        reads = torch.empty(len(plan['readout']), self.hidden, dtype=torch.bfloat16, device=self.device)
        at = 0
        for k, st in enumerate(plan['steps']):
            n_rows = len(p['tables'][k][1])
            self._step(k, st, plan, p['pools'], p['head'], p['req'], p['tables'][k], reads[at:at + n_rows])
            at += n_rows
        return self._readout(reads[:at], p['ro'])

    def _finish_pass(self, req, p):
        """What a finished pass leaves in the request: the sequences read, the nodes whose K/V are now kept, and in
        pinned mode the slot of every kept offset for the next pass's plan (`lean_core.py:565-575`)."""
        req.read.update(p['seqs'])
        if req.retain or req.pinned:
            req.computed.update(p['need'])
        if req.pinned:
            n, plan, pinned = req.tree.num_tokens, p['plan'], p['pinned']
            req.tables = {}
            for kk in 'gs':
                table = np.full(n, -1)
                table[pinned[kk]] = plan['slot_of'][kk][pinned[kk]]
                req.tables[kk] = table

    @torch.inference_mode()
    def run(self, req, seqs, available=None):
        """Label probabilities of sequences `seqs` of `req`, computing only the nodes it has not kept yet
        (`lean_core.py:495-576`): one list per sequence, in order, each the softmax over that sequence's labels."""
        p = self.prepare_pass(req, seqs, available)
        self.last_need = p['need']
        self.timing = {'host_setup_ms': p['host_ms'], 'steps': len(p['plan']['steps']), 'tokens': p['tokens']}
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        probs = self.execute_pass(p)
        end.record()
        self.enqueued = time.perf_counter()  # every launch queued; the copy below waits for the GPU
        flat = probs.cpu().numpy()
        self.d2h_bytes = flat.nbytes
        code = nat.device_error(self._stream())
        if self.peer is not None:
            code = self.peer.end_pass(code)
        if code:
            raise nat.NativeFailure(f'a kernel reported device error 0x{code:x}')
        bounds = np.cumsum([0] + [len(ids) for ids in p['labels']])
        out = [flat[a:b].astype(np.float64).tolist() for a, b in zip(bounds[:-1], bounds[1:])]
        self.gpu_ms = self.timing['gpu_ms'] = start.elapsed_time(end)
        self._finish_pass(req, p)
        return out

    def _readout_tables(self, plan, labels):
        """Per requested sequence: its row among the readout rows of all steps (in step order) and its label CSR."""
        offset, pos = 0, {}
        for k in range(len(plan['steps'])):
            rows = sorted({r for kk, r in plan['readout'] if kk == k})
            for j, r in enumerate(rows):
                pos[(k, r)] = offset + j
            offset += len(rows)
        t = _Tables(self.device)
        t.add('seq_row', [pos[(k, r)] for k, r in plan['readout']])
        indptr = np.concatenate([[0], np.cumsum([len(ids) for ids in labels])])
        t.add('indptr', indptr)
        t.add('labels', np.concatenate([np.asarray(ids, dtype=np.int64) for ids in labels]))
        t.upload()
        self.h2d_bytes += t.nbytes
        return dict(t=t, n_seq=len(labels), n_labels=int(indptr[-1]))

    def _readout(self, reads, ro):
        """Final norm + label rows + softcap + per-sequence softmax in one kernel (`lean_core.py:558-561`) over the
        readout rows of every step (`reads`, in step order)."""
        H, t = self.hidden, ro['t']
        probs = torch.empty(ro['n_labels'], dtype=torch.float32, device=self.device)
        self._k('head', 'morj_label_head', reads.data_ptr(), H, t.ptr('seq_row'), t.ptr('indptr'), t.ptr('labels'),
                ro['n_seq'], self.norm.data_ptr(), self.embed.data_ptr(), H, self.eps, self.softcap,
                probs.data_ptr(), self._stream())
        return probs

    def _k(self, kind, name, *args, flops=0):
        """Launch one native kernel; with `trace` on, bracket it with CUDA events (for per-kernel timing)."""
        self.launches += 1
        if self.trace is None:
            nat.call(name, *args)
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        nat.call(name, *args)
        e1.record()
        self.trace.append((kind, flops, e0, e1))

    # ---- forward over one step ------------------------------------------------------------------------------------
    def _step_tables(self, k, st, plan, req):
        t = _Tables(self.device)
        n = len(st['tokens'])
        t.add('tokens', st['tokens'])
        t.add('positions', st['positions'])
        for kk in 'gs':
            t.add('slots_' + kk, st['slots'][kk])
            t.add('kv_indptr_' + kk, st['kv_indptr_' + kk])
            t.add('kv_indices_' + kk, st['kv_indices_' + kk])
        qo = np.asarray(st['qo_indptr'], dtype=np.int32)
        t.add('qo', qo)
        n_work = {}
        for kk, kind in (('s', 'sliding_attention'), ('g', 'full_attention')):
            sliding = kind == 'sliding_attention'
            w = nat.attention_work(qo, st['kv_indptr_' + kk], int(st['n_bidir']) if sliding else 0, self.hq,
                                   self.geom[kind][0], self.window if sliding else 0)
            t.add('work_' + kk, w)
            n_work[kk] = len(w) // 2
        if req.features is not None:
            t.add('feature_row', req.blocks.feature_rows(st['tokens'], st['positions'], self.image_id))
        # readout rows of this step and the last layer's tables for them: each row attends to its segment's path up
        # to and including itself (reference `lean_core.py:713-727`)
        rows = sorted({r for kk, r in plan['readout'] if kk == k})
        last_kind = KINDS[self.types[-1]]
        if rows:
            seg = np.searchsorted(st['qo_indptr'], rows, side='right') - 1
            ind, ptr = [], [0]
            for row, sg in zip(rows, seg):
                lo, hi = st['kv_indptr_' + last_kind][sg], st['kv_indptr_' + last_kind][sg + 1]
                back = st['qo_indptr'][sg + 1] - 1 - row
                ind.append(st['kv_indices_' + last_kind][lo:hi - back])
                ptr.append(ptr[-1] + len(ind[-1]))
            t.add('ro_rows', rows)
            t.add('ro_positions', st['positions'][rows])
            t.add('ro_qo', np.arange(len(rows) + 1))
            t.add('ro_kv_indptr', ptr)
            t.add('ro_kv_indices', np.concatenate(ind))
            last_sliding = self.types[-1] == 'sliding_attention'
            ro_work = nat.attention_work(np.arange(len(rows) + 1), ptr, 0, self.hq, self.geom[self.types[-1]][0],
                                         self.window if last_sliding else 0)
            t.add('ro_work', ro_work)
            n_work['ro'] = len(ro_work) // 2
        t.upload()
        self.h2d_bytes += t.nbytes
        return t, rows, n_work

    def _gemm(self, a, w, out, epi=nat.EPI_STORE, w_rows=None, w_offset_rows=0):
        M, K = a.shape
        N = w.shape[0] if w_rows is None else w_rows
        wp = w.data_ptr() + w_offset_rows * w.stride(0) * w.element_size()
        self._k('gemm_geglu' if epi == nat.EPI_GEGLU else 'gemm', 'morj_gemm_bf16', a.data_ptr(), a.stride(0), wp,
                w.stride(0), out.data_ptr(), out.stride(0), M, N, K, epi, self._stream(), flops=2 * M * N * K)

    def _peer_site(self, a, w, mode, n, w_a, scalar, w_b, has_next, push_x):
        """Tensor parallelism over peer memory: the row-parallel projection a . w^T delivers its partial tiles to the
        row blocks' owners, each owner reduces its rows with the post-attention (mode 0) or post-MLP (mode 1)
        epilogue and pushes the new h rows (x rows too when `push_x`) to every rank, then the stream waits for all
        of h (`morj_gemm_bf16_peer`, `morj_peer_reduce`, `morj_peer_wait`)."""
        import ctypes
        from .tp import partial_target, row_target
        ex, s = self.peer, self._stream()
        desc = ctypes.addressof(ex.desc)
        K, N = a.shape[1], w.shape[0]
        self._k('gemm', 'morj_gemm_bf16_peer', a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), n, N, K, desc,
                s, flops=2 * n * N * K)
        ex.sites += 1
        self._k('tp_reduce', 'morj_peer_reduce', desc, mode, n, w_a.data_ptr(), _ptr(scalar), _ptr(w_b), self.eps,
                has_next, push_x, partial_target(ex.sites, ex.world, self.hidden), s)
        self._k('tp_reduce', 'morj_peer_wait', desc, n, row_target(ex.sites), s)

    def _peer_rows(self, n):
        """The exchange's x and h rows for an n-row step; a larger step than the exchange holds rebuilds it on every
        rank (all ranks plan the same steps, so they rebuild together)."""
        if n > self.peer.max_rows:
            import torch.distributed as dist
            from .tp import PeerExchange
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.tp_group)
            self.peer.close()
            self.peer = PeerExchange(self.tp_group, self.hidden, n, self.device)
        return self.peer.rows_view('x', n), self.peer.rows_view('h', n)

    def _reduce(self, t):
        """Tensor parallelism: sum the row-parallel projection's partial output over the ranks (NCCL all-reduce on
        the current stream); nothing on one GPU."""
        if self.tp_world > 1:
            import torch.distributed as dist
            if self.trace is not None:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                dist.all_reduce(t, group=self.tp_group)
                e1.record()
                self.trace.append(('allreduce', 0, e0, e1))
            else:
                dist.all_reduce(t, group=self.tp_group)

    def _rope(self, kind, max_pos):
        """The RoPE table of `kind` covering positions 0..max_pos (grown to the next power of two, at least 4096)."""
        tab = self.rope.get(kind)
        if tab is None or tab.shape[0] <= max_pos:
            rows = max(4096, 1 << int(max_pos).bit_length())
            inv = self.inv_freq[kind]
            tab = torch.empty(rows, inv.numel(), 2, dtype=torch.float32, device=self.device)
            self._k('rows', 'morj_rope_table', inv.data_ptr(), inv.numel(), rows, tab.data_ptr(), self._stream())
            self.rope[kind] = tab
        return tab

    def _qkv(self, a, layer, row0, M, hq, hk, has_v, d, kind, positions, slots, q_out, k_pool, v_pool):
        """QKV projection with the fused head norm + RoPE + pool scatter (`morj_gemm_qkv_rope`); `row0` skips the q
        rows of the fused weight for the K/V-only call."""
        w = layer['qkv']
        H = a.shape[1]
        n_out = (hq + (2 if has_v else 1) * hk) * d
        flops = 2 * M * n_out * H
        wp = w.data_ptr() + row0 * w.stride(0) * w.element_size()
        rope = self.rope[kind]
        self._k('gemm_qkv', 'morj_gemm_qkv_rope', a.data_ptr(), a.stride(0), wp, w.stride(0), M, H, hq, hk, has_v,
                d, layer['q_norm'].data_ptr(), layer['k_norm'].data_ptr(), positions, rope.data_ptr(), rope.shape[0],
                slots, self.eps, _ptr(q_out), _ptr(k_pool), _ptr(v_pool), self._stream(), flops=flops)

    def _attention(self, q, k_pool, v_pool, out, t, qo, kv_indptr, kv_indices, n_seg, n_bidir, kind, work, n_work):
        hk, d = self.geom[kind]
        window = self.window if kind == 'sliding_attention' else 0
        self._k('attention', 'morj_tree_attention', q.data_ptr(), q.shape[0], k_pool.data_ptr(), v_pool.data_ptr(),
                k_pool.shape[0], out.data_ptr(), t.ptr(qo), t.ptr(kv_indptr), t.ptr(kv_indices), None, n_seg, n_bidir,
                self.hq, hk, d, 1, window, 1.0, t.ptr(work), n_work, self._stream())

    def _step(self, k, st, plan, pools, head, req, tables, out):
        """One forward over a planned step (`lean_core.py:599-694`): embedding and first norm, every full layer, the
        pruned last layer; the residual rows of the step's readout tokens go to `out` (rows in step-row order)."""
        t, rows, n_work = tables
        n = len(st['tokens'])
        H, hq = self.hidden, self.hq
        dev, bf = self.device, torch.bfloat16
        if self.peer is not None:
            x, h = self._peer_rows(n)
        else:
            x = torch.empty(n, H, dtype=bf, device=dev)
            h = torch.empty(n, H, dtype=bf, device=dev)
        for kind in set(self.types):
            self._rope(kind, int(np.max(st['positions'])) if n else 0)
        feat = req.features
        self._k('rows', 'morj_embed_rmsnorm', t.ptr('tokens'), t.ptr('feature_row') if feat is not None else None,
                _ptr(feat), self.embed.data_ptr(), n, H, self.embed_scale, self.layers[0]['in_ln'].data_ptr(),
                self.eps, x.data_ptr(), h.data_ptr(), self._stream())
        d_max = max(dd for _, dd in self.geom.values())
        bufs = dict(x=x, h=h, q=torch.empty(n, hq * d_max, dtype=bf, device=dev),
                    attn=torch.empty(n, hq * d_max, dtype=bf, device=dev), o=torch.empty(n, H, dtype=bf, device=dev),
                    act=torch.empty(n, self.layers[0]['gu'].shape[0] // 2, dtype=bf, device=dev),
                    nb=int(st['n_bidir']), n_seg=len(st['qo_indptr']) - 1)
        # one step without kept pools: one temporary pool per layer kind, rewritten by every layer of that kind
        temp = {} if pools is not None else {kind: self._kv_pool(kind, plan['cap'][KINDS[kind]])
                                             for kind in set(self.types)}
        last = len(self.layers) - 1
        for i in range(len(self.layers)):
            kind = self.types[i]
            if pools is not None:
                kv = pools[i]
            else:
                kv = temp[kind]
                if len(head):
                    self._copy_head([kv], plan['slot_of'], head, layers=[i])
            if i == last and self.prune_last:
                self._last_layer(t, rows, n_work, self.layers[i], h, x, kv, out)
                return
            self._layer(i, t, n_work, kv, bufs)
        if rows:  # (no pruning) the readout rows' residual stream
            self._k('rows', 'morj_gather_rows', x.data_ptr(), H, t.ptr('ro_rows'), len(rows), H, out.data_ptr(), H,
                    self._stream())

    def _layer(self, i, t, n_work, kv, bufs):
        """Full decoder layer i over every token of a step (`lean_core.py:655-689`): QKV with the head epilogue into
        the pools, tree attention, O, residual + norms, gate/up with GeGLU, down, residual x scalar + the next layer's
        input norm. `bufs` holds the step's x and h (updated in place) and its scratch activations."""
        layer, kind = self.layers[i], self.types[i]
        hk, d = self.geom[kind]
        kk = KINDS[kind]
        k_pool, v_pool = kv
        x, h, o, act = bufs['x'], bufs['h'], bufs['o'], bufs['act']
        n, H, hq, eps, s = x.shape[0], self.hidden, self.hq, self.eps, self._stream()
        sliding = kind == 'sliding_attention'
        q, attn = bufs['q'][:, :hq * d], bufs['attn'][:, :hq * d]
        self._qkv(h, layer, 0, n, hq, hk, int(sliding), d, kind, t.ptr('positions'), t.ptr('slots_' + kk), q,
                  k_pool, v_pool)
        self._attention(q, k_pool, v_pool, attn, t, 'qo', 'kv_indptr_' + kk, 'kv_indices_' + kk, bufs['n_seg'],
                        bufs['nb'] if sliding else 0, kind, 'work_' + kk, n_work[kk])
        last = len(self.layers) - 1
        nxt = self.layers[i + 1]['in_ln'] if i < last else layer['in_ln']
        if self.peer is not None:
            # x rows go back to every rank once, after the last full layer (the readout gathers them)
            final = i == last - 1 if self.prune_last else i == last
            self._peer_site(attn, layer['o'], 0, n, layer['post_attn'], None, layer['pre_ff'], 1, 0)
            self._gemm(h, layer['gu'], act, nat.EPI_GEGLU)
            self._peer_site(act, layer['down'], 1, n, layer['post_ff'], layer['scalar'], nxt, int(i < last),
                            int(final))
            return
        self._gemm(attn, layer['o'], o)
        self._reduce(o)
        self._k('rows', 'morj_attn_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), layer['post_attn'].data_ptr(),
                layer['pre_ff'].data_ptr(), n, H, eps, s)
        self._gemm(h, layer['gu'], act, nat.EPI_GEGLU)
        self._gemm(act, layer['down'], o)
        self._reduce(o)
        self._k('rows', 'morj_mlp_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), layer['post_ff'].data_ptr(),
                layer['scalar'].data_ptr(), nxt.data_ptr(), n, H, eps, int(i < last), s)

    def _last_layer(self, t, rows, n_work, layer, h, x, kv, xr):
        """Last layer (`lean_core.py:696-737`): K/V of every token (later readouts attend to them), then q,
        attention, O and MLP for the readout rows only; their residual rows end in `xr`."""
        s = self._stream()
        n = h.shape[0]
        H, eps, hq = self.hidden, self.eps, self.hq
        kind = self.types[-1]
        hk, d = self.geom[kind]
        kk = KINDS[kind]
        k_pool, v_pool = kv
        has_v = int(kind == 'sliding_attention')
        dev, bf = self.device, torch.bfloat16
        qd = hq * d
        self._qkv(h, layer, qd, n, 0, hk, has_v, d, kind, t.ptr('positions'), t.ptr('slots_' + kk), None, k_pool,
                  v_pool)
        if not rows:
            return
        R = len(rows)
        hr = torch.empty(R, H, dtype=bf, device=dev)
        self._k('rows', 'morj_gather_rows', h.data_ptr(), H, t.ptr('ro_rows'), R, H, hr.data_ptr(), H, s)
        q = torch.empty(R, qd, dtype=bf, device=dev)
        self._qkv(hr, layer, 0, R, hq, 0, has_v, d, kind, t.ptr('ro_positions'), None, q, None, None)
        attn = torch.empty(R, qd, dtype=bf, device=dev)
        self._attention(q, k_pool, v_pool, attn, t, 'ro_qo', 'ro_kv_indptr', 'ro_kv_indices', R, 0, kind, 'ro_work',
                        n_work['ro'])
        o = torch.empty(R, H, dtype=bf, device=dev)
        self._gemm(attn, layer['o'], o)
        self._reduce(o)
        self._k('rows', 'morj_gather_rows', x.data_ptr(), H, t.ptr('ro_rows'), R, H, xr.data_ptr(), H, s)
        h2 = torch.empty(R, H, dtype=bf, device=dev)
        self._k('rows', 'morj_attn_epilogue', o.data_ptr(), xr.data_ptr(), h2.data_ptr(), layer['post_attn'].data_ptr(),
                layer['pre_ff'].data_ptr(), R, H, eps, s)
        act = torch.empty(R, layer['gu'].shape[0] // 2, dtype=bf, device=dev)
        self._gemm(h2, layer['gu'], act, nat.EPI_GEGLU)
        self._gemm(act, layer['down'], o)
        self._reduce(o)
        self._k('rows', 'morj_mlp_epilogue', o.data_ptr(), xr.data_ptr(), xr.data_ptr(), layer['post_ff'].data_ptr(),
                layer['scalar'].data_ptr(), layer['in_ln'].data_ptr(), R, H, eps, 0, s)

    def forward_tree(self, tree, label_ids):
        """Every sequence of an already built tree in one pass (reference `lean_core.py:739-742`)."""
        req = self.prepare([s.tolist() for s in tree.seqs], label_ids)
        return self.run(req, list(range(len(tree.seqs))))
