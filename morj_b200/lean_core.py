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
    """One request's tree, label ids, computed nodes and (with `retain`) its K/V pools
    (reference `lean_core.py:323-336`)."""

    def __init__(self, tree, label_ids, retain, head_nodes, pinned=False):
        self.tree, self.label_ids, self.retain = tree, label_ids, retain
        self.pinned = pinned
        self.head_nodes = head_nodes
        self.computed = set(head_nodes)
        self.read = set()
        self.tables = None
        self.pools = None
        self.n_real = len(tree.seqs)
        self.features = None
        self.bidir = frozenset()


def expand_images(seqs, images, image_id, boi_id, eoi_id):
    """Image placeholders -> BOI + one image token per soft token + EOI; block bounds and the split sequences that
    put node boundaries at every block's start and end (reference `lean_core.py:433-444,461-462,471-484`)."""
    out = []
    for seq in seqs:
        exp, k = [], 0
        for t in seq:
            if t == image_id:
                if k >= len(images):
                    raise ValueError('more image placeholders than images')
                exp += [boi_id] + [image_id] * len(images[k]) + [eoi_id]
                k += 1
            else:
                exp.append(t)
        if k != len(images):
            raise ValueError(f'{len(images)} images but {k} placeholders')
        out.append(exp)
    first = np.asarray(out[0])
    run_start = (first == image_id) & np.r_[True, first[:-1] != image_id]
    starts = np.flatnonzero(run_start)
    blobs = [(int(s), int(s) + len(f)) for s, f in zip(starts, images)]
    end = blobs[-1][1]
    if any(len(s) <= end or s[:end] != out[0][:end] for s in out):
        raise ValueError('every branch must hold the same images in its shared prefix')
    splits = []
    for s, e in blobs:
        splits += [out[0][:s], out[0][:e]]
    blob_start = np.asarray([s for s, _ in blobs])
    blob_end = np.asarray([e for _, e in blobs])
    blob_off = np.concatenate([[0], np.cumsum([e - s for s, e in blobs])])[:-1]

    def bidir_nodes(tree):
        return frozenset(n for n in tree.paths[0]
                         if any(s <= tree.nodes[n][1] and tree.nodes[n][2] <= e for s, e in blobs))
    return dict(seqs=out, splits=splits, blob_start=blob_start, blob_end=blob_end, blob_off=blob_off,
                bidir_nodes=bidir_nodes)


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
        """Compute and keep the K/V of a prefix many requests start with (reference `lean_core.py:419-426`)."""
        self.shared, self.shared_kv = None, None
        req = self.prepare([list(tokens)], [[0]], retain=True)
        self.run(req, [0])
        self.shared = np.asarray(tokens, dtype=np.int64)
        slots = np.concatenate([req.tree.slots(n) for n in req.tree.paths[0]])
        idx = torch.as_tensor(slots.astype(np.int32), device=self.device)
        kv = [(self._gather(k, idx), self._gather(v, idx)) for k, v in req.pools]
        torch.cuda.current_stream(self.device).synchronize()
        self.shared_kv = kv

    def prepare(self, seqs, label_ids, retain=False, images=None, available=None):
        """A request over `seqs` (reference `lean_core.py:428-469`): the tree (with image blocks expanded and split,
        and the shared head attached when every sequence starts with it), the retention decision, and retained
        pools with the shared head's K/V copied in."""
        seqs = [list(s) for s in seqs]
        splits, layout = [], None
        if images:
            layout = expand_images(seqs, images, self.image_id, self.boi_id, self.eoi_id)
            seqs, splits = layout['seqs'], layout['splits']
        shared = self.shared is not None and len(seqs) and all(
            len(s) > len(self.shared) and np.array_equal(np.asarray(s[:len(self.shared)]), self.shared) for s in seqs)
        tree = Tree(seqs + splits + ([self.shared] if shared else []))
        head = tree.paths[-1] if shared else []
        avail = self.free_bytes if available is None else available
        fits = tree.num_tokens * self.kv_bytes <= min(
            self.retain_budget, avail - min(tree.num_tokens, self.single_max) * self.act_bytes)
        req = Request(tree, list(label_ids) + [[0]] * len(splits) + ([[0]] if shared else []), retain and fits, head,
                      pinned=retain and not fits)
        req.n_real = len(seqs)
        if images:
            req.features = torch.cat([f.to(self.device, torch.bfloat16) for f in images]).contiguous()
            req.blob_start, req.blob_end, req.blob_off = layout['blob_start'], layout['blob_end'], layout['blob_off']
            req.bidir = layout['bidir_nodes'](tree)
        if req.retain:
            req.pools = [self._pool(kind, tree.num_tokens) for kind in self.types]
            if shared:
                head_slots = np.concatenate([tree.slots(n) for n in head])
                for (k, v), (sk, sv) in zip(req.pools, self.shared_kv):
                    self._fill_head(k, v, head_slots, sk, sv)
        return req

    def _pool(self, kind, n):
        hk, d = self.geom[kind]
        shape = (max(n, 1), hk, d)
        if POISON:  # test only: a slot read before it is written turns the answer into NaN
            return (torch.full(shape, float('nan'), dtype=torch.bfloat16, device=self.device),
                    torch.full(shape, float('nan'), dtype=torch.bfloat16, device=self.device))
        return (torch.empty(shape, dtype=torch.bfloat16, device=self.device),
                torch.empty(shape, dtype=torch.bfloat16, device=self.device))

    def _gather(self, src, idx):
        width = src[0].numel()
        out = torch.empty((len(idx),) + tuple(src.shape[1:]), dtype=src.dtype, device=self.device)
        self._k('rows', 'morj_gather_rows', src.data_ptr(), width, idx.data_ptr(), len(idx), width, out.data_ptr(), width,
                 self._stream())
        return out

    def _fill_head(self, k, v, slots, sk, sv):
        """Copy the shared head's K/V rows into pool slots (reference `lean_core.py:594-597`)."""
        idx = torch.as_tensor(np.asarray(slots, dtype=np.int32), device=self.device)
        width = k[0].numel()
        for dst, src in ((k, sk), (v, sv)):
            nat.call('morj_scatter_rows', src.data_ptr(), width, idx.data_ptr(), len(idx), width, dst.data_ptr(),
                     width, self._stream())

    def _grow(self, req, cap, kinds):
        """Pinned-mode pools with at least `cap` slots per kind; existing slots keep their contents
        (reference `lean_core.py:578-592`)."""
        old = req.pools
        if old is not None and all(old[i][0].shape[0] >= cap[kinds[k]] for i, k in enumerate(self.types)):
            return old
        pools = []
        for i, kind in enumerate(self.types):
            k, v = self._pool(kind, cap[kinds[kind]])
            if old is not None:
                n = min(old[i][0].shape[0], k.shape[0])
                k[:n].copy_(old[i][0][:n])
                v[:n].copy_(old[i][1][:n])
            pools.append((k, v))
        req.pools = pools
        return pools

    def _stream(self):
        s = torch.cuda.current_stream(self.device).cuda_stream
        if self.gemm_ws is not None:
            self.gemm_ws.register(s)
        return s

    # ---- pass -----------------------------------------------------------------------------------------------------
    def plan(self, req, seqs, available=None):
        """The planning half of `run` (reference `lean_core.py:497-529`): nodes to compute, pinned offsets and the
        pass plan after the memory-fit loop (raises MemoryError when nothing fits). No device work."""
        tree = req.tree
        cached = req.computed if req.retain or req.pinned else set(req.head_nodes)
        need = tree.pass_nodes(seqs, cached)
        per_token = {kk: sum(4 * self.geom[k][0] * self.geom[k][1] for k in self.types if KINDS[k] == kk)
                     for kk in 'gs'}
        head = np.concatenate([tree.slots(n) for n in req.head_nodes]) if req.head_nodes else np.zeros(0, np.int64)
        pinned = None
        if req.pinned:
            future = [b for b in range(req.n_real) if b not in req.read and b not in set(seqs)]
            pinned = tree.pinned_for(cached | set(need), future, self.window)
        step, single = self.step_tokens, self.single_max
        while True:
            plan = tree.plan_pass(need, seqs, self.window, single, step, req.retain,
                                  prealloc=() if req.retain else head, initial=req.tables, pinned=pinned,
                                  bidir=req.bidir)
            multi = len(plan['steps']) > 1
            persistent = req.pinned or (multi and not req.retain)
            largest = max(len(st['tokens']) for st in plan['steps'])
            pools = sum(plan['cap'][kk] * per_token[kk] for kk in 'gs') if persistent else 0
            budget = self.free_bytes if available is None else available
            if pools + largest * self.act_bytes <= budget:
                break
            if step <= 512:
                raise MemoryError(f'request needs {pools / 2**30:.1f} GiB of K/V pools; '
                                  f'{budget / 2**30:.1f} GiB available')
            if not multi and single:
                single = 0  # pools for every layer at once: cut the pass into steps so slots are freed as it goes
            else:
                step //= 2
        return need, head, pinned, plan

    def prepare_pass(self, req, seqs, available=None):
        """Host half of `run`: plan (with the memory-fit loop), the pools the pass writes (retained, pinned, per-pass,
        or per-step temporaries), and every step's tables uploaded to the device. The result can be executed any
        number of times (`execute_pass`); each execution recomputes the same nodes into the same slots."""
        tree = req.tree
        t0 = time.perf_counter()
        need, head, pinned, plan = self.plan(req, seqs, available)
        multi = len(plan['steps']) > 1
        if req.retain:
            pools = req.pools
        elif req.pinned:  # pools kept for the request; grown (old slots copied) when a pass needs more
            pools = self._grow(req, plan['cap'], KINDS)
            if req.tables is None and len(head):
                for i, (k, v) in enumerate(pools):
                    self._fill_head(k, v, plan['slot_of'][KINDS[self.types[i]]][head], *self.shared_kv[i])
        elif multi:  # pools for the pass, every layer
            pools = [self._pool(kind, plan['cap'][KINDS[kind]]) for kind in self.types]
            if len(head):
                for i, (k, v) in enumerate(pools):
                    self._fill_head(k, v, plan['slot_of'][KINDS[self.types[i]]][head], *self.shared_kv[i])
        else:
            pools = None  # one forward: a temporary pool per kind
        labels = [req.label_ids[b] for b in seqs]
        if any(len(ids) > MAX_LABELS for ids in labels):
            raise ValueError(f'at most {MAX_LABELS} labels per sequence')
        self.h2d_bytes = 0
        tables = [self._step_tables(k, st, plan, req) for k, st in enumerate(plan['steps'])]
        ro = self._readout_tables(plan, labels)
        host_ms = 1000 * (time.perf_counter() - t0)
        return dict(req=req, seqs=list(seqs), need=need, head=head, pinned=pinned, plan=plan, pools=pools,
                    labels=labels, tables=tables, ro=ro, host_ms=host_ms, h2d_bytes=self.h2d_bytes,
                    tokens=sum(len(st['tokens']) for st in plan['steps']))

    def execute_pass(self, p):
        """Device half of `run`: every step's forward and the label head; returns the FP32 probabilities (device,
        CSR over the requested sequences' labels). Launches only; nothing waits for the GPU."""
        plan = p['plan']
        finals = [self._step(k, st, plan, p['pools'], p['head'], p['req'], p['tables'][k])
                  for k, st in enumerate(plan['steps'])]
        return self._readout(finals, p['ro'])

    @torch.inference_mode()
    def run(self, req, seqs, available=None):
        """Label probabilities for sequences `seqs` of `req`, computing only the nodes not cached yet
        (reference `lean_core.py:495-576`: the same planning, memory-fit loop, pool strategy and state updates)."""
        tree = req.tree
        p = self.prepare_pass(req, seqs, available)
        self.last_need = p['need']
        plan, pinned, labels = p['plan'], p['pinned'], p['labels']
        self.timing = {'host_setup_ms': p['host_ms'], 'steps': len(plan['steps']), 'tokens': p['tokens']}
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        probs = self.execute_pass(p)
        end.record()
        self.enqueued = time.perf_counter()  # host done launching; the copy below waits for the GPU
        flat = probs.cpu().numpy()
        self.d2h_bytes = flat.nbytes
        code = nat.device_error(self._stream())
        if code:
            raise nat.NativeFailure(f'a kernel reported device error 0x{code:x}')
        out, o = [], 0
        for ids in labels:
            out.append(flat[o:o + len(ids)].astype(np.float64).tolist())
            o += len(ids)
        self.gpu_ms = start.elapsed_time(end)
        self.timing['gpu_ms'] = self.gpu_ms
        req.read.update(seqs)
        if req.retain or req.pinned:
            req.computed.update(p['need'])
        if req.pinned:
            req.tables = {}
            for kk in 'gs':
                table = np.full(tree.num_tokens, -1)
                table[pinned[kk]] = plan['slot_of'][kk][pinned[kk]]
                req.tables[kk] = table
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

    def _readout(self, finals, ro):
        """Final norm + label rows + softcap + per-sequence softmax in one kernel (reference `lean_core.py:558-561`)."""
        H = self.hidden
        xs = [xr for xr, rows in finals if rows]
        x_all = xs[0] if len(xs) == 1 else torch.cat(xs)
        t = ro['t']
        probs = torch.empty(ro['n_labels'], dtype=torch.float32, device=self.device)
        self._k('head', 'morj_label_head', x_all.data_ptr(), H, t.ptr('seq_row'), t.ptr('indptr'), t.ptr('labels'),
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
            rows = np.flatnonzero(st['tokens'] == self.image_id)
            fr = np.full(n, -1, np.int64)
            if len(rows):
                depth = st['positions'][rows]
                kb = np.searchsorted(req.blob_start, depth, side='right') - 1
                if (kb < 0).any() or (depth >= req.blob_end[kb]).any():
                    raise ValueError('image placeholder outside an image block')
                fr[rows] = req.blob_off[kb] + depth - req.blob_start[kb]
            t.add('feature_row', fr)
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

    def _step(self, k, st, plan, pools, head, req, tables):
        """One forward over a planned step (reference `lean_core.py:599-694`); returns (the residual rows of the
        step's readout tokens after the last layer, their row indices in the step)."""
        t, rows, n_work = tables
        s = self._stream()
        n = len(st['tokens'])
        H, eps, hq = self.hidden, self.eps, self.hq
        dev, bf = self.device, torch.bfloat16
        nb = int(st['n_bidir'])
        n_seg = len(st['qo_indptr']) - 1
        if self.peer is not None:
            x, h = self._peer_rows(n)
        else:
            x = torch.empty(n, H, dtype=bf, device=dev)
            h = torch.empty(n, H, dtype=bf, device=dev)
        max_pos = int(np.max(st['positions'])) if n else 0
        for kind in set(self.types):
            self._rope(kind, max_pos)
        feat = req.features
        self._k('rows', 'morj_embed_rmsnorm', t.ptr('tokens'), t.ptr('feature_row') if feat is not None else None,
                 _ptr(feat), self.embed.data_ptr(), n, H, self.embed_scale, self.layers[0]['in_ln'].data_ptr(), eps,
                 x.data_ptr(), h.data_ptr(), s)
        temp = {}
        if pools is None:  # one forward: a temporary pool per kind, rewritten by every layer of that kind
            for kind in set(self.types):
                temp[kind] = self._pool(kind, plan['cap'][KINDS[kind]])
        last = len(self.layers) - 1
        F = self.layers[0]['gu'].shape[0] // 2
        d_max = max(dd for _, dd in self.geom.values())
        q = torch.empty(n, hq * d_max, dtype=bf, device=dev)
        attn = torch.empty(n, hq * d_max, dtype=bf, device=dev)
        o = torch.empty(n, H, dtype=bf, device=dev)
        act = torch.empty(n, F, dtype=bf, device=dev)
        for i, layer in enumerate(self.layers):
            kind = layer['kind']
            hk, d = self.geom[kind]
            kk = KINDS[kind]
            if pools is not None:
                k_pool, v_pool = pools[i]
            else:
                k_pool, v_pool = temp[kind]
                if len(head):
                    self._fill_head(k_pool, v_pool, plan['slot_of'][kk][head], *self.shared_kv[i])
            has_v = int(kind == 'sliding_attention')
            if i == last and self.prune_last:
                return self._last_layer(t, rows, n_work, layer, h, x, k_pool, v_pool, kind, has_v)
            q_i = q[:, :hq * d]
            self._qkv(h, layer, 0, n, hq, hk, has_v, d, kind, t.ptr('positions'), t.ptr('slots_' + kk), q_i,
                      k_pool, v_pool)
            a_i = attn[:, :hq * d]
            self._attention(q_i, k_pool, v_pool, a_i, t, 'qo', 'kv_indptr_' + kk, 'kv_indices_' + kk, n_seg,
                            nb if kind == 'sliding_attention' else 0, kind, 'work_' + kk, n_work[kk])
            nxt = self.layers[i + 1]['in_ln'] if i < last else layer['in_ln']
            if self.peer is not None:
                # x rows go back to every rank once, after the last full layer (the readout gathers them)
                final = i == last - 1 if self.prune_last else i == last
                self._peer_site(a_i, layer['o'], 0, n, layer['post_attn'], None, layer['pre_ff'], 1, 0)
                self._gemm(h, layer['gu'], act, nat.EPI_GEGLU)
                self._peer_site(act, layer['down'], 1, n, layer['post_ff'], layer['scalar'], nxt, int(i < last),
                                int(final))
                continue
            self._gemm(a_i, layer['o'], o)
            self._reduce(o)
            self._k('rows', 'morj_attn_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), layer['post_attn'].data_ptr(),
                     layer['pre_ff'].data_ptr(), n, H, eps, s)
            self._gemm(h, layer['gu'], act, nat.EPI_GEGLU)
            self._gemm(act, layer['down'], o)
            self._reduce(o)
            self._k('rows', 'morj_mlp_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), layer['post_ff'].data_ptr(),
                     layer['scalar'].data_ptr(), nxt.data_ptr(), n, H, eps, int(i < last), s)
        # (no pruning) the readout rows' residual stream
        if not rows:
            return None, []
        xr = torch.empty(len(rows), H, dtype=bf, device=dev)
        self._k('rows', 'morj_gather_rows', x.data_ptr(), H, t.ptr('ro_rows'), len(rows), H, xr.data_ptr(), H, s)
        return xr, rows

    def _last_layer(self, t, rows, n_work, layer, h, x, k_pool, v_pool, kind, has_v):
        """Last layer (reference `lean_core.py:696-737`): K/V of every token, then q, attention, O and MLP for the
        readout rows only."""
        s = self._stream()
        n = h.shape[0]
        H, eps, hq = self.hidden, self.eps, self.hq
        hk, d = self.geom[kind]
        kk = KINDS[kind]
        dev, bf = self.device, torch.bfloat16
        qd = hq * d
        # K/V of every token (later readouts attend to them), straight into the pools
        self._qkv(h, layer, qd, n, 0, hk, has_v, d, kind, t.ptr('positions'), t.ptr('slots_' + kk), None, k_pool,
                  v_pool)
        if not rows:
            return None, []
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
        xr = torch.empty(R, H, dtype=bf, device=dev)
        self._k('rows', 'morj_gather_rows', x.data_ptr(), H, t.ptr('ro_rows'), R, H, xr.data_ptr(), H, s)
        h2 = torch.empty(R, H, dtype=bf, device=dev)
        self._k('rows', 'morj_attn_epilogue', o.data_ptr(), xr.data_ptr(), h2.data_ptr(), layer['post_attn'].data_ptr(),
                 layer['pre_ff'].data_ptr(), R, H, eps, s)
        F = layer['gu'].shape[0] // 2
        act = torch.empty(R, F, dtype=bf, device=dev)
        self._gemm(h2, layer['gu'], act, nat.EPI_GEGLU)
        self._gemm(act, layer['down'], o)
        self._reduce(o)
        self._k('rows', 'morj_mlp_epilogue', o.data_ptr(), xr.data_ptr(), xr.data_ptr(), layer['post_ff'].data_ptr(),
                 layer['scalar'].data_ptr(), layer['in_ln'].data_ptr(), R, H, eps, 0, s)
        return xr, rows

    def forward_tree(self, tree, label_ids):
        """Every sequence of an already built tree in one pass (reference `lean_core.py:739-742`)."""
        req = self.prepare([s.tolist() for s in tree.seqs], label_ids)
        return self.run(req, list(range(len(tree.seqs))))
