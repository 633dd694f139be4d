"""Tree-prefill throughput on B200: the lean engine's forward over a token tree at the 31B-class BF16 config.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload text|multimodal|latency]

One step = one forward pass over one request tree (every tree token computed, 60 layers, label probabilities at the
end). `value` is device-timed tokens/s with the plan tables already resident in HBM (CUDA events over K steps, max
over ranks); `e2e` is the same metric through the engine's public call `LeanGemma4.run` from host token ids to host
probabilities (planning, host-to-device tables, kernels, device-to-host probabilities inside the timed region).
N > 1: one process per GPU, each a full model replica on its own seeded tree (independent trees: no collective on
the data path; weak scaling). Weights (~52 GB BF16) and every input are larger than L2, so no L2 flush is needed.

`e2e` calls `prepare` then `run` per request, as `LeanEngine._score_pass` does (`lean_engine.py:111-122`).

`--impl reference` times the reference's own lean path (`aleria_judge/lean_core.py`, unmodified, installed under
`baseline/_ref`) on the host CPU, on the same workload tree: `LeanGemma4.prepare` + `run` over a 3-layer cut of the
model (one sliding, one global and the pruned global last layer) with torch-eager stand-ins for its GPU-only
FlashInfer calls and Triton kernels (`oracle/ref_cpu.py`). `ms_per_step` is that timed step; `value` extrapolates its
per-layer times to the 60-layer pattern. This process never loads the B200 library (`native_library_loaded`).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'tree-prefill tokens/s per B200 at 31B BF16'
UNIT = 'tokens/s'


def peaks():
    try:
        with open(os.path.join(ROOT, 'MEASURED_PEAKS.json')) as f:
            p = json.load(f)
        return dict(hbm=p['hbm_gbs'], bf16=p['bf16_tflops'], bf16_sustained=p['bf16_tflops_sustained'],
                    source='measured')
    except (OSError, KeyError, ValueError):
        return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source='fallback')


def workload(name, rank):
    from morj_b200 import workloads as w
    if name == 'text':
        return w.text_tree(seed=rank), 'text tree: 1500-token prefix + 3 questions x 3 rotations x 60 tokens'
    if name == 'latency':
        return w.latency_tree(seed=rank), 'latency tree: 8192-token prefix + 8 branches x 64 tokens'
    if name == 'multimodal':
        return (w.multimodal_tree(seed=rank),
                'multimodal tree: 8 x 560 image soft tokens + 300 text + 2 questions x 4 rotations x 40 tokens')
    if name == 'sweep':
        forests = w.pack_forests(w.sweep_trees(seed=rank, count=64))
        return forests, (f'replication sweep: 64 seeded trees per GPU (prefix log-uniform 64-8192, 2-8 branches of '
                         f'16-128, 2-16 labels) packed into {len(forests)} forests of <= 8192 tokens')
    raise ValueError(name)


class Clocks:
    """nvidia-smi samples of this process's GPU while a region runs."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_id):
        self.gpu_id, self.proc, self.rows = gpu_id, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '200', '-i', self.gpu_id], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(',')]
            if len(parts) == 9:
                self.rows.append(parts)

    def summary(self):
        if not self.rows:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled'], 'samples': 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace('.', '').isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == 'active'})
        power = [float(r[3]) for r in self.rows if r[3].replace('.', '').isdigit()]
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': reasons, 'samples': len(self.rows), 'power_w_max': max(power) if power else None}


def _cpu_model():
    try:
        with open('/proc/cpuinfo') as f:
            for line in f:
                if line.startswith('model name'):
                    return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


def _native_loaded():
    """Whether this process has mapped the B200 library (the reference arm must not)."""
    try:
        with open('/proc/self/maps') as f:
            return any('_morj_b200' in line for line in f)
    except OSError:
        return None


def tree_flops(top, plan, tokens):
    """Algorithmic FLOPs of one pass: 2 x linear parameters per computed token plus 4 x Hq x d per visible (query,
    key) pair, from a planner's pass plan (the reference's and this engine's plans are identical)."""
    from morj_b200 import workloads as w
    c = top['text_config']
    pairs = w.attention_pairs(plan, c['sliding_window'], c['layer_types'])
    return w.linear_flops_per_token(top) * tokens + 4 * c['num_attention_heads'] * c['head_dim'] * pairs


def bench_config(args, world, desc, tokens, flops):
    """The `config` object of the JSON line; both arms print the same one for the same arguments."""
    tp = args.mode == 'tp' and world > 1
    par = (f'replicas x{world} (independent trees, no collective)' if not tp else
           f'tensor parallel x{world} (O/down partial rows read by their row owners over NVLink, reduced with the '
           f'epilogues)' if args.tp_comm == 'peer' else f'tensor parallel x{world} (NCCL all-reduce after O and down)')
    work = (f'31B-class Gemma-style decoder, {desc}' if not args.layers else
            f'31B-class Gemma-style decoder cut to {args.layers} layers (profiling), {desc}')
    return dict(workload=work, tokens=tokens, parallelism=par,
                l2='inputs larger than L2 (52 GB of weights streamed per step)',
                tflops_per_tree_specified=round(flops / 1e12, 2))


def reference_cpu(args, rank=0):
    """The reference's own lean path on the host CPU (`oracle.ref_cpu.TimedReference`) over this run's workload
    tree; raises ImportError when the reference package is not installed beside the repository."""
    import torch
    from morj_b200 import workloads as w
    from oracle.ref_cpu import TimedReference
    torch.set_num_threads(os.cpu_count())
    top = w.gemma31b_config()
    if args.layers:
        top = w.reduced_config(top, args.layers)
    tree_in, desc = workload(args.workload, rank)
    if isinstance(tree_in, list):
        raise ImportError('the CPU reference times one request tree, not a forest sweep')
    return TimedReference(top, tree_in), top, desc


def cpu_reference_line(tr, samples):
    med = {k: statistics.median(s[k] for s in samples) for k in ('seconds', 'setup', 'sliding', 'global_', 'last')}
    tree_s = statistics.median(tr.extrapolate(s) for s in samples)
    body = tr.full_types[:-1]
    n_s = sum(1 for k in body if k == 'sliding_attention')
    return tree_s, samples[0]['tokens'], dict(
        step=('the reference LeanGemma4.prepare + run (aleria_judge/lean_core.py:428-576, unmodified, from '
              'baseline/_ref) on the host CPU over a 3-layer cut of the model (1 sliding, 1 global, the pruned global '
              'last layer) at the full tree; FlashInfer and its 3 Triton kernels replaced by torch-eager stand-ins '
              '(oracle/ref_cpu.py)'),
        ms_per_step_timed=round(1000 * med['seconds'], 1),
        ms_setup=round(1000 * med['setup'], 1), ms_sliding_layer=round(1000 * med['sliding'], 1),
        ms_global_layer=round(1000 * med['global_'], 1), ms_last_layer_and_readout=round(1000 * med['last'], 1),
        extrapolated_tree_ms=round(1000 * tree_s, 1),
        extrapolation=f'setup + {n_s} x sliding + {len(body) - n_s} x global + last',
        samples=len(samples), cores=os.cpu_count(), threads=__import__('torch').get_num_threads(), cpu=_cpu_model())


def reference_arm(args, rank, world):
    """The reference arm: rank 0 times the reference's own lean path on the host CPU (no other rank works). A step is
    one request through a 3-layer cut of the model; `ms_per_step` is that timed step, `value` the tokens/s of the
    whole model extrapolated from its per-layer times (the metric is per 60-layer tree)."""
    if rank != 0:
        return
    try:
        tr, top, desc = reference_cpu(args)
    except ImportError as error:
        print(json.dumps(dict(impl='reference', unavailable=f'reference package not installed: {error}')),
              flush=True)
        return
    for _ in range(args.warmup):
        tr.sample()
    samples = [tr.sample() for _ in range(args.steps)]
    tree_s, tokens, run = cpu_reference_line(tr, samples)
    plan = tr.plan_of_last_request()
    value = tokens / tree_s
    line = dict(metric=METRIC, value=value, unit=UNIT, n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                ms_per_step=run['ms_per_step_timed'], higher_is_better=True,
                scaling='strong' if args.mode == 'tp' and world > 1 else 'weak', vs_baseline=None,
                dtype='bf16', data='synthetic (timing weights: a seeded N(0, 0.02) block tiled; uniform token ids)',
                impl='reference', value_basis='extrapolated from the timed 3-layer step to the full layer pattern',
                config=bench_config(args, world, desc, tokens, tree_flops(top, plan, tokens)),
                reference_run=run,
                cpu_baseline=dict(value=value, unit=UNIT, cores=os.cpu_count(), kind='reference',
                                  sample=(f'{args.steps} requests of the {tokens}-token tree through the reference '
                                          f'run on a 3-layer cut, extrapolated to {len(tr.full_types)} layers'),
                                  cpu=_cpu_model()),
                e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0),
                native_library_loaded=_native_loaded())
    print(json.dumps(line), flush=True)


def kernel_arm(args):
    """One kernel alone on a mid-size case (per-kernel timing and small ncu captures):
    gemm / geglu: the 31B gate-up GEMM shape (M = 2040 text-tree tokens, K = 5376) with a plain or GeGLU epilogue;
    attention / attention-window: the op-level paged tree attention (2048 + 8 x 64 tokens, 32/16 heads of 128, pages
    of 64 through a shuffled page table), global or sliding window 1024;
    attention-text-sliding / attention-text-global: one layer's attention of the 31B text tree on its planner tables;
    attn-epilogue / mlp-epilogue: a residual epilogue on `--m` rows of 5376 (2040: the text tree);
    peer-reduce: one tensor-parallel site's owner reduction on the latency tree's rows, `--world` ranks emulated."""
    import torch
    from morj_b200 import _native as nat
    sys.path.insert(0, os.path.join(ROOT, 'tests'))
    dev = torch.device('cuda', 0)
    s = torch.cuda.current_stream().cuda_stream
    ws = None
    if not args.no_split:  # (the engine's configuration: split tiles on its stream)
        ws = nat.GemmWorkspace(dev)
        ws.register(s)
    if args.kernel == 'qkv':
        # the sliding-layer QKV projection with the fused head norm + RoPE + pool scatter epilogue
        M, H, d, hq, hk = args.m, 5376, 128, 32, 16
        n_out = (hq + 2 * hk) * d
        a = torch.randn(M, H, device=dev).to(torch.bfloat16)
        w = (torch.randn(n_out, H, device=dev) * 0.02).to(torch.bfloat16)
        qn = torch.ones(d, device=dev, dtype=torch.bfloat16)
        pos = torch.arange(M, device=dev, dtype=torch.int32)
        inv = (1.0 / (10000 ** (torch.arange(0, d, 2, device=dev).float() / d))).contiguous()
        rope = torch.empty(M, d // 2, 2, device=dev)
        nat.call('morj_rope_table', inv.data_ptr(), d // 2, M, rope.data_ptr(), s)
        slots = torch.randperm(M, device=dev).to(torch.int32)
        q_out = torch.empty(M, hq, d, device=dev, dtype=torch.bfloat16)
        kp = torch.empty(M, hk, d, device=dev, dtype=torch.bfloat16)
        vp = torch.empty(M, hk, d, device=dev, dtype=torch.bfloat16)
        flops = 2 * M * n_out * H

        def launch():
            nat.call('morj_gemm_qkv_rope', a.data_ptr(), H, w.data_ptr(), H, M, H, hq, hk, 1 | args.force, d,
                     qn.data_ptr(),
                     qn.data_ptr(), pos.data_ptr(), rope.data_ptr(), M, slots.data_ptr(), 1e-6, q_out.data_ptr(),
                     kp.data_ptr(), vp.data_ptr(), s)
        shape = dict(M=M, N=n_out, K=H)
    elif args.kernel in ('gemm', 'geglu'):
        M, N, K = args.m, args.n, args.k
        a = torch.randn(M, K, device=dev).to(torch.bfloat16)
        # launches cycle through enough copies of the weights to exceed L2 (126 MB), so each reads them from HBM
        bs = [(torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16) for _ in range(-(-300_000_000 // (2 * N * K)))]
        epi = (nat.EPI_GEGLU if args.kernel == 'geglu' else nat.EPI_STORE) | args.force
        c = torch.empty(M, N // 2 if args.kernel == 'geglu' else N, device=dev, dtype=torch.bfloat16)
        flops = 2 * M * N * K
        turn = [0]

        def launch():
            b = bs[turn[0] % len(bs)]
            turn[0] += 1
            nat.call('morj_gemm_bf16', a.data_ptr(), K, b.data_ptr(), K, c.data_ptr(), c.stride(0), M, N, K, epi, s)
        shape = dict(M=M, N=N, K=K, weight_copies=len(bs))
    elif args.kernel.startswith('attention-text'):
        # one full layer's tree attention of the 31B text tree with the planner's own tables (1500-token prefix + 9
        # branches of 60; 32 / 16 heads of 128; sliding: window 1024), q and k scaled as the model's q/k norms leave
        # them (unit-variance logits at scale 1)
        from morj_b200 import workloads as w
        from morj_b200.tree import Tree
        sliding = args.kernel.endswith('sliding')
        window, kk = (1024, 's') if sliding else (0, 'g')
        tree_in = w.text_tree(0)
        tree = Tree(tree_in['seqs'])
        plan = tree.plan_pass(tree.pass_nodes(range(len(tree.seqs)), set()), list(range(len(tree.seqs))), 1024, 16384,
                              8192, False)
        st = plan['steps'][0]
        n, hq, hk, d = len(st['tokens']), 32, 16, 128
        g = torch.Generator(device=dev).manual_seed(0)
        q = (torch.randn(n, hq, d, device=dev, generator=g) * d ** -0.25).to(torch.bfloat16)
        cap = plan['cap'][kk]
        kp = (torch.randn(cap, hk, d, device=dev, generator=g) * d ** -0.25).to(torch.bfloat16)
        vp = torch.randn(cap, hk, d, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty_like(q)
        qo = np.asarray(st['qo_indptr'], np.int32)
        kvp = np.asarray(st['kv_indptr_' + kk], np.int32)
        work = nat.attention_work(qo, kvp, 0, hq, hk, window)
        t = [torch.as_tensor(x, device=dev) for x in (qo, kvp, np.asarray(st['kv_indices_' + kk], np.int32), work)]
        flops = 4 * hq * d * w.attention_pairs(plan, 1024, ['sliding_attention' if sliding else 'full_attention'])

        def launch():
            nat.call('morj_tree_attention', q.data_ptr(), n, kp.data_ptr(), vp.data_ptr(), cap, out.data_ptr(),
                     t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), None, len(qo) - 1, 0, hq, hk, d, 1, window,
                     1.0, t[3].data_ptr(), len(work) // 2, s)
        shape = dict(tokens=n, window=window, tiles=len(work) // 2)
    elif args.kernel in ('attn-epilogue', 'mlp-epilogue'):
        # the post-attention / post-MLP residual epilogue on the text tree's rows (2040 x 5376); launches cycle through
        # four sets of rows (264 MB, past L2) so each reads its inputs from HBM
        n, H = args.m, 5376
        g = torch.Generator(device=dev).manual_seed(0)
        sets = [[torch.randn(n, H, device=dev, generator=g).to(torch.bfloat16) for _ in range(3)] for _ in range(4)]
        wn = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).to(torch.bfloat16)
        sc = torch.full((1,), 0.75, device=dev).to(torch.bfloat16)
        nbytes = 4 * n * H * 2  # o (or d) and x read, x and h written
        turn = [0]

        def launch():
            o, x, h = sets[turn[0] % 4]
            turn[0] += 1
            if args.kernel == 'attn-epilogue':
                nat.call('morj_attn_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), wn.data_ptr(), wn.data_ptr(),
                         n, H, 1e-6, s)
            else:
                nat.call('morj_mlp_epilogue', o.data_ptr(), x.data_ptr(), h.data_ptr(), wn.data_ptr(), sc.data_ptr(),
                         wn.data_ptr(), n, H, 1e-6, 1, s)
        shape = dict(rows=n, hidden=H)
    elif args.kernel == 'peer-reduce':
        # the owner's reduction of one tensor-parallel site (post-attention epilogue) on the latency tree's rows
        # (8192 + 8 x 64, hidden 5376), the `args.world` ranks of a group emulated on this GPU: every rank's
        # row-parallel GEMM has written its partials once, so the timed launches of rank 0's reduction find their
        # counters met and read and write this GPU's memory only (no NVLink: the kernel's own cost)
        import ctypes
        from morj_b200.tp import exchange_layout, owner, partial_target
        world, n, H, k = args.world, 8704, 5376, 64
        lay = exchange_layout(world, H, n)
        bufs = [torch.zeros(lay['nbytes'], dtype=torch.uint8, device=dev) for _ in range(world)]
        descs = []
        for r in range(world):
            d = nat.PeerDesc()
            d.world, d.rank, d.max_blocks, d.hidden = world, r, lay['max_blocks'], H
            for q in range(world):
                for name, (off, _) in lay['regions'].items():
                    getattr(d, name)[q] = bufs[q].data_ptr() + off
            descs.append(d)
        g = torch.Generator(device=dev).manual_seed(0)
        wn = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).to(torch.bfloat16)
        for r in range(world):
            a = torch.randn(n, k, device=dev, generator=g).to(torch.bfloat16)
            wt = (torch.randn(H, k, device=dev, generator=g) * 0.1).to(torch.bfloat16)
            nat.call('morj_gemm_bf16_peer', a.data_ptr(), k, wt.data_ptr(), k, n, H, k, ctypes.addressof(descs[r]), s)
        d0, tgt = ctypes.addressof(descs[0]), partial_target(1, world, H)
        owned = sum(min(n, (b + 1) * 128) - b * 128 for b in range(-(-n // 128)) if owner(b, world) == 0)
        nbytes = owned * H * 2 * (world + 2 + world)  # every rank's partial, x read and written, h to every rank

        def launch():
            nat.call('morj_peer_reduce', d0, 0, n, wn.data_ptr(), None, wn.data_ptr(), 1e-6, 1, 0, tgt, s)
        shape = dict(rows=n, owned_rows=owned, hidden=H, world=world)
    else:
        from attn_cases import op_level_case, unmasked_pairs
        window = 1024 if args.kernel == 'attention-window' else 0
        case = op_level_case()
        q, kp, vp = case['q'].to(dev), case['k_pool'].to(dev), case['v_pool'].to(dev)
        out = torch.empty_like(q)
        qo = case['qo_indptr']
        work = nat.attention_work(qo, case['kv_indptr'], 0, case['hq'], case['hk'], window, case['page_size'],
                                  case['last_page_len'])
        nw = len(work) // 2
        t = [torch.as_tensor(x, device=dev) for x in (qo, case['kv_indptr'], case['kv_indices'],
                                                       case['last_page_len'], work)]
        kv_len = [(case['kv_indptr'][i + 1] - case['kv_indptr'][i] - 1) * case['page_size'] + case['last_page_len'][i]
                  for i in range(len(qo) - 1)]
        flops = 4 * case['hq'] * case['d'] * unmasked_pairs(qo, kv_len, window)

        def launch():
            nat.call('morj_tree_attention', q.data_ptr(), q.shape[0], kp.data_ptr(), vp.data_ptr(), kp.shape[0],
                     out.data_ptr(), t[0].data_ptr(),
                     t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(), len(qo) - 1, 0, case['hq'], case['hk'],
                     case['d'], case['page_size'], window, float(case['sm_scale']), t[4].data_ptr(), nw, s)
        shape = dict(tokens=int(qo[-1]), window=window, pages=len(case['kv_indices']))
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    pk = peaks()
    if args.kernel in ('peer-reduce', 'attn-epilogue', 'mlp-epilogue'):
        gbs = nbytes / (ms / 1000) / 1e9
        print(json.dumps(dict(kernel=args.kernel, shape=shape, ms=round(ms, 4), gbs=round(gbs, 1),
                              frac_of_copy_peak=round(gbs / pk['hbm'], 4), peak_source=pk['source'],
                              mbytes=round(nbytes / 1e6, 1))), flush=True)
    else:
        tf = flops / (ms / 1000) / 1e12
        extra = {}
        if args.kernel in ('gemm', 'geglu'):  # operand bytes (the weights dominate at small M: HBM-bound there)
            ob = 2 * (args.m * args.k + args.n * args.k + args.m * (args.n // 2 if args.kernel == 'geglu' else args.n))
            extra = dict(gbs=round(ob / (ms / 1000) / 1e9, 1), frac_of_copy_peak=round(ob / (ms / 1000) / 1e9 /
                                                                                        pk['hbm'], 4))
        print(json.dumps(dict(kernel=args.kernel, shape=shape, ms=round(ms, 4), tflops=round(tf, 1),
                              frac_of_burst_peak=round(tf / pk['bf16'], 4), peak_source=pk['source'],
                              gflop=round(flops / 1e9, 2), **extra)), flush=True)
    assert nat.device_error(s) == 0
    if ws is not None:
        ws.close()


def vision_arm(args):
    """The image path: `args.images` images (random pixels, 896 x 896, the processor's default 280 soft tokens each)
    through `morj_b200.vision.VisionTower` and, on the same GPU, through the reference's own path (transformers'
    Gemma4VisionModel + Gemma4MultimodalEmbedder in BF16 with SDPA attention, as `lean_core.py:752-781` runs them),
    transformers' default Gemma 4 vision config with seeded random weights, text hidden 5376. Prints ms per batch of
    both and the soft tokens' relative difference."""
    import torch
    from PIL import Image
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig, Gemma4VisionConfig
    from transformers.models.gemma4.image_processing_gemma4 import Gemma4ImageProcessor
    from transformers.models.gemma4.modeling_gemma4 import Gemma4MultimodalEmbedder, Gemma4VisionModel
    from morj_b200.vision import VisionTower
    dev = torch.device('cuda', 0)
    vc = Gemma4VisionConfig()
    vc._attn_implementation = 'sdpa'
    tower = Gemma4VisionModel(vc).to(torch.bfloat16)
    embedder = Gemma4MultimodalEmbedder(vc, Gemma4TextConfig(hidden_size=5376)).to(torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    state = {}
    for prefix, module in (('model.vision_tower.', tower), ('model.embed_vision.', embedder)):
        for k, v in module.state_dict().items():
            t = (1 + 0.1 * torch.randn(v.shape, generator=g)) if v.dim() == 1 else torch.randn(v.shape, generator=g) * (
                0.3 if 'position_embedding_table' in k else 0.02)
            if k.endswith(('q_norm.weight', 'k_norm.weight')):
                t = t * v.shape[0] ** -0.25
            state[prefix + k] = t.to(torch.bfloat16)
        module.load_state_dict({k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}, strict=False)
    tower, embedder = tower.to(dev).eval(), embedder.to(dev).eval()
    vcfg = dict(vc.to_dict(), rope_parameters=vc.rope_parameters)
    ours = VisionTower(vcfg, 5376, lambda k: state[k], dev)
    rng = np.random.default_rng(0)
    imgs = [Image.fromarray((rng.random((896, 896, 3)) * 255).astype(np.uint8)) for _ in range(args.images)]
    p = Gemma4ImageProcessor()(imgs, return_tensors='pt')
    pv, pos = p['pixel_values'], p['image_position_ids']

    def ref():
        with torch.inference_mode():
            h = tower(pixel_values=pv.to(dev, torch.bfloat16), pixel_position_ids=pos.to(dev)).last_hidden_state
            return embedder(inputs_embeds=h).reshape(-1, 5376)

    def mine():
        return ours.forward(pv, pos)[0]

    out = {}
    for name, fn in (('reference_transformers', ref), ('morj_b200', mine)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            r = fn()
        e1.record()
        torch.cuda.synchronize()
        out[name] = dict(ms_per_batch=round(e0.elapsed_time(e1) / args.steps, 3))
        out[name + '_result'] = r.float()
    diff = float((out.pop('morj_b200_result') - out['reference_transformers_result']).norm() /
                 out.pop('reference_transformers_result').norm())
    print(json.dumps(dict(kernel='vision', images=len(imgs), patches_per_image=int(pv.shape[1]),
                          soft_tokens=int(p['num_soft_tokens_per_image'].sum()), config='Gemma4VisionConfig() defaults',
                          relative_difference=round(diff, 5), speedup=round(
                              out['reference_transformers']['ms_per_batch'] / out['morj_b200']['ms_per_batch'], 2),
                          **out)), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--workload', default='text', choices=['text', 'multimodal', 'latency', 'sweep'])
    ap.add_argument('--layers', type=int, default=0,
                    help='profiling only: the 31B-class model cut to its first L layers (same row and GEMM shapes, '
                         'a few GB on the device); 0 = all 60')
    ap.add_argument('--tp-comm', default='peer', choices=['peer', 'nccl'],
                    help='tensor parallelism: reduce over peer memory fused with the epilogues, or NCCL all-reduce')
    ap.add_argument('--mode', default='replicas', choices=['replicas', 'tp'],
                    help='replicas: one model per GPU on independent trees (weak scaling); tp: one tree, the model '
                         'sharded over all GPUs with NCCL all-reduces (strong scaling, single-tree latency)')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-tp-leg', action='store_true',
                    help='replicas at N > 1: skip the tensor-parallel latency leg that follows the replica measurement')
    ap.add_argument('--kernel', choices=['gemm', 'geglu', 'qkv', 'attention', 'attention-window',
                                         'attention-text-sliding', 'attention-text-global', 'peer-reduce',
                                         'attn-epilogue', 'mlp-epilogue', 'vision'],
                    help='time one kernel alone instead of the tree forward')
    ap.add_argument('--no-split', action='store_true',
                    help='no split-tile workspace registered (every GEMM tile computed whole)')
    ap.add_argument('--force', type=lambda v: int(v, 0), default=0,
                    help='kernel mode: or-ed into the GEMM epilogue (0x100 SM-pair kernel, 0x200 one-CTA kernel)')
    ap.add_argument('--images', type=int, default=8, help='--kernel vision: images per batch')
    ap.add_argument('--world', type=int, default=2, help='--kernel peer-reduce: ranks of the emulated group')
    ap.add_argument('--m', type=int, default=2040)
    ap.add_argument('--n', type=int, default=43008)
    ap.add_argument('--k', type=int, default=5376)
    args = ap.parse_args()
    if args.kernel == 'vision':
        return vision_arm(args)
    if args.kernel:
        return kernel_arm(args)
    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    if args.impl == 'reference':
        return reference_arm(args, rank, world)

    import datetime
    import torch
    import torch.distributed as dist
    from morj_b200 import workloads as w
    from morj_b200.lean_core import LeanGemma4
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=600))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    tp = args.mode == 'tp' and world > 1
    top = w.gemma31b_config()
    if args.layers:
        top = w.reduced_config(top, args.layers)
    t_init = time.perf_counter()
    model = LeanGemma4.random_init(top, seed=0, device=dev, tp_group=dist.group.WORLD if tp else None,
                                   tp_comm=args.tp_comm)
    if args.no_split and model.gemm_ws is not None:  # every GEMM tile computed whole
        model.gemm_ws.close()
        model.gemm_ws = None
    torch.cuda.synchronize()
    init_s = time.perf_counter() - t_init
    tree_in, desc = workload(args.workload, 0 if tp else rank)
    requests = tree_in if isinstance(tree_in, list) else [tree_in]
    for r in requests:  # image features start in pinned host memory (the end-to-end call copies them in)
        r['host_images'] = [f.pin_memory() for f in r['images']] if r['images'] else None
    preps = []
    for r in requests:
        images = [f.to(dev) for f in r['images']] if r['images'] else None
        req = model.prepare(r['seqs'], r['label_ids'], images=images)
        preps.append(model.prepare_pass(req, list(range(len(r['seqs'])))))
    tokens = sum(p['tokens'] for p in preps)
    c = top['text_config']
    flops = sum(tree_flops(top, p['plan'], p['tokens']) for p in preps)
    pairs = sum(w.attention_pairs(p['plan'], c['sliding_window'], c['layer_types']) for p in preps)
    flops_attn = 4 * c['num_attention_heads'] * c['head_dim'] * pairs

    def execute_all():
        for p in preps:
            model.execute_pass(p)

    copied = {'h2d': 0, 'd2h': 0}

    def run_all():
        """What a caller does per request (`LeanEngine._score_pass`, `lean_engine.py:111-122`): prepare, then run;
        host token ids and pinned host image features in, host probabilities out."""
        out, h2d, d2h = [], 0, 0
        for r in requests:
            req = model.prepare(r['seqs'], r['label_ids'], images=r['host_images'])
            out.append(model.run(req, list(range(len(r['seqs'])))))
            h2d += model.h2d_bytes + sum(f.numel() * f.element_size() for f in r['host_images'] or [])
            d2h += model.d2h_bytes
        copied.update(h2d=h2d, d2h=d2h)
        return out
    props = torch.cuda.get_device_properties(dev)
    clocks = Clocks('GPU-' + str(props.uuid) if hasattr(props, 'uuid') else str(local))

    # ---- device-timed forward over a resident plan -------------------------------------------------------------
    with torch.inference_mode():
        for _ in range(args.warmup):
            execute_all()
        barrier()
        clocks.start()
        launches0 = model.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        for _ in range(args.steps):
            execute_all()
        e1.record()
        barrier()
        ms = e0.elapsed_time(e1) / args.steps
        launches = (model.launches - launches0) // args.steps
        # ---- end to end through the public calls (host ids -> host probabilities) -------------------------------
        for _ in range(2):
            probs = run_all()
        barrier()
        lat = []
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record()
        for _ in range(args.steps):
            t0 = time.perf_counter()
            run_all()
            lat.append(1000 * (time.perf_counter() - t0))
        e3.record()
        barrier()
        clocks.stop()
        e2e_ms = e2.elapsed_time(e3) / args.steps
        h2d, d2h = copied['h2d'], copied['d2h']
        # ---- the same planned pass captured once in a CUDA graph and replayed (launch gaps between kernels gone) ----
        graph_ms = None
        if not tp:  # (a graph holding NCCL calls is not worth its teardown rules here)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                execute_all()
            graph.replay()
            barrier()
            e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e4.record()
            for _ in range(args.steps):
                graph.replay()
            e5.record()
            barrier()
            graph_ms = round(e4.elapsed_time(e5) / args.steps, 3)
            del graph
        # ---- one traced step (CUDA events around every kernel) for the per-kernel roofline: the stream is held by a
        # device-side sleep while the host queues the whole step, so no event pair holds host launch latency ------
        model.trace = []
        torch.cuda._sleep(int(0.25 * 2.0e9))  # ~0.25 s at 2 GHz (longer at the power-capped clock)
        execute_all()
        torch.cuda.synchronize()
        trace, model.trace = model.trace, None
        trace_span = trace[0][2].elapsed_time(trace[-1][3])
    per_kind = {}
    for kind, fl, a, b in trace:
        d = per_kind.setdefault(kind, dict(ms=0.0, launches=0, flops=0))
        d['ms'] += a.elapsed_time(b)
        d['launches'] += 1
        d['flops'] += fl
    ms_max = max_over_ranks(ms)
    e2e_max = max_over_ranks(e2e_ms)
    trees = 1 if tp else world  # tensor parallelism: all ranks work on the same tree
    value = tokens * trees / (ms_max / 1000)
    e2e_value = tokens * trees / (e2e_max / 1000)
    pk = peaks()
    # dominant kernel: the gate/up GEMM with the GeGLU epilogue (M = tree tokens, N = 2 x 21504, K = 5376); the
    # last layer's readout-only launch (M = reads) is left out so every averaged launch has the captured shape
    big = [(fl, a.elapsed_time(b)) for kind, fl, a, b in trace if kind == 'gemm_geglu' and fl == max(
        f for k, f, _, _ in trace if k == 'gemm_geglu')]
    g_ms = sum(t for _, t in big)
    achieved = sum(f for f, _ in big) / (g_ms / 1000) / 1e12
    allg = [(fl, a.elapsed_time(b)) for kind, fl, a, b in trace if kind.startswith('gemm')]
    all_tf = sum(f for f, _ in allg) / (sum(t for _, t in allg) / 1000) / 1e12
    traffic, kname = None, 'gemm kernel<GEGLU>'
    tfile = os.path.join(ROOT, 'profiles', 'gemm_geglu_traffic.json')
    if os.path.exists(tfile):
        with open(tfile) as f:
            tr = json.load(f)
        kname = tr.get('kernel', kname)
        if tr.get('M') == tokens and not tp and len(preps) == 1:
            traffic = tr.get('bytes_per_launch')
    attn_ms = per_kind.get('attention', {}).get('ms', 0.0)
    alone = attention_alone(model, preps[0], top, args.steps) if (len(preps) == 1 and not tp and
                                                                    len(preps[0]['plan']['steps']) == 1) else None
    parity = None
    if rank == 0 and args.workload == 'text' and not args.layers:
        # the bench tree's probabilities against the oracle's on the same weights and tree, recorded by
        # tests/golden/make_oracle_31b.py (tests/test_gpu_parity_31b.py checks the record reproduces)
        gfile = os.path.join(ROOT, 'tests', 'golden', 'oracle_31b_text.json')
        if os.path.exists(gfile):
            with open(gfile) as f:
                rec = json.load(f)
            got = np.concatenate([np.asarray(r, np.float64) for r in probs[0]])
            bf = np.concatenate([np.asarray(r, np.float64) for r in rec['probs']])
            fp = np.concatenate([np.asarray(r, np.float64) for r in rec['probs_fp32']])
            parity = dict(vs='oracle on the same weights and tree: BF16 (the reference lean path\'s rounding points) '
                             'and FP32 (the exact model)',
                          max_abs_vs_bf16_path=float(np.abs(got - bf).max()),
                          max_abs_vs_fp32=float(np.abs(got - fp).max()),
                          bf16_path_max_abs_vs_fp32=float(np.abs(bf - fp).max()), probabilities=int(len(got)))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            tr, _, _ = reference_cpu(args)
            tr.sample()  # warm-up
            samples = [tr.sample() for _ in range(2)]
            tree_s, ref_tokens, run = cpu_reference_line(tr, samples)
            cpu = dict(value=ref_tokens / tree_s, unit=UNIT, cores=os.cpu_count(), kind='reference',
                       sample=(f"2 requests of the {ref_tokens}-token tree through the reference's LeanGemma4.run on "
                               f"the host CPU over a 3-layer cut (sliding {run['ms_sliding_layer']} ms, global "
                               f"{run['ms_global_layer']} ms per layer), extrapolated to {len(tr.full_types)} layers"),
                       cpu=run['cpu'], threads=run['threads'])
            del tr
        except Exception as error:  # the baseline must not take the GPU number down with it
            cpu = dict(value=None, unit=UNIT, cores=os.cpu_count(), kind='reference', sample=f'failed: {error}')
    if rank == 0:
        line = dict(
            metric=METRIC, value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=ms_max, higher_is_better=True, scaling='strong' if tp else 'weak', vs_baseline=None,
            dtype='bf16',
            data='synthetic (seeded random-init weights N(0, 0.02), uniform token ids)',
            config=bench_config(args, world, desc, tokens, flops),
            model_tflops=round(trees * flops / (ms_max / 1000) / 1e12, 1),
            p50_tree_latency_ms=round(statistics.median(lat), 3),
            roofline=dict(bound='tensor', kernel=f'{kname}: gate/up projection {tokens}x43008x5376',
                          achieved=round(achieved, 1), peak=pk['bf16_sustained'], unit='TFLOP/s',
                          frac=round(achieved / pk['bf16_sustained'], 4), traffic=traffic,
                          peak_source=f"{pk['source']} sustained cuBLAS BF16 (kernel timed inside a long step)",
                          launches=len(big), avg_launch_us=round(1000 * g_ms / max(len(big), 1), 2),
                          all_gemms_tflops=round(all_tf, 1),
                          attention=dict(achieved=round(flops_attn / (attn_ms / 1000) / 1e12, 1) if attn_ms else None,
                                         peak=pk['bf16_sustained'],
                                         frac=round(flops_attn / (attn_ms / 1000) / 1e12 / pk['bf16_sustained'], 4)
                                         if attn_ms else None,
                                         unit='TFLOP/s', ms_per_tree=round(attn_ms, 3),
                                         tflop_per_tree=round(flops_attn / 1e12, 3),
                                         basis='algorithmic FLOPs (4 x Hq x d per visible pair, all layers as '
                                               'specified) / summed attention launch times of one traced tree (an '
                                               'event pair around every launch); peak: sustained cuBLAS BF16 '
                                               '(kernels timed inside a step run at its power-capped clock)',
                                         back_to_back=alone)),
            breakdown_ms={k: round(v['ms'], 3) for k, v in per_kind.items()},
            breakdown_basis=('one traced tree: a CUDA event pair around every launch, the whole tree queued behind a '
                             'device sleep first (no host latency inside a pair; the overlap of programmatic '
                             'dependent launches between kernels is lost, so the sum exceeds ms_per_step)'),
            traced_span_ms=round(trace_span, 3), graph_replay_ms=graph_ms,
            e2e=dict(value=e2e_value, unit=UNIT, h2d_bytes_per_step=int(h2d), d2h_bytes_per_step=int(d2h),
                     ms_per_step=e2e_max),
            gpu_launches=int(launches * args.steps),
            clocks=clocks.summary(), init_s=round(init_s, 1))
        if cpu is not None:
            line['cpu_baseline'] = cpu
        if parity is not None:
            line['parity'] = parity
    if world > 1 and not tp and not args.no_tp_leg and not args.layers:
        from morj_b200 import workloads as wl
        one_gpu = None
        if rank == 0:  # the latency tree on this GPU alone: the check of the sharded model's probabilities
            t_in = wl.latency_tree(seed=0)
            with torch.inference_mode():
                one_gpu = np.concatenate(model.run(model.prepare(t_in['seqs'], t_in['label_ids']),
                                                   list(range(len(t_in['seqs'])))))
        model = preps = None  # the replica's weights go back to the allocator before the sharded model loads
        torch.cuda.empty_cache()
        try:
            leg = tp_leg(args, one_gpu, top, dev, world, rank, barrier, max_over_ranks)
        except Exception as error:  # (every rank fails the same way: the pass protocol shares device errors)
            leg = dict(gpus=world, error=f'{type(error).__name__}: {error}')
        if rank == 0:
            line['tp'] = leg
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        if model is not None and model.peer is not None:  # every rank is done with the peers' buffers first
            barrier()
            model.peer.close()
            barrier()
        dist.destroy_process_group()


def attention_alone(model, p, top, reps):
    """The step's tree-attention launches (every full layer's, with the step's own tables, pool sizes and work
    lists) back to back, without the trace's per-launch events: ms per tree and TFLOP/s. Queries and pools are seeded
    random values of the step's shapes."""
    import torch
    from morj_b200 import workloads as w
    from morj_b200.lean_core import KINDS
    plan, st = p['plan'], p['plan']['steps'][0]
    t, _, n_work = p['tables'][0]
    n, hq, c = len(st['tokens']), model.hq, top['text_config']
    d = max(dd for _, dd in model.geom.values())
    g = torch.Generator(device=model.device).manual_seed(0)
    # queries and keys as the model's q/k norms leave them (entries ~ d^-1/4, unit-variance logits at scale 1)
    qk_std = d ** -0.25
    q = (torch.randn(n, hq * d, device=model.device, generator=g) * qk_std).to(torch.bfloat16)
    out = torch.empty_like(q)
    pools = {}
    for kind in set(model.types):
        kp, vp = model._kv_pool(kind, plan['cap'][KINDS[kind]])
        kp.copy_(torch.randn(kp.shape, device=model.device, generator=g) * qk_std)
        vp.copy_(torch.randn(vp.shape, device=model.device, generator=g))
        pools[kind] = (kp, vp)
    layers = model.types[:-1]  # the full layers (the last layer attends for its readout rows only)

    def tree():
        for kind in layers:
            kk = KINDS[kind]
            sliding = kind == 'sliding_attention'
            model._attention(q[:, :hq * model.geom[kind][1]], *pools[kind], out, t, 'qo', 'kv_indptr_' + kk,
                             'kv_indices_' + kk, len(st['qo_indptr']) - 1, int(st['n_bidir']) if sliding else 0,
                             kind, 'work_' + kk, n_work[kk])
    with torch.inference_mode():
        tree()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            tree()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 4 * hq * c['head_dim'] * w.attention_pairs(plan, c['sliding_window'], layers)
    return dict(ms_per_tree=round(ms, 3), launches=len(layers), tflop=round(flops / 1e12, 3),
                achieved=round(flops / (ms / 1000) / 1e12, 1),
                note='the 59 full layers\' attention launches of the bench tree, back to back, CUDA events around '
                     'the whole sequence; seeded random queries and pools of the step\'s shapes, q and k scaled as the '
                     'model\'s q/k norms leave them')


def tp_leg(args, one_gpu, top, dev, world, rank, barrier, max_over_ranks):
    """The tensor-parallel latency leg of a multi-GPU run: after the replica measurement, one latency tree (8192 +
    8 x 64 tokens) on the model sharded over all `world` GPUs with the peer-memory exchange, checked against the
    probabilities rank 0's replica computed for the same tree alone (`one_gpu`). Returns (rank 0) the leg's figures;
    every rank takes the same collective steps."""
    import torch
    import torch.distributed as dist
    from morj_b200 import workloads as w
    from morj_b200.lean_core import LeanGemma4
    tree_in = w.latency_tree(seed=0)
    seqs = list(range(len(tree_in['seqs'])))
    barrier()
    t_init = time.perf_counter()
    model = LeanGemma4.random_init(top, seed=0, device=dev, tp_group=dist.group.WORLD, tp_comm='peer')
    barrier()
    init_s = time.perf_counter() - t_init
    with torch.inference_mode():
        p = model.prepare_pass(model.prepare(tree_in['seqs'], tree_in['label_ids']), seqs)
        for _ in range(args.warmup):
            model.execute_pass(p)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            model.execute_pass(p)
        e1.record()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        got = np.concatenate(model.run(model.prepare(tree_in['seqs'], tree_in['label_ids']), seqs))
        # the bench's text tree on the sharded model, for the oracle record of the same weights and tree
        text = w.text_tree(seed=0)
        got_text = np.concatenate(model.run(model.prepare(text['seqs'], text['label_ids']),
                                            list(range(len(text['seqs'])))))
        model.trace = []
        model.execute_pass(p)
        torch.cuda.synchronize()
        trace, model.trace = model.trace, None
        reduce_ms = max_over_ranks(sum(a.elapsed_time(b) for kind, _, a, b in trace if kind == 'tp_reduce'))
    barrier()
    model.peer.close()
    barrier()
    del model
    if rank != 0:
        return None
    parity = None
    gfile = os.path.join(ROOT, 'tests', 'golden', 'oracle_31b_text.json')
    if os.path.exists(gfile):
        with open(gfile) as f:
            rec = json.load(f)
        bf = np.concatenate([np.asarray(r, np.float64) for r in rec['probs']])
        fp = np.concatenate([np.asarray(r, np.float64) for r in rec['probs_fp32']])
        parity = dict(vs='text tree on the sharded model against the oracle record of the same weights and tree '
                         '(the one-GPU line\'s parity criterion)',
                      max_abs_vs_bf16_path=float(np.abs(got_text - bf).max()),
                      max_abs_vs_fp32=float(np.abs(got_text - fp).max()),
                      bf16_path_max_abs_vs_fp32=float(np.abs(bf - fp).max()), probabilities=int(len(got_text)))
    return dict(gpus=world, workload='latency tree: 8192-token prefix + 8 branches x 64 tokens (seed 0, every rank)',
                exchange='peer memory over NVLink: row-parallel partials reduced by row owners with the norm epilogues',
                tokens=int(p['tokens']), ms_per_tree=round(ms, 3), tokens_per_s=round(p['tokens'] / (ms / 1000), 1),
                tp_reduce_ms_per_tree=round(reduce_ms, 3), steps=args.steps, warmup=args.warmup,
                max_abs_vs_1gpu=float(np.abs(got - one_gpu).max()),
                rms_vs_1gpu=float(np.sqrt(np.mean((got - one_gpu) ** 2))), init_s=round(init_s, 1),
                max_abs_note='one GPU and the sharded model sum the row-parallel projections in different orders; '
                             'over 60 BF16 layers such differences reach the order of 1e-2 (the oracle against itself '
                             'with another GEMM summation order drifts as far)',
                timing='CUDA events over the steps on every rank, max over ranks; tp_reduce from one traced tree',
                parity=parity)


if __name__ == '__main__':
    main()
