"""The oracle's label probabilities on the 31B-class model (60 layers, hidden 5376) for the bench's text tree, with
the bench's seeded random-init weights; TEST INFRASTRUCTURE (runs on a machine with a CUDA device: the weights are
drawn by the CUDA generator exactly as `LeanGemma4.random_init` draws them, and the oracle's torch code runs there on
torch's own library kernels, never this repository's):

    python tests/golden/make_oracle_31b.py            # writes tests/golden/oracle_31b_text.json

The weights are generated on the GPU one tensor at a time in checkpoint order and consumed by the streamed oracle
(`OracleModel.streamed`) layer by layer, so the 52 GB model is never held at once.
`bench.py` compares the probabilities of its own timed tree with the recorded ones (`parity` in its JSON line), and
`tests/test_gpu_parity_31b.py` checks that the oracle run on the engine's resident weights reproduces this record.

Helpers shared with that test: `engine_fetch` (an engine's layers in the oracle's layout: gate/up de-interleaved),
`generated_model` (the streamed oracle over freshly generated weights) and `oracle_probs`.
"""
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from morj_b200 import workloads  # noqa: E402
from morj_b200.checkpoint import PREFIX, iter_random_state  # noqa: E402
from oracle.lean_oracle import OracleModel, layer_from_state  # noqa: E402

OUT = os.path.join(HERE, 'oracle_31b_text.json')
GLU_BLOCK = 128  # the engine interleaves gate/up rows in blocks of this many


def engine_fetch(model, device='cpu'):
    """(embed, norm, fetch) over a `LeanGemma4`'s resident weights: layer i in the oracle's layout (fused
    [q; k(; v)], [gate; up] with the engine's 128-row interleave undone), as copies on `device`."""
    def fetch(i):
        layer = model.layers[i]
        gu = layer['gu']
        F2, H = gu.shape
        F = F2 // 2
        blocks = gu.view(F // GLU_BLOCK, 2, GLU_BLOCK, H)
        out = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in layer.items() if k != 'gu'}
        out['gu'] = torch.cat([blocks[:, 0].reshape(F, H), blocks[:, 1].reshape(F, H)]).to(device)
        return out
    return model.embed, model.norm, fetch


def generated_model(top, seed=0, device='cuda', oracle_device='cpu'):
    """The streamed oracle (on `oracle_device`) over weights drawn as `LeanGemma4.random_init(top, seed)` draws them
    (CUDA generator, checkpoint order). Layers must be fetched in increasing order, which a forward does."""
    gen = iter_random_state(top, seed=seed, device=device)
    pending = {}

    def take(key):
        while key not in pending:
            k, t = next(gen)
            pending[k] = t
        return pending.pop(key).to(oracle_device)
    embed, norm = take(PREFIX + 'embed_tokens.weight'), take(PREFIX + 'norm.weight')
    types = top['text_config']['layer_types']
    return OracleModel.streamed(top, embed, norm, lambda i: layer_from_state(take, i, types[i]), oracle_device)


def oracle_probs(oracle, tree_in, expand=None, precision='bf16'):
    """Label probabilities of every sequence of a workload tree through the oracle's tree form: BF16 rounding where
    the reference rounds (`precision='bf16'`), or the exact model in FP32."""
    from morj_b200.tree import Tree
    images = tree_in.get('images')
    return oracle.forward_tree(Tree, tree_in['seqs'], tree_in['label_ids'], precision, images=images or None,
                               expand=expand)


def exact_library_math():
    """torch settings for an oracle run on a GPU: FP32 GEMMs in FP32 (no TF32), BF16 GEMMs reduced in FP32."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False


def main():
    """Record the oracle's probabilities for the bench tree: BF16 (the reference's rounding points) and FP32 (the
    exact model), both computed on the GPU by torch's library kernels in exact-math mode."""
    exact_library_math()
    top = workloads.gemma31b_config()
    tree_in = workloads.text_tree(seed=0)
    t0 = time.perf_counter()
    probs = {prec: oracle_probs(generated_model(top, 0, 'cuda', 'cuda'), tree_in, precision=prec)
             for prec in ('bf16', 'fp32')}
    flat = {k: [p for row in v for p in row] for k, v in probs.items()}
    rec = dict(source='oracle/lean_oracle.py tree form, streamed layer by layer, on the GPU (torch library kernels)',
               model='31B-class (workloads.gemma31b_config), LeanGemma4.random_init seed 0 (CUDA generator)',
               tree='workloads.text_tree(seed=0)', torch=torch.__version__, probs=probs['bf16'],
               probs_fp32=probs['fp32'],
               bf16_vs_fp32_max_abs=max(abs(a - b) for a, b in zip(flat['bf16'], flat['fp32'])),
               seconds=round(time.perf_counter() - t0, 1))
    with open(OUT, 'w') as f:
        json.dump(rec, f)
    print('wrote', OUT, rec['seconds'], 's; BF16 vs FP32 max abs', rec['bf16_vs_fp32_max_abs'])


if __name__ == '__main__':
    main()
