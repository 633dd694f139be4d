"""Parity at the configuration the headline is quoted on: the whole 60-layer 31B-class model (hidden 5376, 32 / 16
heads of 128, GeGLU 21504, vocabulary 262144, 5 sliding-1024 : 1 global layers) on the text tree of the bench
(1500 + 3 x 3 x 60 tokens), the multimodal tree (8 x 560 image rows + 300 + 2 x 4 x 40 tokens, a 255-label and a
2-label question) and the latency tree (8192 + 8 x 64 tokens).

References: the oracle (`oracle/lean_oracle.py`, the reference's lean path `aleria_judge/lean_core.py:599-737` and
readout `558-561` restated) on the engine's own weights, run on the GPU by torch's library kernels in exact-math mode,
in BF16 with the reference's rounding points ("the reference's BF16 lean path") and in FP32 (the exact model).

Over 60 layers two correct BF16 implementations do not agree to 1e-2: every layer's BF16 roundings of the residual
stream depend on FP32 summation order, and the differences accumulate (the oracle against itself with another GEMM
summation order drifts as far from itself as the engine drifts from it). So the checks are:
  * per layer: engine layer i fed the oracle's inputs (x_i, h_i) gives the oracle's x_{i+1} to BF16 rounding
    (relative norm error <= LAYER_TOL on every one of the 59 full layers) - a wrong kernel or epilogue shows here;
  * end to end: the engine's probabilities are no further from the exact model than the reference's BF16 path's are
    (max |engine - FP32| <= 1.5 x max |BF16 path - FP32| + 2e-3), and within 1e-2 of the BF16 path or within twice
    that path's own distance from the exact model, whichever is larger.
The measured numbers are printed with `-s`.
"""
import json
import os

import numpy as np
import pytest
import torch

from morj_b200 import workloads

pytestmark = pytest.mark.gpu

TOL = 1e-2
LAYER_TOL = 8e-3
HERE = os.path.dirname(os.path.abspath(__file__))


def flat(rows):
    return np.concatenate([np.asarray(r, dtype=np.float64) for r in rows])


@pytest.fixture(scope='module')
def model():
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from make_oracle_31b import exact_library_math
    from morj_b200.lean_core import LeanGemma4
    exact_library_math()
    m = LeanGemma4.random_init(workloads.gemma31b_config(), seed=0, device='cuda')
    yield m
    del m
    torch.cuda.empty_cache()


def run_engine(m, tree_in):
    images = [f.cuda() for f in tree_in['images']] if tree_in['images'] else None
    req = m.prepare(tree_in['seqs'], tree_in['label_ids'], images=images)
    return flat(m.run(req, list(range(len(tree_in['seqs'])))))


def oracle(m, top):
    from make_oracle_31b import engine_fetch
    from oracle.lean_oracle import OracleModel
    embed, norm, fetch = engine_fetch(m, device='cuda')
    return OracleModel.streamed(top, embed, norm, fetch, device='cuda')


def oracle_flat(m, top, tree_in, precision):
    from make_oracle_31b import oracle_probs
    from morj_b200.lean_core import expand_images
    return flat(oracle_probs(oracle(m, top), tree_in, expand=expand_images, precision=precision))


def check_probs(name, got, bf, fp):
    d_ref = np.abs(bf - fp).max()
    d_eng = np.abs(got - fp).max()
    d_pair = np.abs(got - bf).max()
    print(f'\n{name}: max |engine - BF16 path| = {d_pair:.3e}, max |engine - FP32| = {d_eng:.3e}, '
          f'max |BF16 path - FP32| = {d_ref:.3e} (rms {np.sqrt(np.mean((got - fp) ** 2)):.3e} / '
          f'{np.sqrt(np.mean((bf - fp) ** 2)):.3e}) over {len(got)} probabilities')
    assert d_eng <= 1.5 * d_ref + 2e-3, (d_eng, d_ref)
    assert d_pair <= max(TOL, 2 * d_ref), (d_pair, d_ref)


def per_layer_errors(m, top, tree_in):
    """Relative norm error of x after each full layer when the engine's layer i runs on the oracle's (x_i, h_i)."""
    import oracle.lean_oracle as lo
    from morj_b200.lean_core import KINDS
    req = m.prepare(tree_in['seqs'], tree_in['label_ids'])
    p = m.prepare_pass(req, list(range(len(tree_in['seqs']))))
    plan = p['plan']
    st = plan['steps'][0]
    t, _, n_work = p['tables'][0]
    n, H, bf, dev = len(st['tokens']), m.hidden, torch.bfloat16, m.device
    d = max(dd for _, dd in m.geom.values())
    bufs = dict(x=torch.empty(n, H, dtype=bf, device=dev), h=torch.empty(n, H, dtype=bf, device=dev),
                q=torch.empty(n, m.hq * d, dtype=bf, device=dev), attn=torch.empty(n, m.hq * d, dtype=bf, device=dev),
                o=torch.empty(n, H, dtype=bf, device=dev),
                act=torch.empty(n, m.layers[0]['gu'].shape[0] // 2, dtype=bf, device=dev),
                nb=int(st['n_bidir']), n_seg=len(st['qo_indptr']) - 1)
    for kind in set(m.types):
        m._rope(kind, int(np.max(st['positions'])))
    pools = {kind: m._kv_pool(kind, plan['cap'][KINDS[kind]]) for kind in set(m.types)}
    orc = oracle(m, top)
    rope = {k: lo.rope_tables(st['positions'], v) for k, v in orc.inv.items()}
    xo = orc.embed_rows(st['tokens'])
    ho = lo._r(lo.rmsnorm(xo, orc.layers[0]['in_ln'], m.eps), True)
    errs = []
    with torch.inference_mode():
        for i in range(len(m.layers) - 1):
            bufs['x'].copy_(xo.to(bf))
            bufs['h'].copy_(ho.to(bf))
            m._layer(i, t, n_work, pools[m.types[i]], bufs)
            xo, ho, _ = orc.layer(i, xo, ho, st, plan['cap'], rope)
            errs.append(float((bufs['x'].float() - xo).norm() / xo.norm()))
    from morj_b200 import _native as nat
    assert nat.device_error(m._stream()) == 0
    return errs


def test_text_tree_every_layer_matches_the_oracle_given_the_same_input(model):
    top = workloads.gemma31b_config()
    errs = per_layer_errors(model, top, workloads.text_tree(seed=0))
    worst = int(np.argmax(errs))
    print(f'\nper-layer relative error of x, engine layer on the oracle input: max {errs[worst]:.3e} (layer {worst}), '
          f'median {np.median(errs):.3e}, over {len(errs)} layers')
    assert max(errs) <= LAYER_TOL, errs


def test_text_tree_60_layers(model):
    top = workloads.gemma31b_config()
    tree_in = workloads.text_tree(seed=0)
    got = run_engine(model, tree_in)
    bf, fp = oracle_flat(model, top, tree_in, 'bf16'), oracle_flat(model, top, tree_in, 'fp32')
    check_probs('31B text tree, 60 layers', got, bf, fp)
    # the record bench.py compares its own tree against is this oracle on these weights
    with open(os.path.join(HERE, 'golden', 'oracle_31b_text.json')) as f:
        rec = json.load(f)
    assert np.abs(flat(rec['probs']) - bf).max() <= 1e-6 and np.abs(flat(rec['probs_fp32']) - fp).max() <= 1e-6


def test_multimodal_tree_60_layers(model):
    top = workloads.gemma31b_config()
    tree_in = workloads.multimodal_tree(seed=0)
    got = run_engine(model, tree_in)
    assert len(got) == 4 * 255 + 4 * 2
    bf, fp = oracle_flat(model, top, tree_in, 'bf16'), oracle_flat(model, top, tree_in, 'fp32')
    check_probs('31B multimodal tree, 60 layers', got, bf, fp)


def test_latency_tree_60_layers(model):
    top = workloads.gemma31b_config()
    tree_in = workloads.latency_tree(seed=0)
    got = run_engine(model, tree_in)
    bf, fp = oracle_flat(model, top, tree_in, 'bf16'), oracle_flat(model, top, tree_in, 'fp32')
    check_probs('31B latency tree, 60 layers', got, bf, fp)
