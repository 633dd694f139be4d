"""Record the reference lean path's label probabilities on the tiny random-init model (run where the reference
source is available; nothing here runs on a GPU):

    python tests/golden/make_forward_golden.py /path/to/reference

The reference's own `LeanGemma4.prepare` / `run` / `_step` / `_last_layer` (`aleria_judge/lean_core.py:428-737`) run
on the CPU with: its Triton kernels in Triton's interpreter (TRITON_INTERPRET=1, with FP32 -> BF16 conversions
rounded to nearest even as the compiled kernels do), and the stand-ins of `oracle/ref_cpu.py` for the GPU-only
FlashInfer calls (written from FlashInfer's documented semantics: paged prefill over page-size-1 pages with the
bottom-right causal mask, `window_left`, `custom_mask`, GQA and `sm_scale`; `rmsnorm`; `gelu_tanh_and_mul`). The
same weights also go through transformers' `Gemma4ForCausalLM` in FP32, one branch at a time.

Writes `tests/golden/forward_tiny.json`: per case the request, the reference's probabilities, and (text cases) the
transformers FP32 probabilities, plus a checksum of the seeded weights so a test can tell if they drifted.
"""
import json
import os
import sys

os.environ['TRITON_INTERPRET'] = '1'

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from morj_b200 import workloads  # noqa: E402
from morj_b200.checkpoint import PREFIX, random_state  # noqa: E402
from oracle.ref_cpu import load_reference, reference_model  # noqa: E402


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
    ref_root = sys.argv[1] if len(sys.argv) > 1 else None
    lean_core = load_reference(ref_root, eager=False)  # the reference's Triton kernels, interpreted
    round_bf16_like_the_gpu()
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
