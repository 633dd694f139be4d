"""The image path on the GPU (`morj_b200/vision.py`) against the reference's own image path: transformers'
`Gemma4VisionModel` + `Gemma4MultimodalEmbedder` (what the reference's `VisionEncoder`, `aleria_judge/lean_core.py:
745-781`, runs), on a seeded random-init tower (4 layers, hidden 256, 4 heads of 64, GeGLU 512, pooling 3) and the
transformers image processor's patch layout for images of several sizes (so padding patches and partial cells occur).

Bar: the soft tokens' relative norm error against the FP32 reference is no larger than the BF16 reference's own
(x 1.5, + 5e-3), and below 3e-2; the soft-token counts equal the processor's."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

VCFG = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=4,
            num_key_value_heads=4, head_dim=64, rms_norm_eps=1e-6, pooling_kernel_size=3, patch_size=16,
            position_embedding_size=10240, rope_parameters={'rope_type': 'default', 'rope_theta': 100.0},
            use_clipped_linears=False, standardize=False, hidden_activation='gelu_pytorch_tanh')
TEXT_HIDDEN = 512


def random_state(seed=0):
    """Checkpoint-layout tensors (`model.vision_tower.*`, `model.embed_vision.*`) for the transformers modules,
    every parameter drawn from a seeded generator: matrices N(0, 0.02), the position table N(0, 0.3), norms
    1 + N(0, 0.1), the q/k norms further scaled by head_dim^-1/4."""
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig, Gemma4VisionConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4MultimodalEmbedder, Gemma4VisionModel
    vc = Gemma4VisionConfig(**VCFG)
    tower, embedder = Gemma4VisionModel(vc), Gemma4MultimodalEmbedder(vc, Gemma4TextConfig(hidden_size=TEXT_HIDDEN))
    g = torch.Generator().manual_seed(seed)
    state = {}
    for prefix, module in (('model.vision_tower.', tower), ('model.embed_vision.', embedder)):
        for k, v in module.state_dict().items():
            if v.dim() == 1:
                t = 1 + 0.1 * torch.randn(v.shape, generator=g)
                if k.endswith(('q_norm.weight', 'k_norm.weight')):
                    # attention runs with scale 1 (the q/k norms carry it): unit-variance logits, not one-hot ones
                    t = t * v.shape[0] ** -0.25
            elif 'position_embedding_table' in k:
                t = 0.3 * torch.randn(v.shape, generator=g)
            else:
                t = 0.02 * torch.randn(v.shape, generator=g)
            state[prefix + k] = t.to(torch.bfloat16)
    return vc, state


def reference(vc, state, pixel_values, position_ids, dtype):
    """transformers' tower + embedder in `dtype` (eager attention), the reference's path after the processor."""
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4MultimodalEmbedder, Gemma4VisionModel
    vc._attn_implementation = 'eager'
    tower = Gemma4VisionModel(vc).to(dtype).eval()
    embedder = Gemma4MultimodalEmbedder(vc, Gemma4TextConfig(hidden_size=TEXT_HIDDEN)).to(dtype).eval()
    for prefix, module in (('model.vision_tower.', tower), ('model.embed_vision.', embedder)):
        sub = {k[len(prefix):]: v.to(dtype) for k, v in state.items() if k.startswith(prefix)}
        missing, unexpected = module.load_state_dict(sub, strict=False)
        assert not missing and not unexpected, (missing, unexpected)
    with torch.no_grad():
        h = tower(pixel_values=pixel_values.to(dtype), pixel_position_ids=position_ids).last_hidden_state
        return embedder(inputs_embeds=h).reshape(-1, TEXT_HIDDEN).float()


def processed(sizes, seed=0):
    from PIL import Image
    from transformers.models.gemma4.image_processing_gemma4 import Gemma4ImageProcessor
    rng = np.random.default_rng(seed)
    imgs = [Image.fromarray((rng.random((h, w, 3)) * 255).astype(np.uint8)) for h, w in sizes]
    return imgs, Gemma4ImageProcessor()


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.parametrize('sizes', [[(200, 300), (64, 64)], [(37, 500)]])
def test_vision_tower_matches_transformers(sizes):
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from morj_b200.vision import VisionEncoder, VisionTower
    vc, state = random_state()
    imgs, processor = processed(sizes)
    tower = VisionTower(dict(VCFG), TEXT_HIDDEN, lambda k: state[k], 'cuda')
    p = processor(imgs, return_tensors='pt')
    got, counts = tower.forward(p['pixel_values'], p['image_position_ids'])
    assert counts == p['num_soft_tokens_per_image'].tolist()
    # the reference's pixels reach the tower in BF16 (`lean_core.py:778`)
    pv = p['pixel_values'].to(torch.bfloat16)
    fp = reference(vc, state, pv, p['image_position_ids'], torch.float32)
    bf = reference(vc, state, pv, p['image_position_ids'], torch.bfloat16)
    assert got.shape == fp.shape
    e_got, e_bf = rel(got.cpu(), fp), rel(bf, fp)
    print(f'\nvision tower {sizes}: relative error vs FP32 {e_got:.3e} (transformers BF16: {e_bf:.3e}), '
          f'vs BF16 {rel(got.cpu(), bf):.3e}, {got.shape[0]} soft tokens')
    assert e_got <= 1.5 * e_bf + 5e-3 and e_got < 3e-2
    # the same through the drop-in encoder (processor on the host, per-image tensors)
    enc = VisionEncoder.from_parts(processor, tower, batch=len(imgs))
    feats = enc.encode(imgs)
    assert [f.shape[0] for f in feats] == counts
    assert torch.equal(torch.cat(feats), got)
