"""Host side of the image path (`morj_b200/vision.py`): the pooled cells and their patch rows match transformers'
`Gemma4VisionPooler` (the reference's vision tower, `aleria_judge/lean_core.py:752-781`) on the patch layouts its
image processor produces, padding included; no GPU."""
import numpy as np
import pytest
import torch

from morj_b200.vision import pool_cells


def processed(sizes, seed=0):
    from PIL import Image
    from transformers.models.gemma4.image_processing_gemma4 import Gemma4ImageProcessor
    rng = np.random.default_rng(seed)
    imgs = [Image.fromarray((rng.random((h, w, 3)) * 255).astype(np.uint8)) for h, w in sizes]
    return Gemma4ImageProcessor()(imgs, return_tensors='pt')


@pytest.mark.parametrize('sizes', [[(200, 300), (64, 64)], [(480, 640)], [(37, 500), (500, 37), (128, 128)]])
def test_pool_cells_match_the_reference_pooler(sizes):
    from transformers.models.gemma4.configuration_gemma4 import Gemma4VisionConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4VisionPooler
    p = processed(sizes)
    pos = p['image_position_ids']
    B, P, _ = pos.shape
    k = 3
    length = P // (k * k)
    H = 16
    g = torch.Generator().manual_seed(1)
    hidden = torch.randn(B, P, H, generator=g)
    padding = (pos == -1).all(-1)
    pooler = Gemma4VisionPooler(Gemma4VisionConfig(hidden_size=H))
    ref, mask = pooler(hidden.clone(), pos, padding, output_length=length)
    want = ref[mask]  # the reference's kept cells, image by image
    got, counts = [], []
    for b in range(B):
        kept, indptr, rows = pool_cells(pos[b].numpy(), length, k)
        counts.append(len(kept))
        assert (mask[b].nonzero().flatten().numpy() == kept).all()
        for c in range(len(kept)):
            got.append(hidden[b, torch.as_tensor(rows[indptr[c]:indptr[c + 1]])].sum(0) / (k * k) * H ** 0.5)
    assert counts == p['num_soft_tokens_per_image'].tolist()
    torch.testing.assert_close(torch.stack(got), want, rtol=1e-5, atol=1e-5)
