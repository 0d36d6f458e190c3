"""GPU parity of the whole TinyViT backbone (sam3cu_tinyvit_*) against the
oracle's restatement of sam3_tinyvit_build (image_encoder_tinyvit.c:
1058-1290) on seeded random weights: patch embed, MBConv layer, three
PatchMerging steps, window-attention layers (7x7 and 14x14 windows, with
padding) and the projection head.  Tolerance 1e-2 normwise."""
import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("img", [112, 224])
def test_tinyvit_backbone(cuda, dt, img):
    import sam3cu
    cfg = synth.tiny_tinyvit_cfg(img)
    w = synth.tinyvit_weights(cfg, seed=img)
    imgs = synth.tinyvit_images(cfg, 2, seed=3)
    tv = sam3cu.TinyViT(cfg, w, sam3cu.F16 if dt == "f16" else sam3cu.BF16, max_batch=2)
    out = tv.encode_host(imgs)
    assert sam3cu.device_error() == 0
    cs, ws, keep = sam3cu.tinyvit_structs(cfg, w)
    for i in range(2):
        ref = O.tinyvit_forward(cs, ws, imgs[i])
        assert rel_err(out[i], ref) < 1e-2, (i, rel_err(out[i], ref))
    tv.close()


def test_tinyvit_21m_1008px_matches_oracle(cuda):
    """BASELINE config 5's architecture at its stated size: TinyViT-21M at
    1008 px (stage grids 252 / 126 / 63->70 padded for the 14x14 windows /
    32), F16, two images in one batch, each against the oracle's
    restatement of sam3_tinyvit_build at the north-star bound 1e-2."""
    import sam3cu
    cfg = dict(synth.TINYVIT_21M)
    w = synth.tinyvit_weights(cfg, seed=0)
    imgs = synth.tinyvit_images(cfg, 2, seed=1)
    tv = sam3cu.TinyViT(cfg, w, sam3cu.F16, max_batch=2)
    out = tv.encode_host(imgs)
    assert sam3cu.device_error() == 0
    assert tv.grid == 32 and out.shape == (2, 1024, 1024)
    tv.close()
    cs, ws, keep = sam3cu.tinyvit_structs(cfg, w)
    for i in range(2):
        ref = O.tinyvit_forward(cs, ws, imgs[i])
        assert rel_err(out[i], ref) < 1e-2, (i, rel_err(out[i], ref))
