"""The drop-in path end to end: the reference's own sam3_vit_build
(compiled from the sam3.c sources into dropin/_ref) evaluating its F32
Hiera-L graph through sam3_cuda_backend_ops(), host buffers in and out, as
a sam3.c build with the CUDA backend registered runs it.  Compared with the
committed goldens of the reference on its CPU backend
(tests/golden/vit_1008_depth{8,32}.npz) at the north star's F32 bound,
1e-4 normwise, on the fixture's sampled positions.  The session keeps the
weights on the device across images (as a sam3_ctx does), so the second
encode of the same image must repeat the first."""
import os
import sys

import numpy as np
import pytest

import synth
from _util import rel_err

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "dropin"))
GOLD = os.path.join(ROOT, "tests", "golden")


def _gold(depth):
    p = os.path.join(GOLD, f"vit_1008_depth{depth}.npz")
    if not os.path.exists(p):
        pytest.skip(f"{p} absent")
    g = np.load(p)
    cfg = dict(zip(("img_size", "patch_size", "embed_dim", "depth", "n_heads", "window_size", "mlp_dim"),
                   (int(v) for v in g["cfg"])))
    w_seed, img_seed = (int(v) for v in g["seeds"])
    return g, cfg, synth.vit_weights(cfg, seed=w_seed), synth.images(cfg, 1, seed=img_seed)[0]


@pytest.mark.parametrize("depth", [8, 32])
def test_reference_encoder_on_cuda_backend_vs_golden(cuda, depth):
    import dropin as D
    import sam3cu
    if not D.available():
        pytest.skip("dropin/_ref/libsam3_dropin.so not built")
    g, cfg, w, img = _gold(depth)
    dv = D.DropinVit(cfg, w, 0)
    del w
    out1, _ = dv.encode(img)
    out2, _ = dv.encode(img)
    dv.close()
    assert sam3cu.device_error() == 0
    err = rel_err(out1.ravel()[g["idx"]], g["f32_sample"])
    assert err < 1e-4, err
    # the second image reuses the cached weights and the grown arena
    assert rel_err(out2, out1) < 1e-6
