"""Full-size encoder parity against committed golden fixtures of the
reference itself (tests/golden/vit_1008_depth{8,32}.npz, made by
tests/golden/gen_vit_golden.py from the reference sam3_vit_build on its CPU
backend): Hiera-L geometry at 1008 px, 8 blocks (block 7 global) and the
full 32 blocks (globals 7/15/23/31), seeded weights and image.  Compared on the fixture's 16384 sampled positions,
normwise: BF16 / F16 / Q8 encoders within 1e-2, the F32 graph through the
CUDA backend vtable within 1e-4."""
import os

import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vit_1008_depth{}.npz")


@pytest.fixture(scope="module", params=[8, 32], ids=["depth8", "depth32"])
def gold(request):
    path = GOLD.format(request.param)
    if not os.path.exists(path):
        pytest.skip(f"{path} absent")
    g = np.load(path)
    cfg = dict(zip(("img_size", "patch_size", "embed_dim", "depth", "n_heads", "window_size", "mlp_dim"),
                   (int(v) for v in g["cfg"])))
    w_seed, img_seed = (int(v) for v in g["seeds"])
    return g, cfg, synth.vit_weights(cfg, seed=w_seed), synth.images(cfg, 1, seed=img_seed)


@pytest.mark.parametrize("wd,ref", [("bf16", "bf16"), ("q8", "q8"), ("f16", "f32")])
def test_encoder_vs_reference_golden(cuda, gold, wd, ref):
    import sam3cu
    g, cfg, w, img = gold
    code = {"bf16": sam3cu.BF16, "q8": sam3cu.Q8_0, "f16": sam3cu.F16}[wd]
    enc = sam3cu.VitEncoder(cfg, w, code, max_batch=1)
    out = enc.encode_host(img)[0].ravel()
    enc.close()
    assert sam3cu.device_error() == 0
    assert rel_err(out[g["idx"]], g[f"{ref}_sample"]) < 1e-2


def test_f32_graph_through_backend_vs_reference_golden(cuda, gold):
    if not O.ref_available():
        pytest.skip("oracle/_ref (the reference model code that builds the graph) not built")
    import sam3cu
    g, cfg, w, img = gold
    out = O.ref_vit_encode_backend(cfg, w, img[0], sam3cu.backend_ops(), sam3cu.CUDA_BACKEND_SIZE,
                                   sam3cu.CUDA_BACKEND_TYPE).ravel()
    assert rel_err(out[g["idx"]], g["f32_sample"]) < 1e-4
