"""The reference's own TinyViT graph (sam3_tinyvit_build, compiled from
image_encoder_tinyvit.c into oracle/_ref) evaluated through the CUDA
backend vtable: every node, including the batched 4-D MATMULs, SOFTMAX,
BATCHNORM, BIAS_ADD, CONCAT (padding) and the depthwise CONV2Ds, lowered to
device kernels.  The graph is F32, so it is compared with the oracle's F32
restatement at 1e-4 normwise, and with the fused sam3cu_tinyvit encoder at
1e-2 (16-bit operands there).  The reference CPU backend cannot run this
graph (its MATMUL is 2-D only), which this test also records."""
import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("img", [112, 224])
def test_reference_tinyvit_graph_on_cuda_backend(cuda, img):
    import sam3cu
    cfg = synth.tiny_tinyvit_cfg(img)
    w = synth.tinyvit_weights(cfg, seed=7)
    cs, ws, keep = sam3cu.tinyvit_structs(cfg, w)
    image = synth.tinyvit_images(cfg, 1, seed=8)[0]
    got = O.ref_tinyvit_encode(cs, ws, image, sam3cu.backend_ops(), sam3cu.CUDA_BACKEND_SIZE,
                               sam3cu.CUDA_BACKEND_TYPE)
    assert sam3cu.device_error() == 0
    ref = O.tinyvit_forward(cs, ws, image)
    assert rel_err(got, ref) < 1e-4, rel_err(got, ref)
    tv = sam3cu.TinyViT(cfg, w, sam3cu.F16, max_batch=1)
    fused = tv.encode_host(image[None])[0]
    tv.close()
    assert rel_err(fused, got) < 1e-2


@needs_ref
def test_reference_cpu_backend_cannot_run_tinyvit(cuda):
    import sam3cu
    cfg = synth.tiny_tinyvit_cfg(112)
    w = synth.tinyvit_weights(cfg, seed=7)
    cs, ws, keep = sam3cu.tinyvit_structs(cfg, w)
    image = synth.tinyvit_images(cfg, 1, seed=8)[0]
    with pytest.raises(RuntimeError):
        O.ref_tinyvit_encode(cs, ws, image)
