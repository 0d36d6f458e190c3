"""The reference's own FPN neck graph (sam3_neck_build, compiled from
necks.c into oracle/_ref) evaluated through the CUDA backend vtable: the
ConvTranspose2d stages (GEMM + pixel shuffle), MaxPool2d, the 1x1 and 3x3
CONV2Ds and BIAS_ADDs all lowered to device kernels.  The graph is F32, so
it is compared with the oracle's restatement at 1e-4 normwise."""
import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("grid,d,dim", [(6, 32, 64), (9, 64, 128), (12, 32, 64)])
def test_reference_neck_graph_on_cuda_backend(cuda, grid, d, dim):
    import sam3cu
    scales = (4.0, 2.0, 1.0, 0.5)
    w = synth.neck_weights(d, dim, scales, seed=grid)
    feat = np.random.default_rng(grid).standard_normal((grid * grid, dim)).astype(np.float32)
    got = O.ref_neck(d, dim, grid, scales, w, feat, sam3cu.backend_ops(), sam3cu.CUDA_BACKEND_SIZE,
                     sam3cu.CUDA_BACKEND_TYPE)
    assert sam3cu.device_error() == 0
    ref = O.neck_forward(d, dim, grid, scales, w, feat)
    for a, r in zip(got, ref):
        assert a.shape == r.shape
        assert rel_err(a, r) < 1e-4, rel_err(a, r)
