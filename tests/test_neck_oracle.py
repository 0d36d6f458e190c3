"""Pins the FPN-neck restatement (oracle.c: orc_neck_forward) against the
reference's own sam3_neck_build (necks.c, compiled from source) on its CPU
backend -- ConvTranspose2d, MaxPool, Conv2d and BIAS_ADD kernels of the
reference -- at a small grid with all four scale stages.  No GPU."""
import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("grid", [6, 9])
def test_neck_restatement_matches_reference(grid):
    d, dim, scales = 32, 64, (4.0, 2.0, 1.0, 0.5)
    w = synth.neck_weights(d, dim, scales, seed=grid)
    feat = np.random.default_rng(grid).standard_normal((grid * grid, dim)).astype(np.float32)
    ours = O.neck_forward(d, dim, grid, scales, w, feat)
    ref = O.ref_neck(d, dim, grid, scales, w, feat)
    for a, r in zip(ours, ref):
        assert a.shape == r.shape
        assert rel_err(a, r) < 1e-5
