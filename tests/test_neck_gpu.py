"""The native FPN neck (sam3cu_neck_*, the sam3_neck_build pipeline with
fused GEMM epilogues) against the oracle's restatement of the reference
neck (pinned to the reference's own sam3_neck_build in
test_neck_oracle.py).  16-bit compute with F32 accumulation: the north-star
bound 1e-2 (normwise) for BF16 / F16."""
import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu


# grid 8 with d_model 64: the 4x stage (32x32x64) runs the 3x3 conv as an
# implicit GEMM (4x32-pixel blocks straight from the NHWC map); the other
# stages and cases run im2col + GEMM
@pytest.mark.parametrize("grid,d,dim,dt", [(6, 32, 64, "bf16"), (9, 64, 128, "bf16"), (12, 32, 64, "f16"),
                                           (8, 64, 128, "bf16"), (8, 64, 128, "f16")])
def test_neck_matches_oracle(cuda, grid, d, dim, dt):
    import torch
    import sam3cu
    scales = (4.0, 2.0, 1.0, 0.5)
    w = synth.neck_weights(d, dim, scales, seed=grid)
    n = 2
    feats = np.random.default_rng(grid).standard_normal((n, grid * grid, dim)).astype(np.float32)
    code = sam3cu.BF16 if dt == "bf16" else sam3cu.F16
    rnd = O.round_bf16 if dt == "bf16" else O.round_fp16
    neck = sam3cu.FpnNeck(d, dim, grid, scales, w, code, max_batch=n)
    outs = neck.forward(torch.from_numpy(feats).cuda())
    neck.close()
    assert sam3cu.device_error() == 0
    # reference on the 16-bit-rounded weights and inputs
    wr = {"w": [[rnd(a) for a in ws] for ws in w["w"]], "b": w["b"]}
    for b in range(n):
        ref = O.neck_forward(d, dim, grid, scales, wr, rnd(feats[b]))
        for i, (o, r) in enumerate(zip(outs, ref)):
            got = o[b].cpu().numpy()
            assert got.shape == r.shape
            assert rel_err(got, r) < 1e-2, (b, i, rel_err(got, r))


def test_neck_full_size_matches_oracle(cuda):
    """The SAM3 configuration the bench times (72x72x1024 -> 288/144/72/36
    at d_model 256; the 288^2 3x3 conv runs as the implicit GEMM), one
    image, BF16, against the oracle's restatement of sam3_neck_build on the
    bf16-rounded weights and input, at 1e-2 per output scale."""
    import torch
    import sam3cu
    scales = (4.0, 2.0, 1.0, 0.5)
    w = synth.neck_weights(256, 1024, scales, seed=1)
    neck = sam3cu.FpnNeck(256, 1024, 72, scales, w, sam3cu.BF16, max_batch=1)
    assert neck.sizes == [288, 144, 72, 36]
    feat = np.random.default_rng(5).standard_normal((1, 5184, 1024)).astype(np.float32)
    outs = neck.forward(torch.from_numpy(feat).cuda())
    neck.close()
    assert sam3cu.device_error() == 0
    wr = {"w": [[O.round_bf16(a) for a in ws] for ws in w["w"]], "b": w["b"]}
    ref = O.neck_forward(256, 1024, 72, scales, wr, O.round_bf16(feat[0]))
    for i, (o, r, s) in enumerate(zip(outs, ref, (288, 144, 72, 36))):
        assert o.shape == (1, s, s, 256)
        assert rel_err(o[0].cpu().numpy(), r) < 1e-2, (i, rel_err(o[0].cpu().numpy(), r))
