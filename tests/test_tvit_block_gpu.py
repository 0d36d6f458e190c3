"""GPU parity of the TinyViT block (sam3cu_tvit_block_*) and MBConv
(sam3cu_tvit_mbconv_*) against the oracle's restatements of
tvit_block_forward / tvit_mbconv_forward (image_encoder_tinyvit.c), with
seeded random weights (linears ~N(0, 0.02)-style scaled by 1/sqrt(K), BN
running stats mean 0-ish / var ~1).  Shapes include padding (H, W not
multiples of the window) and the 1008px stage widths.  Tolerance 1e-2
normwise on the updated residual stream."""
import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu


def block_weights(C, heads, ws, mlp, seed):
    rng = np.random.default_rng(seed)
    n = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)
    return {
        "attn_norm_w": 1 + n(C, sc=0.1), "attn_norm_b": n(C, sc=0.1),
        "qkv_w": n(3 * C, C, sc=C ** -0.5), "qkv_b": n(3 * C, sc=0.1),
        "proj_w": n(C, C, sc=C ** -0.5), "proj_b": n(C, sc=0.1),
        "attn_bias": n(heads, ws * ws),
        "lc_w": n(C, 3, 3, 1, sc=0.3), "lc_b": None,
        "lc_bn_w": 1 + n(C, sc=0.1), "lc_bn_b": n(C, sc=0.1), "lc_bn_mean": n(C, sc=0.1),
        "lc_bn_var": (1 + rng.random(C)).astype(np.float32),
        "mlp_norm_w": 1 + n(C, sc=0.1), "mlp_norm_b": n(C, sc=0.1),
        "fc1_w": n(mlp, C, sc=C ** -0.5), "fc1_b": n(mlp, sc=0.1),
        "fc2_w": n(C, mlp, sc=mlp ** -0.5), "fc2_b": n(C, sc=0.1),
    }


def mbconv_weights(C, mid, seed):
    rng = np.random.default_rng(seed)
    n = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)
    w = {}
    for i, (o, k) in enumerate(((mid, C), (mid, 9), (C, mid)), 1):
        shape = (o, 1, 1, k) if i != 2 else (o, 3, 3, 1)
        w[f"conv{i}_w"] = n(*shape, sc=k ** -0.5)
        w[f"conv{i}_b"] = None
        w[f"bn{i}_w"] = 1 + n(o, sc=0.1)
        w[f"bn{i}_b"] = n(o, sc=0.1)
        w[f"bn{i}_mean"] = n(o, sc=0.1)
        w[f"bn{i}_var"] = (1 + rng.random(o)).astype(np.float32)
    return w


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,H,W,C,heads,ws", [
    (2, 14, 14, 64, 2, 7),    # no padding
    (1, 17, 20, 96, 3, 7),    # padded on both sides
    (1, 32, 32, 192, 6, 14),  # stage-2-like window 14, padded (32 -> 42)
])
def test_tvit_block(cuda, dt, B, H, W, C, heads, ws):
    import torch
    import sam3cu
    mlp = 4 * C
    w = block_weights(C, heads, ws, mlp, seed=C + ws)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((B, H, W, C)).astype(np.float32)
    blk = sam3cu.TvitBlock(C, heads, ws, mlp, w, sam3cu.BF16 if dt == "bf16" else sam3cu.F16)
    xd = torch.from_numpy(x).cuda()
    blk.forward(xd)
    torch.cuda.synchronize()
    assert sam3cu.device_error() == 0
    wo = dict(w)
    wo["attn_bias"] = O.tvit_expand_bias(w["attn_bias"], ws)
    ref = np.stack([O.tvit_block_forward(wo, x[b], heads, ws) for b in range(B)])
    assert rel_err(to_np(xd), ref) < 1e-2
    blk.close()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,H,W,C", [(2, 16, 16, 64), (1, 63, 63, 96)])
def test_tvit_mbconv(cuda, dt, B, H, W, C):
    import torch
    import sam3cu
    mid = 4 * C
    w = mbconv_weights(C, mid, seed=C)
    x = np.random.default_rng(2).standard_normal((B, H, W, C)).astype(np.float32)
    mb = sam3cu.TvitMBConv(C, mid, w, sam3cu.BF16 if dt == "bf16" else sam3cu.F16)
    xd = torch.from_numpy(x).cuda()
    mb.forward(xd)
    mb.forward(xd)  # two blocks in a row (the second reuses the 16-bit copy path)
    torch.cuda.synchronize()
    assert sam3cu.device_error() == 0
    ref = O.tvit_mbconv_forward(w, O.tvit_mbconv_forward(w, x))
    assert rel_err(to_np(xd), ref) < 1e-2
    mb.close()
