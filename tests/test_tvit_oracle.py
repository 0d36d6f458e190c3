"""Pins the TinyViT part of the oracle (oracle.c: orc_tvit_*, orc_dwconv3x3_bn)
against the reference's own code, and checks the library's host-side bias
expansion.  No GPU.

The reference runs TinyViT only on Metal (its CPU MATMUL is 2-D only,
cpu_matmul.c:196-229), so the window attention is pinned against the
reference CPU kernels applied one (window, head) slice at a time -- MUL,
TRANSPOSE, MATMUL, ADD, SOFTMAX, MATMUL, the node sequence of
tvit_window_attention (image_encoder_tinyvit.c:823-854) -- and the bias
expansion against the reference's expand_attention_bias compiled from its
source (oracle/ref_tinyvit.c)."""
import numpy as np
import pytest

import oracle as O
from _util import rel_err

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("ws", [3, 7, 14])
def test_expand_bias_matches_reference(ws):
    rng = np.random.default_rng(ws)
    comp = rng.standard_normal((4, O.tvit_n_offsets(ws))).astype(np.float32)
    assert np.array_equal(O.tvit_expand_bias(comp, ws), O.ref_tvit_expand_bias(comp, ws))


def test_expand_bias_library_matches_oracle():
    import sam3cu
    rng = np.random.default_rng(1)
    for ws in (7, 14):
        comp = rng.standard_normal((6, ws * ws)).astype(np.float32)
        dense = sam3cu.tvit_expand_bias(comp, ws)
        n = ws * ws
        assert dense.shape == (6, n, (n + 3) // 4 * 4)
        assert np.array_equal(dense[:, :, :n], O.tvit_expand_bias(comp, ws))
        assert not dense[:, :, n:].any()


def test_expand_bias_rejects_wrong_table():
    import sam3cu
    with pytest.raises(sam3cu.Sam3cuError):
        sam3cu.tvit_expand_bias(np.zeros((2, 40), np.float32), 7)


@needs_ref
@pytest.mark.parametrize("ws,heads,hd,bias", [(7, 2, 32, True), (7, 3, 32, False), (4, 2, 64, True)])
def test_window_attention_matches_reference_kernels(ws, heads, hd, bias):
    rng = np.random.default_rng(ws * 10 + heads)
    N, nw = ws * ws, 3
    qkv = rng.standard_normal((nw * N, 3 * heads * hd)).astype(np.float32)
    b = O.tvit_expand_bias(rng.standard_normal((heads, N)).astype(np.float32), ws) if bias else None
    a = O.tvit_window_attention(qkv, nw, N, heads, hd, b)
    r = O.ref_tvit_window_attention(qkv, nw, N, heads, hd, b)
    assert rel_err(a, r) < 1e-5


@needs_ref
@pytest.mark.parametrize("cb", [False, True])
def test_dwconv_bn_matches_reference(cb):
    rng = np.random.default_rng(3)
    C = 24
    x = rng.standard_normal((2, 9, 11, C)).astype(np.float32)
    w = rng.standard_normal((C, 3, 3, 1)).astype(np.float32)
    bias = rng.standard_normal(C).astype(np.float32) if cb else None
    bn = (rng.standard_normal(C).astype(np.float32), rng.standard_normal(C).astype(np.float32),
          rng.standard_normal(C).astype(np.float32), (rng.random(C) + 0.5).astype(np.float32))
    assert rel_err(O.dwconv3x3_bn(x, w, bias, bn), O.ref_dwconv3x3_bn(x, w, bias, bn)) < 1e-6
