"""Pins the CPU oracle (oracle/oracle.c) -- the checker every GPU parity test
relies on -- against (a) the known-answer values of the reference's own unit
tests and (b) the reference CPU backend itself, compiled from the sam3.c
sources into oracle/_ref/libsam3_ref.so (skipped where it was not built)."""
import numpy as np
import pytest

import oracle as O
from _util import rel_err

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


# ---- (a) known answers from the reference test-suite
def test_gelu_known_values():
    # tests/test_cpu_kernels.c:264-288 (tanh form, 1e-3)
    y = O.gelu(np.array([0.0, 1.0, -1.0, 2.0], np.float32))
    assert np.allclose(y, [0.0, 0.8412, -0.1588, 1.9545], atol=1e-3)


def test_layernorm_known_values():
    # tests/test_cpu_kernels.c:385-470: mean 0 / var 1 without affine,
    # mean = beta with gamma 2, beta 1; per-row on a 2x4 input
    y = O.layernorm(np.array([[1, 2, 3, 4]], np.float32))
    assert abs(y.mean()) < 1e-5 and abs((y * y).mean() - 1) < 1e-3
    y = O.layernorm(np.array([[1, 2, 3, 4]], np.float32), np.full(4, 2, np.float32),
                    np.ones(4, np.float32))
    assert abs(y.mean() - 1) < 1e-3
    y = O.layernorm(np.arange(1, 9, dtype=np.float32).reshape(2, 4))
    assert np.allclose(y.mean(axis=1), 0, atol=1e-5)


def test_rope_known_values():
    # tests/test_new_ops.c:569-700: identity, 90 degrees, known values
    x = np.arange(1, 9, dtype=np.float32).reshape(1, 2, 1, 4)
    y = O.rope(x, np.ones((2, 2), np.float32), np.zeros((2, 2), np.float32))
    assert np.allclose(y, x)
    y = O.rope(np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 1, 4),
               np.zeros((1, 2), np.float32), np.ones((1, 2), np.float32))
    assert np.allclose(y.ravel(), [-2, 1, -4, 3])
    y = O.rope(np.array([1, 0, 0, 1, 2, 1, 1, 2], np.float32).reshape(1, 1, 2, 4),
               np.array([[0.5, 0.866]], np.float32), np.array([[0.866, 0.5]], np.float32))
    assert np.allclose(y.ravel(), [0.5, 0.866, -0.5, 0.866, 0.134, 2.232, -0.134, 2.232], atol=1e-5)


def test_q8_known_properties():
    # tests/test_quant.c:24-130: block sizes, round trip error bounds, zeros, tail
    assert O.Q8_DTYPE.itemsize == 36
    src = (np.arange(32, dtype=np.float32) - 16) * 0.5
    q = O.q8_quantize(src)
    assert len(q) == 1 and np.abs(O.q8_dequantize(q, 32) - src).max() <= 0.04
    q = O.q8_quantize(np.zeros(32, np.float32))
    assert q["scale"][0] == 0 and not q["data"].any()
    src = np.arange(40, dtype=np.float32) * 0.1
    q = O.q8_quantize(src)
    assert len(q) == 2 and np.abs(O.q8_dequantize(q, 40) - src).max() <= 0.04
    assert not q["data"][1][8:].any()  # zero-padded tail
    src = np.sin(np.arange(1024, dtype=np.float32) * 0.1) * 10
    assert np.abs(O.q8_dequantize(O.q8_quantize(src), 1024) - src).max() <= 0.08


def test_bf16_fp16_rounding_rne():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 65520.0, 2 ** -25, 3 * 2 ** -26], np.float32)
    assert O.round_bf16(x)[0] == 1.0 and O.round_bf16(x)[1] == 1.0 + 2 ** -6
    f = O.round_fp16(x)
    assert np.isinf(f[2]) and f[3] == 0.0 and f[4] == 2 ** -24


# ---- (b) the reference CPU backend itself
@needs_ref
def test_rounding_matches_reference_bits():
    import torch  # bit patterns via torch for an independent third opinion
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(50000, dtype=np.float32) * s for s in (1e-6, 1, 1e4)])
    ours = O.round_bf16(x)
    assert np.array_equal(ours, torch.from_numpy(x).bfloat16().float().numpy())
    assert np.array_equal(O.round_fp16(x), torch.from_numpy(x).half().float().numpy())


@needs_ref
def test_q8_quantizer_bitexact_vs_reference():
    rng = np.random.default_rng(1)
    w = rng.standard_normal(4096 + 13, dtype=np.float32) * 0.02
    w[:32] = 0
    assert O.q8_quantize(w).tobytes() == O.ref_q8_quantize(w).tobytes()


@needs_ref
@pytest.mark.parametrize("M,K,N", [(37, 64, 29), (64, 256, 96)])
def test_matmul_vs_reference(M, K, N):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32)
    ref = O.ref_matmul(a, np.ascontiguousarray(w.T))
    assert rel_err(O.linear(a, w), ref) < 1e-6
    ab, wb = O.round_bf16(a), O.round_bf16(w)
    bits = lambda z: (z.view(np.uint32) >> 16).astype(np.uint16)
    rb = O.ref_matmul(bits(ab), bits(np.ascontiguousarray(wb.T)), "bf16")
    rbf = (rb.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(O.round_bf16(O.linear(ab, wb)), rbf)


@needs_ref
def test_matmul_q8_vs_reference_kernel():
    # single-op convention of cpu_matmul_q8.c:28-35: B [K,N] quantised flat
    rng = np.random.default_rng(3)
    M, K, N = 16, 128, 32
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal((K, N), dtype=np.float32)
    bq = O.q8_quantize(b)
    ref = O.ref_matmul_q8(a, bq, K, N)
    bdq = O.q8_dequantize(bq, K * N).reshape(K, N)
    assert rel_err(O.linear(a, np.ascontiguousarray(bdq.T)), ref) < 1e-6


@needs_ref
def test_gelu_layernorm_rope_sdpa_vs_reference():
    rng = np.random.default_rng(4)
    x = rng.standard_normal(5000, dtype=np.float32) * 3
    assert np.abs(O.gelu(x) - O.ref_gelu(x)).max() < 1e-6
    x = rng.standard_normal((64, 1024), dtype=np.float32)
    g, b = rng.standard_normal(1024, dtype=np.float32), rng.standard_normal(1024, dtype=np.float32)
    assert rel_err(O.layernorm(x, g, b), O.ref_layernorm(x, g, b)) < 1e-5
    cs, sn = O.rope_table(576, 24, 64, 1.0)
    q = rng.standard_normal((2, 576, 4, 64), dtype=np.float32)
    assert np.array_equal(O.rope(q, cs, sn), O.ref_rope(q, cs, sn))
    q, k, v = (rng.standard_normal((2, 3, 100, 64), dtype=np.float32) for _ in range(3))
    assert rel_err(O.sdpa(q, k, v), O.ref_sdpa(q, k, v)) < 1e-6


@needs_ref
def test_vit_forward_vs_reference():
    import synth
    cfg = synth.tiny_cfg(depth=8)
    w = synth.vit_weights(cfg, seed=3)
    img = synth.images(cfg, 1, seed=4)[0]
    assert rel_err(O.vit_forward(cfg, w, img), O.ref_vit_encode(cfg, w, img)) < 1e-5


def test_oracle_vit_vs_reference_golden_fixture():
    """The restated full forward at 1008 px (8 blocks, one global) against
    the committed outputs of the reference sam3_vit_build (~1 min)."""
    import os
    import synth
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vit_1008_depth8.npz"))
    cfg = dict(zip(("img_size", "patch_size", "embed_dim", "depth", "n_heads", "window_size", "mlp_dim"),
                   (int(v) for v in g["cfg"])))
    w = synth.vit_weights(cfg, seed=int(g["seeds"][0]))
    img = synth.images(cfg, 1, seed=int(g["seeds"][1]))[0]
    y = O.vit_forward(cfg, w, img).ravel()
    assert rel_err(y[g["idx"]], g["f32_sample"]) < 1e-5
