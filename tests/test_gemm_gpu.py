"""GPU parity of the fused tcgen05 linear (sam3cu_linear / sam3cu_linear_q8)
against the CPU oracle's restatement of gh_linear (+GELU, +residual).

Inputs are rounded to the operand type first, so the oracle sees exactly the
values the tensor cores see; what remains is FP32 accumulation order and the
output rounding.  Tolerances (normwise max relative error): F32 output 1e-4
... 2e-3 depending on K, 16-bit output 1e-2.
"""
import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 64, 256),      # one tile
    (257, 128, 320),     # M and N tails
    (100, 200, 40),      # K not a multiple of 64, N % 32 != 0
    (5184, 1024, 1024),  # ViT proj
    (5184, 1024, 3072),  # ViT qkv
]


def _inputs(M, K, N, seed, dt):
    import torch
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
    b = rng.standard_normal(N, dtype=np.float32) / np.float32(np.sqrt(K))
    rnd = O.round_bf16 if dt == "bf16" else O.round_fp16
    x, w = rnd(x), rnd(w)
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    dev = torch.device("cuda")
    return (x, w, b, torch.from_numpy(x).to(dev, tdt), torch.from_numpy(w).to(dev, tdt),
            torch.from_numpy(b).to(dev))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_linear_bias_f32out(cuda, dt, M, K, N):
    import torch
    import sam3cu
    x, w, b, tx, tw, tb = _inputs(M, K, N, 1, dt)
    y = sam3cu.linear(tx, tw, bias=tb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert sam3cu.device_error() == 0
    ref = O.linear(x, w, b)
    assert rel_err(to_np(y), ref) < 1e-4 * max(1.0, K / 256)


@pytest.mark.parametrize("M,K,N", [(257, 128, 320), (5184, 1024, 4736)])
def test_linear_gelu_bf16out(cuda, M, K, N):
    import sam3cu
    x, w, b, tx, tw, tb = _inputs(M, K, N, 2, "bf16")
    y = sam3cu.linear(tx, tw, bias=tb, act=sam3cu.ACT_GELU_TANH)
    ref = O.linear(x, w, b, act=1)
    assert rel_err(to_np(y), ref) < 1e-2


# the fc2-sized shapes run split-K on the pair kernel (4 K slices
# reduce-added into the residual; the bias is added by the first slice only)
@pytest.mark.parametrize("M,K,N", [(300, 256, 128), (5184, 4736, 1024), (5184, 1024, 1024), (10368, 4736, 1024),
                                   (5000, 4736, 1000),  # ragged M and N tiles under split-K
                                   (2000, 2048, 1000)])
def test_linear_residual_inplace(cuda, M, K, N):
    import torch
    import sam3cu
    x, w, b, tx, tw, tb = _inputs(M, K, N, 3, "bf16")
    res = np.random.default_rng(4).standard_normal((M, N), dtype=np.float32)
    tres = torch.from_numpy(res).cuda()
    sam3cu.linear(tx, tw, bias=tb, residual=tres, out=tres)  # x += linear(...)
    ref = O.linear(x, w, b, res=res)
    assert rel_err(to_np(tres), ref) < 2e-4 * max(1.0, K / 1024)


def test_q8_quantize_bitexact(cuda):
    import torch
    import sam3cu
    rng = np.random.default_rng(5)
    w = rng.standard_normal(4736 * 1024 + 17, dtype=np.float32) * np.float32(0.02)
    w[:64] = 0.0  # zero blocks: scale 0
    blocks = sam3cu.q8_quantize(torch.from_numpy(w).cuda())
    ref = O.q8_quantize(w)
    assert blocks.cpu().numpy().tobytes() == ref.tobytes()


@pytest.mark.parametrize("M,K,N", [(257, 128, 320), (5184, 1024, 4736)])
def test_linear_q8(cuda, M, K, N):
    import torch
    import sam3cu
    rng = np.random.default_rng(6)
    x = O.round_bf16(rng.standard_normal((M, K), dtype=np.float32))
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    b = rng.standard_normal(N, dtype=np.float32) * np.float32(0.01)
    blocks = O.q8_quantize(w)
    wdq = O.q8_dequantize(blocks, N * K).reshape(N, K)
    tb = torch.from_numpy(np.frombuffer(blocks.tobytes(), np.uint8).copy()).cuda()
    q, sc = sam3cu.q8_repack(tb, N, K)
    y = sam3cu.linear_q8(torch.from_numpy(x).cuda().bfloat16(), q, sc,
                         bias=torch.from_numpy(b).cuda(), out_dtype=torch.float32)
    # the dequantised weight is rounded to bf16 on chip: compare against the
    # exact x . dequant(W)^T at the north-star tolerance, and against the
    # bf16-rounded dequantised weight tightly
    assert rel_err(to_np(y), O.linear(x, wdq, b)) < 1e-2
    assert rel_err(to_np(y), O.linear(x, O.round_bf16(wdq), b)) < 1e-4 * max(1.0, K / 256)


@pytest.mark.parametrize("M,K,N", [(300, 64, 128), (5184, 1024, 4736)])
def test_linear_q8_f32_activations(cuda, M, K, N):
    """BASELINE config 0 as stated: F32 activations ~N(0,1) x Q8_0 weights
    (the reference's own quantiser, blocks along K) + F32 bias -> F32, the
    operands of cpu_kernel_matmul_q8 (cpu_matmul_q8.c:168-235), against the
    exact x . dequant(W)^T + b at the north-star Q8 bound 1e-2."""
    import torch
    import sam3cu
    rng = np.random.default_rng(7)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    b = rng.standard_normal(N, dtype=np.float32) * np.float32(0.01)
    blocks = O.q8_quantize(w)
    wdq = O.q8_dequantize(blocks, N * K).reshape(N, K)
    tb = torch.from_numpy(np.frombuffer(blocks.tobytes(), np.uint8).copy()).cuda()
    q, sc = sam3cu.q8_repack(tb, N, K)
    y = sam3cu.linear_q8(torch.from_numpy(x).cuda(), q, sc, bias=torch.from_numpy(b).cuda(),
                         out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert sam3cu.device_error() == 0
    assert rel_err(to_np(y), O.linear(x, wdq, b)) < 1e-2


@pytest.mark.parametrize("M,K,N", [(128, 32, 256), (257, 100, 320), (5184, 1024, 1024),
                                   (5184, 4736, 1024)])
def test_linear_f32_3xtf32(cuda, M, K, N):
    """F32 x F32 (3xTF32 on the tensor cores) against the F32 oracle at the
    north-star F32 bound 1e-4 (normwise), with bias and in-place residual."""
    import torch
    import sam3cu
    rng = np.random.default_rng(9)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
    b = rng.standard_normal(N, dtype=np.float32)
    y = sam3cu.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                      bias=torch.from_numpy(b).cuda(), out_dtype=torch.float32)
    assert rel_err(to_np(y), O.linear(x, w, b)) < 1e-4
    res = rng.standard_normal((M, N), dtype=np.float32)
    tres = torch.from_numpy(res).cuda()
    sam3cu.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), residual=tres, out=tres,
                  act=sam3cu.ACT_GELU_TANH)
    assert rel_err(to_np(tres), O.linear(x, w, None, res=res, act=1)) < 1e-4


@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("M,K,N", [(300, 256, 160), (5184, 1024, 1024)])
def test_linear_separate_residual(cuda, out_dtype, M, K, N):
    """y = x . W^T + b + r with r a different buffer from y: the TMA-store
    epilogue adds r in registers."""
    import torch
    import sam3cu
    x, w, b, tx, tw, tb = _inputs(M, K, N, 5, "bf16")
    res = np.random.default_rng(6).standard_normal((M, N), dtype=np.float32)
    tres = torch.from_numpy(res).cuda()
    odt = torch.float32 if out_dtype == "f32" else torch.bfloat16
    y = torch.empty((M, N), dtype=odt, device="cuda")
    sam3cu.linear(tx, tw, bias=tb, residual=tres, out=y)
    ref = O.linear(x, w, b, res=res)
    assert np.array_equal(to_np(tres), res)  # the residual is only read
    tol = 2e-4 * max(1.0, K / 1024) if out_dtype == "f32" else 1e-2
    assert rel_err(to_np(y), ref) < tol


@pytest.mark.parametrize("kind", ["f32", "q8"])
def test_streamk_residual_f32_and_q8(cuda, kind):
    """x += x . W^T + b on the 1-SM kernel with 64 / 48 tiles for 148 SMs: the
    3xTF32 kernel runs it stream-K (equal k-ranges per CTA, pieces of a tile
    reduce-added); the in-GEMM Q8_0 kernel runs it with whole tiles (or
    stream-K under S3CU_GEMM_STREAMK=2)."""
    import torch
    import sam3cu
    rng = np.random.default_rng(12)
    M, K, N = (2000, 1024, 1000) if kind == "f32" else (1500, 2048, 1024)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
    b = rng.standard_normal(N, dtype=np.float32)
    res = rng.standard_normal((M, N), dtype=np.float32)
    tres = torch.from_numpy(res).cuda()
    if kind == "f32":
        sam3cu.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), bias=torch.from_numpy(b).cuda(),
                      residual=tres, out=tres)
        ref, tol = O.linear(x, w, b, res=res), 1e-4
    else:
        blocks = O.q8_quantize(w)
        wdq = O.q8_dequantize(blocks, N * K).reshape(N, K)
        tb = torch.from_numpy(np.frombuffer(blocks.tobytes(), np.uint8).copy()).cuda()
        q, sc = sam3cu.q8_repack(tb, N, K)
        xb = O.round_bf16(x)
        sam3cu.linear_q8(torch.from_numpy(xb).cuda().bfloat16(), q, sc, bias=torch.from_numpy(b).cuda(),
                         residual=tres, out=tres)
        ref, tol = O.linear(xb, wdq, b, res=res), 1e-2
    torch.cuda.synchronize()
    assert sam3cu.device_error() == 0
    assert rel_err(to_np(tres), ref) < tol
