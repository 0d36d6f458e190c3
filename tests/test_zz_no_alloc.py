"""The allocation-free CONV2D entry point (sam3cu_conv2d_nhwc_noalloc).

It serves callers that cannot let the library allocate device memory: hosts
that reserve all GPU memory in their own pool up front, fixed-budget
deployments, and latency-critical loops where cudaMalloc / cudaFree would
synchronise the device.  Its column buffer is a static device array shared
by every call, so the test makes two calls in a row (with different inputs
and shapes) through the C ABI and checks each against the allocating CONV2D
path of the CUDA backend (the vtable's graph_eval), or the CPU oracle where
the reference library is absent, at the tolerances of the other parity
tests: 1e-4 (F32) and 1e-2 (BF16, F16), normwise.  It also checks the
optional bias and that a warm call leaves the device's free memory
unchanged.  It sits in a file pytest collects last and must pass alone in a
fresh process as well.
"""
import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu


def _conv_existing(x, w, stride, pad):
    """The allocating path: a CONV2D node evaluated by sam3_cuda_backend_ops
    (or, without the reference harness, the oracle's im2col + linear)."""
    import sam3cu
    n, H, W, C = x.shape
    OC, kh, kw, _ = w.shape
    OH, OW = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    if O.ref_available():
        ins = [(x, "f32", x.shape), (w, "f32", w.shape)]
        return O.ref_node_graph(O.OP["CONV2D"], ins, "f32", (n, OH, OW, OC), params=(stride, pad, 1, 0),
                                ops=sam3cu.backend_ops(), be_size=sam3cu.CUDA_BACKEND_SIZE,
                                be_type=sam3cu.CUDA_BACKEND_TYPE)
    xp = np.pad(x, ((0, 0), (pad, pad), (pad, pad), (0, 0)))
    cols = np.stack([xp[:, oy * stride:oy * stride + kh, ox * stride:ox * stride + kw, :].reshape(n, -1)
                     for oy in range(OH) for ox in range(OW)], axis=1).reshape(-1, kh * kw * C)
    return O.linear(cols, w.reshape(OC, -1)).reshape(n, OH, OW, OC)


def _case(rng, n, H, W, C, OC, k, stride, pad):
    x = rng.standard_normal((n, H, W, C), dtype=np.float32)
    w = rng.standard_normal((OC, k, k, C), dtype=np.float32) * np.float32(0.05)
    return x, w


def test_noalloc_conv_matches_allocating_path_twice(cuda):
    import torch
    import sam3cu
    rng = np.random.default_rng(21)
    # call 1: the patch-embed shape (14x14 stride 14, K = 588), one 1008 px image
    # call 2: a padded 3x3 conv whose K = 27 is not a multiple of 4 (padded weight)
    for (n, H, W, C, OC, k, stride, pad) in [(1, 1008, 1008, 3, 1024, 14, 14, 0), (2, 40, 36, 3, 64, 3, 1, 1)]:
        x, w = _case(rng, n, H, W, C, OC, k, stride, pad)
        ref = _conv_existing(x, w, stride, pad)
        y = sam3cu.conv2d_nhwc_noalloc(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                                       stride=stride, pad=pad)
        torch.cuda.synchronize()
        assert sam3cu.device_error() == 0
        assert rel_err(to_np(y), ref) < 1e-4
        for dt in (torch.bfloat16, torch.float16):
            y16 = sam3cu.conv2d_nhwc_noalloc(torch.from_numpy(x).cuda().to(dt),
                                             torch.from_numpy(w).cuda().to(dt), stride=stride, pad=pad)
            torch.cuda.synchronize()
            assert sam3cu.device_error() == 0
            assert rel_err(to_np(y16), ref) < 1e-2


def test_noalloc_conv_bias(cuda):
    """With an F32 bias [OC]: the allocating path's result plus the bias."""
    import torch
    import sam3cu
    rng = np.random.default_rng(22)
    x, w = _case(rng, 1, 48, 48, 3, 64, 3, 2, 1)
    b = rng.standard_normal(64, dtype=np.float32)
    ref = _conv_existing(x, w, 2, 1) + b
    for dt, tol in ((torch.float32, 1e-4), (torch.float16, 1e-2)):
        y = sam3cu.conv2d_nhwc_noalloc(torch.from_numpy(x).cuda().to(dt), torch.from_numpy(w).cuda().to(dt),
                                       bias=torch.from_numpy(b).cuda(), stride=2, pad=1)
        torch.cuda.synchronize()
        assert sam3cu.device_error() == 0
        assert rel_err(to_np(y), ref) < tol


def test_noalloc_conv_allocates_nothing(cuda):
    """A warm call leaves the device's free memory unchanged: nothing on the
    path (im2col, weight padding, GEMM) allocated device memory."""
    import torch
    import sam3cu
    rng = np.random.default_rng(23)
    x, w = _case(rng, 2, 40, 36, 3, 64, 3, 1, 1)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.empty((2, 40, 36, 64), device="cuda")
    sam3cu.conv2d_nhwc_noalloc(xd, wd, stride=1, pad=1, out=out)   # warm: module loaded
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        sam3cu.conv2d_nhwc_noalloc(xd, wd, stride=1, pad=1, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert sam3cu.device_error() == 0


def test_noalloc_conv_rejects_oversize(cuda):
    import torch
    import sam3cu
    x = torch.zeros((4, 1008, 1008, 3), device="cuda")   # 4 images: 48.8 MB of F32 columns
    w = torch.zeros((1024, 14, 14, 3), device="cuda")
    with pytest.raises(sam3cu.Sam3cuError, match="scratch"):
        sam3cu.conv2d_nhwc_noalloc(x, w, stride=14)
