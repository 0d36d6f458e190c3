"""GPU parity of sam3cu_layernorm against the oracle (cpu_layernorm.c
restated), F32 statistics; F32 output within 1e-5, 16-bit output within the
16-bit rounding (1e-2)."""
import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols", [(5184, 1024), (37, 128), (9, 96), (3, 2048), (1, 1000)])
@pytest.mark.parametrize("affine", [False, True])
def test_layernorm_f32(cuda, rows, cols, affine):
    import torch
    import sam3cu
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols), dtype=np.float32) * 3 + 1.5)
    g = rng.standard_normal(cols, dtype=np.float32) if affine else None
    b = rng.standard_normal(cols, dtype=np.float32) if affine else None
    tg = torch.from_numpy(g).cuda() if affine else None
    tb = torch.from_numpy(b).cuda() if affine else None
    y = sam3cu.layernorm(torch.from_numpy(x).cuda(), tg, tb)
    assert rel_err(to_np(y), O.layernorm(x, g, b)) < 1e-5


@pytest.mark.parametrize("out", ["bf16", "f16"])
def test_layernorm_f32_to_16(cuda, out):
    import torch
    import sam3cu
    rng = np.random.default_rng(7)
    x = rng.standard_normal((5184, 1024), dtype=np.float32)
    g = rng.standard_normal(1024, dtype=np.float32)
    b = rng.standard_normal(1024, dtype=np.float32)
    odt = torch.bfloat16 if out == "bf16" else torch.float16
    y = sam3cu.layernorm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                         torch.from_numpy(b).cuda(), out_dtype=odt)
    ref = O.layernorm(x, g, b)
    rnd = O.round_bf16 if out == "bf16" else O.round_fp16
    assert np.array_equal(to_np(y), rnd(ref)) or rel_err(to_np(y), ref) < 1e-2


def test_layernorm_inplace(cuda):
    import torch
    import sam3cu
    rng = np.random.default_rng(8)
    x = rng.standard_normal((1000, 1024), dtype=np.float32)
    t = torch.from_numpy(x).cuda()
    sam3cu.layernorm(t, out=t)
    assert rel_err(to_np(t), O.layernorm(x)) < 1e-5
