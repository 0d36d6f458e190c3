"""GPU parity of the fused attention (sam3cu_sdpa) against the oracle's
restatement of cpu_sdpa.c on the same 16-bit Q/K/V, for window groups (576
tokens), ragged groups and one global 5184-token image.  Tolerance 1e-2
(normwise; P is rounded to 16 bit before P.V on the tensor cores)."""
import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu


def _run(n_groups, seq, heads, dt, seed, check_heads=None):
    import torch
    import sam3cu
    E = heads * 64
    rng = np.random.default_rng(seed)
    qkv = rng.standard_normal((n_groups * seq, 3 * E), dtype=np.float32)
    rnd = O.round_bf16 if dt == "bf16" else O.round_fp16
    qkv = rnd(qkv)
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    out = sam3cu.sdpa_packed(torch.from_numpy(qkv).cuda().to(tdt), n_groups, seq, heads)
    torch.cuda.synchronize()
    o = to_np(out).reshape(n_groups, seq, heads, 64)
    q = qkv[:, :E].reshape(n_groups, seq, heads, 64)
    k = qkv[:, E:2 * E].reshape(n_groups, seq, heads, 64)
    v = qkv[:, 2 * E:].reshape(n_groups, seq, heads, 64)
    hs = check_heads if check_heads is not None else range(heads)
    for h in hs:
        ref = O.sdpa(q[:, :, h], k[:, :, h], v[:, :, h])
        assert rel_err(o[:, :, h], ref) < 1e-2, h


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_window_groups(cuda, dt):
    _run(9, 576, 16, dt, 11, check_heads=[0, 7, 15])


def test_ragged_seq(cuda):
    _run(3, 100, 2, "bf16", 12)
    _run(2, 1, 1, "bf16", 13)


def test_global_image(cuda):
    _run(1, 5184, 16, "bf16", 14, check_heads=[3])
