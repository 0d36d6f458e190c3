"""GPU parity of the TinyViT window attention (sam3cu_tvit_window_attention)
against the oracle's restatement of tvit_window_attention, on the same
16-bit qkv, at the 1008px TinyViT shapes: 7x7 windows (49 tokens, 6 and 18
heads) and 14x14 windows (196 tokens, 12 heads), head_dim 32, with the
expanded relative position bias.  Tolerance 1e-2 normwise."""
import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu


def _run(nw, ws, heads, hd, dt, bias, seed):
    import torch
    import sam3cu
    N = ws * ws
    rng = np.random.default_rng(seed)
    rnd = O.round_bf16 if dt == "bf16" else O.round_fp16
    qkv = rnd(rng.standard_normal((nw * N, 3 * heads * hd), dtype=np.float32))
    b_dense = None
    b_dev = None
    if bias:
        comp = (rng.standard_normal((heads, N)) * 2).astype(np.float32)
        b_dense = O.tvit_expand_bias(comp, ws)
        b_dev = torch.from_numpy(sam3cu.tvit_expand_bias(comp, ws)).cuda()
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    out = sam3cu.tvit_window_attention(torch.from_numpy(qkv).cuda().to(tdt), nw, N, heads, hd, b_dev)
    torch.cuda.synchronize()
    assert sam3cu.device_error() == 0
    ref = O.tvit_window_attention(qkv, nw, N, heads, hd, b_dense)
    assert rel_err(to_np(out), ref) < 1e-2


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("ws,heads", [(7, 6), (14, 12), (7, 18)])
def test_tvit_window_attention(cuda, dt, ws, heads):
    _run(25, ws, heads, 32, dt, True, ws + heads)


def test_tvit_window_attention_no_bias(cuda):
    _run(10, 7, 3, 32, "bf16", False, 5)


def test_tvit_window_attention_hd64(cuda):
    _run(6, 14, 4, 64, "f16", True, 6)


def test_tvit_window_attention_many_windows(cuda):
    # stage-1 at 1008px: 18 x 18 = 324 windows of 7 x 7, 6 heads
    _run(324, 7, 6, 32, "bf16", True, 9)
