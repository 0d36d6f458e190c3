"""Failure detection on the GPU without a GPU fault: a kernel waits on an
mbarrier that nothing arrives on, with a 20 ms limit.  The bounded wait must
give up, record its error code and return; the host reads the status, and
the same context then runs a GEMM correctly."""
import time

import numpy as np
import pytest

import oracle as O
from _util import rel_err, to_np

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda):
    import torch
    import sam3cu
    t0 = time.perf_counter()
    assert sam3cu.selftest_wait_timeout(20_000_000)
    assert time.perf_counter() - t0 < 5.0  # bounded, not hung
    assert sam3cu.device_error() == 0      # the self test cleared its word
    rng = np.random.default_rng(0)
    x = O.round_bf16(rng.standard_normal((256, 128), dtype=np.float32))
    w = O.round_bf16(rng.standard_normal((192, 128), dtype=np.float32) * 0.1)
    y = sam3cu.linear(torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda().bfloat16(),
                      out=torch.empty(256, 192, device="cuda", dtype=torch.float32))
    torch.cuda.synchronize()
    assert rel_err(to_np(y), O.linear(x, w)) < 1e-2
