"""The graph/backend structs mirrored in include/sam3cu_backend.h have the
reference's exact layout: a small C probe prints sizeof / offsetof of every
field, compiled once against the mirror and once against the sam3.c headers
(skipped where the reference sources are absent).  CPU only."""
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

def _ref_dir() -> str:
    """The sam3.c checkout: SAM3C_REF, else BASELINE.json's reference_path."""
    if os.environ.get("SAM3C_REF"):
        return os.environ["SAM3C_REF"]
    try:
        import json
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            return json.load(f).get("reference_path", "")
    except (OSError, ValueError):
        return ""


REF = _ref_dir()

PROBE = r"""
#include <stdio.h>
#include <stddef.h>
%s
#define P(T, F) printf(#T "." #F " %%zu\n", offsetof(struct T, F))
int main(void) {
  printf("tensor %%zu node %%zu graph %%zu ops %%zu be %%zu\n", sizeof(struct sam3_tensor),
         sizeof(struct sam3_node), sizeof(struct sam3_graph), sizeof(struct sam3_backend_ops),
         sizeof(struct sam3_backend));
  P(sam3_tensor, dtype); P(sam3_tensor, n_dims); P(sam3_tensor, dims); P(sam3_tensor, strides);
  P(sam3_tensor, data); P(sam3_tensor, nbytes); P(sam3_tensor, ephemeral);
  P(sam3_tensor, dbg_force_readback);
  P(sam3_node, op); P(sam3_node, inputs); P(sam3_node, n_inputs); P(sam3_node, output);
  P(sam3_node, params); P(sam3_graph, nodes); P(sam3_graph, n_nodes); P(sam3_graph, no_readback);
  P(sam3_backend_ops, init); P(sam3_backend_ops, free); P(sam3_backend_ops, alloc_tensor);
  P(sam3_backend_ops, graph_eval); P(sam3_backend_ops, arena_reset);
  P(sam3_backend_ops, cache_invalidate); P(sam3_backend, type); P(sam3_backend, ops);
  printf("SDPA %%d COUNT %%d Q8 %%d\n", (int)SAM3_OP_SDPA, (int)SAM3_OP_COUNT, (int)SAM3_DTYPE_Q8_0);
  return 0;
}
"""


def _run(include, flags):
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "p.c")
        exe = os.path.join(d, "p")
        open(src, "w").write(PROBE % include)
        subprocess.run(["gcc", "-std=gnu11", *flags, src, "-o", exe], check=True,
                       capture_output=True)
        return subprocess.run([exe], check=True, capture_output=True, text=True).stdout


@pytest.mark.skipif(not REF or not os.path.isdir(os.path.join(REF, "src")), reason="reference sources absent")
def test_struct_layouts_match_reference():
    ours = _run('#include "sam3cu_backend.h"', ["-I" + os.path.join(ROOT, "include")])
    ref = _run('#include "backend/backend.h"',
               ["-I" + os.path.join(REF, "include"), "-I" + os.path.join(REF, "src")])
    assert ours == ref
