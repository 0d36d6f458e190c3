"""End-to-end encoder parity: sam3cu_vit_encode against the reference's own
sam3_vit_build on its CPU backend (oracle/_ref) and the oracle restatement,
on seeded random weights rounded to the weight type (so both sides use the
same weight values).  Tolerance 1e-2 normwise for BF16/F16/Q8 (activations
are 16-bit on the GPU, F32 on the CPU)."""
import numpy as np
import pytest

import oracle as O
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu


def _ref(cfg, w, img):
    if O.ref_available():
        return O.ref_vit_encode(cfg, w, img)
    return O.vit_forward(cfg, w, img)


@pytest.mark.parametrize("wd", ["bf16", "f16", "q8"])
def test_tiny_vit(cuda, wd):
    import sam3cu
    cfg = synth.tiny_cfg(depth=8)
    w = synth.vit_weights(cfg, seed=1)
    imgs = synth.images(cfg, 2, seed=2)
    if wd == "q8":
        rw = synth.round_weights(w, lambda a: O.q8_dequantize(O.q8_quantize(a), a.size).reshape(a.shape))
        rw["patch_w"] = O.round_bf16(w["patch_w"])
        code = sam3cu.Q8_0
    else:
        rnd = O.round_bf16 if wd == "bf16" else O.round_fp16
        rw = synth.round_weights(w, rnd)
        code = sam3cu.BF16 if wd == "bf16" else sam3cu.F16
    enc = sam3cu.VitEncoder(cfg, w, code, max_batch=2)
    out = enc.encode_host(imgs)
    assert sam3cu.device_error() == 0
    for i in range(2):
        ref = _ref(cfg, rw, imgs[i])
        assert rel_err(out[i], ref) < 1e-2, (wd, i, rel_err(out[i], ref))
    # determinism: a second call (graph replay) gives identical bits
    out2 = enc.encode_host(imgs)
    assert np.array_equal(out, out2)
    enc.close()


@pytest.mark.parametrize("n,mb,chunk", [(7, 2, 2), (5, 8, 3)])  # (5, 8): one batch split in halves
def test_host_encode_pipelined_chunks(cuda, n, mb, chunk):
    """Host buffers with more images than max_batch: chunks of max_batch on
    two staging sets with overlapped copies.  Every image's features must be
    those of an on-device encode of the same chunk, and the order kept."""
    import torch
    import sam3cu
    cfg = synth.tiny_cfg(depth=4)
    w = synth.vit_weights(cfg, seed=3)
    imgs = synth.images(cfg, n, seed=4)
    enc = sam3cu.VitEncoder(cfg, w, sam3cu.BF16, max_batch=mb)
    hin = torch.from_numpy(np.ascontiguousarray(imgs)).pin_memory()
    hout = torch.empty((n, enc.np, cfg["embed_dim"]), dtype=torch.float32).pin_memory()
    enc.encode_ptr(hin.data_ptr(), n, hout.data_ptr(), on_device=False)
    assert sam3cu.device_error() == 0
    got = hout.numpy()
    for first in range(0, n, chunk):
        cn = min(chunk, n - first)
        din = torch.from_numpy(np.ascontiguousarray(imgs[first:first + cn])).cuda()
        dout = torch.empty((cn, enc.np, cfg["embed_dim"]), dtype=torch.float32, device="cuda")
        enc.encode_ptr(din.data_ptr(), cn, dout.data_ptr(), on_device=True)
        assert np.array_equal(got[first:first + cn], dout.cpu().numpy()), first
    enc.close()


def test_profile_detail_kinds(cuda):
    """sam3cu_vit_profile_detail: one launch per linear and block in its
    own kind, window / global attention apart, one Q8_0 dequantisation
    launch per block; the coarse sam3cu_vit_profile counts are their sums."""
    import torch
    import sam3cu
    cfg = synth.tiny_cfg(depth=8)
    w = synth.vit_weights(cfg, seed=5)
    img = torch.from_numpy(synth.images(cfg, 1, seed=6)).cuda()
    for code in (sam3cu.BF16, sam3cu.Q8_0):
        enc = sam3cu.VitEncoder(cfg, w, code, max_batch=1)
        out = torch.empty((1, enc.np, cfg["embed_dim"]), dtype=torch.float32, device="cuda")
        d = enc.profile_detail(img, out)
        c = enc.profile(img, out)
        enc.close()
        n = {k: v[1] for k, v in d.items()}
        assert n["qkv"] == n["proj"] == n["fc1"] == n["fc2"] == 8 and n["patch"] == 1
        assert n["attn_global"] == 1 and n["attn_window"] == 7  # block 7 is global
        assert n["dequant"] == (8 if code == sam3cu.Q8_0 else 0)
        assert n["layernorm"] == 17
        gemm = sum(n[k] for k in ("patch", "qkv", "proj", "fc1", "fc2", "dequant"))
        assert c["gemm"][1] == gemm and c["attention"][1] == 8 and c["layernorm"][1] == 17
        assert all(v[0] >= 0.0 for v in d.values())
