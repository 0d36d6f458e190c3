"""The encoder created from a .sam3 file (sam3cu_vit_create_from_sam3, the
sam3_weight_open + sam3_vit_load path) on the GPU.  Files are written by the
reference's own sam3_weight_write (oracle/_ref).

- F32 file -> BF16 encoder: identical output to sam3cu_vit_create on the
  same host arrays, and within 1e-2 of the reference's own encoder loaded
  from the same file (sam3_vit_load with the file, sam3_vit_build on its CPU
  backend).
- Q8_0 file (the converter's rule: every tensor of >= 1024 elements) ->
  Q8_0 encoder: the linear blocks go up as stored and are only repacked, so
  the output is identical to sam3cu_vit_create given the original linear
  weights (which it quantises itself, bit-identically) and the dequantised
  copies of the other quantised tensors; within 1e-2 of the oracle.
- Missing / mis-sized tensors give SAM3CU_EMODEL; a missing patch bias is
  zero, as in the reference."""
import numpy as np
import pytest

import oracle as O
import sam3cu
import synth
from _util import rel_err

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")

LINEAR = ("qkv_w", "proj_w", "fc1_w", "fc2_w")


def _write(path, cfg, w, quantize, patch_bias=True, drop=None, resize=None):
    t = synth.vit_sam3_tensors(cfg, w, patch_bias=patch_bias)
    if drop:
        t = [x for x in t if not x[0].endswith(drop)]
    if resize:
        t = [(n, a[:-1] if n.endswith(resize) else a) for n, a in t]
    O.ref_write_sam3(str(path), t, quantize=quantize, image_size=cfg["img_size"],
                     encoder_dim=cfg["embed_dim"], n_layers=cfg["depth"])
    return str(path)


def _q8_roundtrip(a):
    a = np.ascontiguousarray(a, np.float32)
    if a.size < 1024:
        return a
    return O.q8_dequantize(O.ref_q8_quantize(a), a.size).reshape(a.shape)


def _file_view(cfg, w):
    """What a Q8 file holds, as F32 host arrays: every file tensor of >= 1024
    elements dequant(quant(x)); the linear weights left as they are (the
    encoder quantises those itself).  qkv_b is three file tensors of e."""
    e = cfg["embed_dim"]
    out = dict(w)
    for k in ("patch_w", "patch_b", "pos_raw", "ln_pre_w", "ln_pre_b"):
        out[k] = _q8_roundtrip(w[k])
    out["blocks"] = []
    for b in w["blocks"]:
        nb = {}
        for k, a in b.items():
            if k in LINEAR:
                nb[k] = a
            elif k == "qkv_b":
                nb[k] = np.concatenate([_q8_roundtrip(a[j * e:(j + 1) * e]) for j in range(3)])
            else:
                nb[k] = _q8_roundtrip(a)
        out["blocks"].append(nb)
    return out


@needs_ref
def test_f32_file_matches_create_and_reference_loader(cuda, tmp_path):
    # window 24: the value a file-derived shape assumes (the file stores none)
    cfg = synth.tiny_cfg(depth=8, img_size=672, window_size=24)
    w = synth.vit_weights(cfg, seed=11)
    img = synth.images(cfg, 2, seed=12)
    path = _write(tmp_path / "vit.sam3", cfg, w, quantize=False)
    enc_f = sam3cu.VitEncoder.from_sam3(path, None, sam3cu.BF16, max_batch=2)
    assert enc_f.cfg == cfg  # shape read from the file
    enc_a = sam3cu.VitEncoder(cfg, w, sam3cu.BF16, max_batch=2)
    got, want = enc_f.encode_host(img), enc_a.encode_host(img)
    enc_f.close()
    enc_a.close()
    assert sam3cu.device_error() == 0
    assert np.array_equal(got, want)
    ref = O.ref_vit_encode_file(path, cfg, img[0])
    assert rel_err(got[0], ref) < 1e-2, rel_err(got[0], ref)


@needs_ref
def test_q8_file_blocks_uploaded_as_stored(cuda, tmp_path):
    # width 1024 so LayerNorm gains and biases cross the converter's
    # 1024-element threshold and arrive as Q8_0 too
    cfg = synth.tiny_cfg(depth=2, embed_dim=1024, img_size=336, window_size=12, mlp_dim=1024)
    w = synth.vit_weights(cfg, seed=21)
    img = synth.images(cfg, 1, seed=22)
    path = _write(tmp_path / "vit_q8.sam3", cfg, w, quantize=True)
    info = sam3cu.sam3_find(path, synth.VIT_PREFIX + "layers.0.layer_norm1.weight")
    assert info["dtype"] == sam3cu.Q8_0
    view = _file_view(cfg, w)
    for _ in range(2):  # twice: the second create reuses nothing of the first
        enc_f = sam3cu.VitEncoder.from_sam3(path, cfg, sam3cu.Q8_0)
        got = enc_f.encode_host(img)[0]
        enc_f.close()
    enc_a = sam3cu.VitEncoder(cfg, view, sam3cu.Q8_0)
    want = enc_a.encode_host(img)[0]
    enc_a.close()
    assert sam3cu.device_error() == 0
    assert np.array_equal(got, want)
    # semantics: the F32 encoder on dequant(quant()) of every quantised tensor
    deq = dict(view)
    deq["blocks"] = [dict(b, **{k: _q8_roundtrip(b[k]) for k in LINEAR}) for b in view["blocks"]]
    ref = O.vit_forward(cfg, deq, img[0])
    assert rel_err(got, ref) < 1e-2, rel_err(got, ref)


@needs_ref
def test_q8_file_into_bf16_encoder(cuda, tmp_path):
    """A quantised file may also feed a 16-bit encoder: blocks dequantised."""
    cfg = synth.tiny_cfg(depth=2)
    w = synth.vit_weights(cfg, seed=31)
    img = synth.images(cfg, 1, seed=32)
    path = _write(tmp_path / "vit_q8.sam3", cfg, w, quantize=True)
    view = _file_view(cfg, w)
    deq = dict(view)
    deq["blocks"] = [dict(b, **{k: _q8_roundtrip(b[k]) for k in LINEAR}) for b in view["blocks"]]
    enc = sam3cu.VitEncoder.from_sam3(path, cfg, sam3cu.BF16)
    got = enc.encode_host(img)[0]
    enc.close()
    ref = O.vit_forward(cfg, synth.round_weights(deq, O.round_bf16), img[0])
    assert rel_err(got, ref) < 1e-2, rel_err(got, ref)


@needs_ref
def test_missing_patch_bias_is_zero_and_bad_tensors_rejected(cuda, tmp_path):
    cfg = synth.tiny_cfg(depth=1)
    w = synth.vit_weights(cfg, seed=41)
    img = synth.images(cfg, 1, seed=42)
    path = _write(tmp_path / "nobias.sam3", cfg, w, quantize=False, patch_bias=False)
    enc = sam3cu.VitEncoder.from_sam3(path, cfg, sam3cu.BF16)
    got = enc.encode_host(img)[0]
    enc.close()
    wz = dict(w, patch_b=np.zeros_like(w["patch_b"]))
    enc = sam3cu.VitEncoder(cfg, wz, sam3cu.BF16)
    want = enc.encode_host(img)[0]
    enc.close()
    assert np.array_equal(got, want)
    for kw in (dict(drop="layers.0.mlp.fc2.bias"), dict(resize="layers.0.attention.k_proj.bias")):
        bad = _write(tmp_path / "bad.sam3", cfg, w, quantize=False, **kw)
        with pytest.raises(sam3cu.Sam3cuError) as ei:
            sam3cu.VitEncoder.from_sam3(bad, cfg, sam3cu.BF16)
        assert f"({sam3cu.EMODEL})" in str(ei.value)


@needs_ref
@pytest.mark.parametrize("half", [1, 2])
def test_half_precision_file(cuda, tmp_path, half):
    """An F16 (1) or BF16 (2) .sam3 file, as sam3_convert writes without
    quantisation: tensors are widened on the device, and both a 16-bit and a
    Q8_0 encoder built from the file match sam3cu_vit_create on the widened
    values exactly."""
    import torch
    cfg = synth.tiny_cfg(depth=2)
    w = synth.vit_weights(cfg, seed=51)
    img = synth.images(cfg, 1, seed=52)
    tdt = torch.float16 if half == 1 else torch.bfloat16
    bits = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(tdt).view(torch.int16).numpy().view(np.uint16)
    wide = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(tdt).float().numpy().reshape(np.shape(a))
    t = [(n, bits(a), half) for n, a in synth.vit_sam3_tensors(cfg, w)]
    path = str(tmp_path / "vit_half.sam3")
    O.ref_write_sam3(path, t, quantize=False, image_size=cfg["img_size"], encoder_dim=cfg["embed_dim"],
                     n_layers=cfg["depth"])
    assert sam3cu.sam3_find(path, synth.VIT_PREFIX + "layer_norm.weight")["dtype"] == half
    ww = dict(w)
    for k in ("patch_w", "patch_b", "pos_raw", "ln_pre_w", "ln_pre_b"):
        ww[k] = wide(w[k])
    ww["blocks"] = [{k: wide(a) for k, a in b.items()} for b in w["blocks"]]
    for code in (sam3cu.BF16, sam3cu.Q8_0):
        enc = sam3cu.VitEncoder.from_sam3(path, cfg, code)
        got = enc.encode_host(img)[0]
        enc.close()
        enc = sam3cu.VitEncoder(cfg, ww, code)
        want = enc.encode_host(img)[0]
        enc.close()
        assert np.array_equal(got, want), code
