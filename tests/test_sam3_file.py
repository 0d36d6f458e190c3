"""The .sam3 reader of the CUDA library (sam3cu_sam3_check / _find, host
code, no GPU) against the reference's own writer and reader: files written
by sam3_weight_write (weight.c:64-236; F32, and Q8_0 by the converter's rule
of cli_convert.c:340-425) are read by both sam3_weight_open/_find and the
library, and every descriptor, offset and payload must agree.  Malformed
files must be rejected by both with SAM3_EMODEL (weight.c:303-470)."""
import os
import struct

import numpy as np
import pytest

import oracle as O
import sam3cu
import synth

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
CFG = synth.tiny_cfg(depth=2, embed_dim=128, img_size=168, window_size=12, mlp_dim=320)


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("sam3")
    w = synth.vit_weights(CFG, seed=5)
    tensors = synth.vit_sam3_tensors(CFG, w)
    out = {}
    for q in (0, 1):
        p = str(d / f"vit_q{q}.sam3")
        O.ref_write_sam3(p, tensors, quantize=bool(q), image_size=CFG["img_size"],
                         encoder_dim=CFG["embed_dim"], n_layers=CFG["depth"])
        out[q] = p
    return out, tensors


@needs_ref
@pytest.mark.parametrize("q", [0, 1])
def test_descriptors_and_payloads_match_reference_reader(files, q):
    paths, tensors = files
    path = paths[q]
    n, ver = sam3cu.sam3_check(path)
    assert (n, ver) == (len(tensors), 4)
    raw = np.fromfile(path, np.uint8)
    for name, arr in tensors:
        ours = sam3cu.sam3_find(path, name)
        ref = O.ref_find_sam3(path, name)
        assert ours == ref, name
        payload = raw[ours["offset"]:ours["offset"] + ours["nbytes"]]
        a = np.ascontiguousarray(arr, np.float32).ravel()
        if q and a.size >= 1024:
            assert ours["dtype"] == sam3cu.Q8_0
            assert payload.tobytes() == O.ref_q8_quantize(a).tobytes(), name
        else:
            assert ours["dtype"] == sam3cu.F32
            assert payload.tobytes() == a.tobytes(), name
    assert sam3cu.sam3_find(path, "no.such.tensor") is None
    assert O.ref_find_sam3(path, "no.such.tensor") is None


def _hdr(raw):
    return struct.unpack_from("<4I", raw, 0)  # magic, version, flags, n_tensors


@needs_ref
def test_version3_header_read_like_reference(files, tmp_path):
    """A v3 file: 48-byte header (no text_backbone), table right after it."""
    paths, tensors = files
    raw = bytearray(open(paths[0], "rb").read())
    _, _, _, n = _hdr(raw)
    table_end_v4 = 52 + n * 176
    if (table_end_v4 + 4095) // 4096 != (table_end_v4 - 4 + 4095) // 4096:
        pytest.skip("table end sits on a page boundary")
    v3 = bytearray(raw[:48]) + raw[52:table_end_v4] + bytes(4) + raw[table_end_v4:]
    struct.pack_into("<I", v3, 4, 3)
    p = str(tmp_path / "v3.sam3")
    open(p, "wb").write(v3)
    assert sam3cu.sam3_check(p)[1] == 3
    for name, _ in tensors[:6]:
        assert sam3cu.sam3_find(p, name) == O.ref_find_sam3(p, name)


@needs_ref
@pytest.mark.parametrize("case", ["magic", "version", "short", "table", "data"])
def test_malformed_files_rejected_like_reference(files, tmp_path, case):
    paths, _ = files
    raw = bytearray(open(paths[0], "rb").read())
    if case == "magic":
        struct.pack_into("<I", raw, 0, 0x12345678)
    elif case == "version":
        struct.pack_into("<I", raw, 4, 5)
    elif case == "short":
        raw = raw[:40]
    elif case == "table":
        struct.pack_into("<I", raw, 12, 10 ** 6)  # n_tensors past the end
    elif case == "data":
        # last descriptor's data_size past the end of the blob
        n = _hdr(raw)[3]
        off = 52 + (n - 1) * 176 + 128 + 8 + 16 + 8
        struct.pack_into("<Q", raw, off, len(raw))
    p = str(tmp_path / f"bad_{case}.sam3")
    open(p, "wb").write(raw)
    assert O.ref_open_sam3(p) == sam3cu.EMODEL
    with pytest.raises(sam3cu.Sam3cuError) as ei:
        sam3cu.sam3_check(p)
    assert f"{sam3cu.EMODEL}" in str(ei.value) or "malformed" in str(ei.value)


@needs_ref
def test_duplicate_and_long_names_like_reference(tmp_path):
    """Duplicate names: the first descriptor wins in both readers (the
    reference probes its table in file order).  Names longer than 127 bytes
    are truncated by the writer and found under the truncated name."""
    long = "x" * 200
    t = [("dup", np.full(8, 1.0, np.float32)), ("dup", np.full(8, 2.0, np.float32)),
         ("y" * 127, np.arange(4, dtype=np.float32)), (long, np.arange(6, dtype=np.float32))]
    p = str(tmp_path / "names.sam3")
    O.ref_write_sam3(p, t)
    raw = np.fromfile(p, np.uint8)
    for name in ("dup", "y" * 127, "x" * 127):
        ours, ref = sam3cu.sam3_find(p, name), O.ref_find_sam3(p, name)
        assert ours == ref, name
    d = sam3cu.sam3_find(p, "dup")
    assert raw[d["offset"]:d["offset"] + d["nbytes"]].view(np.float32)[0] == 1.0
    assert sam3cu.sam3_find(p, long) is None and O.ref_find_sam3(p, "x" * 127)["dims"] == (6,)


@needs_ref
@pytest.mark.parametrize("pad", [False, True])
def test_empty_table_like_reference(tmp_path, pad):
    """A v4 header with no tensors: valid only when the file reaches the
    page-aligned data blob start (4096), as sam3_weight_open rules."""
    hdr = struct.pack("<4I5i4I", 0x334D4153, 4, 0, 0, 1008, 1024, 256, 32, 0, 0, 0, 0, 0)
    assert len(hdr) == 52
    p = str(tmp_path / "empty.sam3")
    open(p, "wb").write(hdr + (bytes(4096 - 52) if pad else b""))
    ref = O.ref_open_sam3(p)
    if pad:
        assert ref == 0 and sam3cu.sam3_check(p) == (0, 4)
    else:
        assert ref == sam3cu.EMODEL
        with pytest.raises(sam3cu.Sam3cuError):
            sam3cu.sam3_check(p)
