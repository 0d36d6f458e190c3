"""Without a usable GPU every entry point fails with a status, never a crash
or a silent CPU fallback: the backend vtable's init returns SAM3_EBACKEND
(as the reference asks of a backend whose device is unavailable,
backend.h:29-56), and the encoder / neck constructors return NULL with an
error status.  The .sam3 reader is host code and works regardless.  Runs
only on hosts without CUDA (the CPU test run)."""
import ctypes as C

import numpy as np
import pytest

import sam3cu
import synth

pytestmark = pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="a GPU is present")


def test_backend_init_reports_ebackend():
    ops = sam3cu.backend_ops()
    assert ops
    init = C.CFUNCTYPE(C.c_int, C.c_void_p)(C.cast(ops, C.POINTER(C.c_void_p))[0])
    be = (C.c_uint8 * sam3cu.CUDA_BACKEND_SIZE)()
    C.cast(be, C.POINTER(C.c_int))[0] = sam3cu.CUDA_BACKEND_TYPE      # base.type
    C.cast(C.addressof(be) + 8, C.POINTER(C.c_void_p))[0] = ops        # base.ops
    assert init(C.addressof(be)) == -4  # SAM3_EBACKEND


def test_init_and_constructors_fail_with_a_status():
    L = sam3cu.lib()
    assert L.sam3cu_init(0) == -4  # SAM3CU_EBACKEND
    cfg = synth.tiny_cfg(depth=1)
    with pytest.raises(sam3cu.Sam3cuError):
        sam3cu.VitEncoder(cfg, synth.vit_weights(cfg, seed=1), sam3cu.BF16)
    with pytest.raises(sam3cu.Sam3cuError):
        sam3cu.FpnNeck(32, 64, 6, (1.0,), synth.neck_weights(32, 64, (1.0,), seed=1), sam3cu.BF16)


def test_sam3_reader_is_host_code():
    # a one-tensor v4 file built by hand: header, one descriptor, page-aligned blob
    import struct
    hdr = struct.pack("<4I5i4I", 0x334D4153, 4, 0, 1, 1008, 1024, 256, 32, 0, 0, 0, 0, 0)
    name = b"t".ljust(128, b"\0")
    desc = name + struct.pack("<2I4iQQQ", 0, 1, 4, 0, 0, 0, 0, 16, 0)
    blob = np.arange(4, dtype=np.float32).tobytes()
    image = hdr + desc + bytes(4096 - len(hdr) - len(desc)) + blob
    assert sam3cu.sam3_check(image) == (1, 4)
    assert sam3cu.sam3_find(image, "t") == dict(dtype=0, dims=(4,), offset=4096, nbytes=16)
