"""ctypes binding of dropin/_ref/libsam3_dropin.so: the reference's own
sam3_vit_build (compiled from the sam3.c sources) evaluated through
sam3_cuda_backend_ops(), one session per device.  Measurement / test
harness of the drop-in path."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libsam3_dropin.so")
_lib = None

ORDER = ("ln1_w", "ln1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ln2_w", "ln2_b",
         "fc1_w", "fc1_b", "fc2_w", "fc2_b")
CFG_KEYS = ("img_size", "patch_size", "embed_dim", "depth", "n_heads", "window_size", "mlp_dim")


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"{LIB} not built (make -C dropin SAM3C_REF=<sam3.c checkout>)")
        _lib = C.CDLL(LIB)
        _lib.dropin_vit_create.restype = C.c_void_p
        _lib.dropin_vit_create.argtypes = [C.POINTER(C.c_int), C.POINTER(C.c_void_p), C.c_int]
        _lib.dropin_vit_encode.restype = C.c_int
        _lib.dropin_vit_encode.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_double)]
        _lib.dropin_vit_free.argtypes = [C.c_void_p]
        _lib.dropin_vit_profile_dump.argtypes = [C.c_void_p]
    return _lib


class DropinVit:
    """The reference encoder on the CUDA backend.  w: the dict of
    sam3.c_b200/synth.py (F32 host arrays, patch weight OHWI)."""

    def __init__(self, cfg: dict, w: dict, device: int = 0):
        self.cfg = cfg
        arrs = [w["patch_w"], w["patch_b"], w["pos_raw"], w["ln_pre_w"], w["ln_pre_b"]]
        for b in w["blocks"]:
            arrs += [b[k] for k in ORDER]
        self._keep = [np.ascontiguousarray(a, np.float32) for a in arrs]
        ptrs = (C.c_void_p * len(self._keep))(*[a.ctypes.data for a in self._keep])
        c = (C.c_int * 7)(*[cfg[k] for k in CFG_KEYS])
        self._s = lib().dropin_vit_create(c, ptrs, device)
        if not self._s:
            raise RuntimeError("dropin_vit_create failed")
        gs = cfg["img_size"] // cfg["patch_size"]
        self.out_shape = (gs * gs, cfg["embed_dim"])

    def encode(self, image: np.ndarray, out: np.ndarray | None = None):
        """image: planar CHW [3,img,img] F32.  Returns (features, seconds of
        the sam3_vit_build call)."""
        image = np.ascontiguousarray(image, np.float32)
        if out is None:
            out = np.empty(self.out_shape, np.float32)
        sec = C.c_double(0.0)
        rc = lib().dropin_vit_encode(self._s, image.ctypes.data, out.ctypes.data, C.byref(sec))
        if rc != 0:
            raise RuntimeError(f"dropin_vit_encode failed rc={rc}")
        return out, sec.value

    def profile_dump(self):
        """Print and reset the backend's per-op profile (only when
        SAM3CU_VTABLE_PROFILE=1 was set before the session was created)."""
        lib().dropin_vit_profile_dump(self._s)

    def close(self):
        if self._s:
            lib().dropin_vit_free(self._s)
            self._s = None

    def __del__(self):
        self.close()
