"""Host-side checks of the C ABI (no GPU needed): the in-tree library loads,
exports exactly what include/sam3cu.h declares, and rejects bad arguments
before touching a device."""
import ctypes as C
import os
import re
import subprocess

import pytest

import sam3cu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    return set(re.findall(r"SAM3CU_API[^;(]*?\b(sam3(?:cu)?_\w+)\s*\(", txt))


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", sam3cu.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_library_present_and_loads():
    assert os.path.exists(sam3cu.LIB_PATH), "run python sam3.c_b200/build.py"
    sam3cu.lib()


def test_exports_match_headers():
    declared = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            declared |= _declared(h)
    exported = _exported()
    missing = declared - exported
    assert not missing, f"declared but not exported: {missing}"
    assert set(sam3cu.EXPORTS) <= exported


def test_strerror_codes():
    L = sam3cu.lib()
    assert L.sam3cu_strerror(0) == b"ok"
    assert L.sam3cu_strerror(-1) == b"invalid argument"
    assert L.sam3cu_strerror(-105).startswith(b"device")
    assert L.sam3cu_strerror(-5).startswith(b"malformed")  # SAM3_EMODEL
    assert L.sam3cu_strerror(-109).startswith(b"tensor not in")


def test_bad_arguments_rejected_on_host():
    L = sam3cu.lib()
    # null operands, bad dtype, bad activation: rejected before any launch
    assert L.sam3cu_linear(None, 2, None, None, None, None, 0, 4, 8, 8, 0, None) == -1
    assert L.sam3cu_linear(C.c_void_p(16), 3, C.c_void_p(16), None, None, C.c_void_p(16), 0, 4, 8, 8, 0,
                           None) == -6  # I32 operands
    assert L.sam3cu_linear(C.c_void_p(16), 2, C.c_void_p(16), None, None, C.c_void_p(16), 0, 4, 8, 8, 9,
                           None) == -1
    assert L.sam3cu_sdpa(None, None, None, 0, None, 0, 2, 1, 1, 1, 64, None) == -1
    st = C.c_int(0)
    assert not L.sam3cu_vit_create(None, None, 2, 1, C.byref(st))
    assert st.value == -1
