"""Python host side of the B200 backend: ctypes bindings of include/sam3cu.h.

This mirrors the per-op and encoder entry points of sam3.c that the CUDA
library replaces (see the header for the reference file:line of each).  It
loads ``lib/libsam3cu.so`` built in tree by ``build.py`` and raises if the
library is missing: there is no CPU fallback.  Device buffers are passed as
torch CUDA tensors (torch is used only for device memory and streams).
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# SAM3CU_LIB selects another build of the library (A/B measurements)
LIB_PATH = os.environ.get("SAM3CU_LIB") or os.path.join(HERE, "lib", "libsam3cu.so")

F32, F16, BF16, Q8_0 = 0, 1, 2, 5
ACT_NONE, ACT_GELU_TANH = 0, 1
EMODEL, ENOENT = -5, -109

EXPORTS = (
    "sam3cu_init", "sam3cu_strerror", "sam3cu_last_device_error",
    "sam3cu_launch_count", "sam3cu_linear", "sam3cu_linear_q8",
    "sam3cu_q8_repack", "sam3cu_q8_quantize", "sam3cu_layernorm",
    "sam3cu_sdpa", "sam3cu_vit_create", "sam3cu_vit_destroy",
    "sam3cu_vit_encode", "sam3cu_vit_encode_async", "sam3cu_vit_stream",
    "sam3cu_vit_launches_per_encode", "sam3cu_vit_profile", "sam3cu_vit_profile_detail",
    "sam3_cuda_backend_ops", "sam3cu_conv2d_nhwc_noalloc",
    "sam3cu_tvit_expand_bias", "sam3cu_tvit_window_attention",
    "sam3cu_tvit_block_create", "sam3cu_tvit_block_forward", "sam3cu_tvit_block_destroy",
    "sam3cu_tvit_mbconv_create", "sam3cu_tvit_mbconv_forward", "sam3cu_tvit_mbconv_destroy",
    "sam3cu_selftest_wait_timeout",
    "sam3cu_tinyvit_create", "sam3cu_tinyvit_encode", "sam3cu_tinyvit_grid", "sam3cu_tinyvit_destroy",
    "sam3cu_sam3_check", "sam3cu_sam3_find", "sam3cu_vit_create_from_sam3", "sam3cu_vit_get_config",
    "sam3cu_neck_create", "sam3cu_neck_forward", "sam3cu_neck_forward_async", "sam3cu_neck_out_size",
    "sam3cu_neck_stream", "sam3cu_neck_destroy",
)

# sizeof(struct sam3_cuda_backend): {enum type; ops*} + int device + void *impl
CUDA_BACKEND_SIZE = 32
CUDA_BACKEND_TYPE = 2

PROFILE_KINDS = ("gemm", "attention", "layernorm", "other")
PROFILE_DETAIL_KINDS = ("patch", "qkv", "proj", "fc1", "fc2", "dequant", "attn_window", "attn_global",
                        "layernorm", "other")

_lib = None


class Sam3cuError(RuntimeError):
    pass


def lib():
    """Load libsam3cu.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise Sam3cuError(f"{LIB_PATH} not built: run `python sam3.c_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
        L.sam3cu_strerror.restype = C.c_char_p
        L.sam3cu_last_device_error.restype = C.c_uint
        L.sam3cu_launch_count.restype = C.c_uint64
        L.sam3cu_launch_count.argtypes = [i32]
        L.sam3cu_linear.argtypes = [vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]
        L.sam3cu_linear_q8.argtypes = [vp, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]
        L.sam3cu_q8_repack.argtypes = [vp, i32, i32, vp, vp, vp]
        L.sam3cu_q8_quantize.argtypes = [vp, vp, i64, vp]
        L.sam3cu_layernorm.argtypes = [vp, i32, vp, vp, vp, i32, i32, i32, vp]
        L.sam3cu_sdpa.argtypes = [vp, vp, vp, i64, vp, i64, i32, i32, i32, i32, i32, vp]
        L.sam3cu_vit_create.restype = vp
        L.sam3cu_vit_create.argtypes = [vp, vp, i32, i32, C.POINTER(C.c_int)]
        L.sam3cu_vit_destroy.argtypes = [vp]
        L.sam3cu_vit_create_from_sam3.restype = vp
        L.sam3cu_vit_create_from_sam3.argtypes = [vp, C.c_size_t, vp, i32, i32, C.POINTER(C.c_int)]
        L.sam3cu_vit_get_config.argtypes = [vp, vp]
        L.sam3cu_neck_create.restype = vp
        L.sam3cu_neck_create.argtypes = [i32, i32, i32, i32, vp, vp, i32, i32, C.POINTER(C.c_int)]
        L.sam3cu_neck_out_size.argtypes = [vp, i32]
        L.sam3cu_neck_forward.argtypes = [vp, vp, i32, vp]
        L.sam3cu_neck_forward_async.argtypes = [vp, vp, i32, vp]
        L.sam3cu_neck_stream.restype = vp
        L.sam3cu_neck_stream.argtypes = [vp]
        L.sam3cu_neck_destroy.argtypes = [vp]
        L.sam3cu_sam3_check.argtypes = [vp, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
        L.sam3cu_sam3_find.argtypes = [vp, C.c_size_t, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                       C.POINTER(C.c_int), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
        L.sam3cu_vit_encode.argtypes = [vp, vp, i32, vp, i32]
        L.sam3cu_vit_encode_async.argtypes = [vp, vp, i32, vp]
        L.sam3cu_vit_stream.restype = vp
        L.sam3cu_vit_stream.argtypes = [vp]
        L.sam3cu_vit_launches_per_encode.argtypes = [vp, i32]
        L.sam3cu_conv2d_nhwc_noalloc.argtypes = [vp, vp, vp, vp] + [i32] * 10 + [vp]
        L.sam3cu_vit_profile.argtypes = [vp, vp, i32, vp, C.POINTER(C.c_double), C.POINTER(C.c_int)]
        L.sam3cu_vit_profile_detail.argtypes = [vp, vp, i32, vp, C.POINTER(C.c_double), C.POINTER(C.c_int)]
        L.sam3cu_tvit_expand_bias.argtypes = [vp, i32, i32, i32, vp, i32]
        L.sam3cu_tvit_window_attention.argtypes = [vp, i64, vp, i64, i32, i32, i32, i32, i32, vp, i32,
                                                   vp]
        L.sam3cu_tvit_block_create.restype = vp
        L.sam3cu_tvit_block_create.argtypes = [i32, i32, i32, i32, i32, vp, C.POINTER(C.c_int)]
        L.sam3cu_tvit_block_forward.argtypes = [vp, vp, i32, i32, i32, vp]
        L.sam3cu_tvit_block_destroy.argtypes = [vp]
        L.sam3cu_tvit_mbconv_create.restype = vp
        L.sam3cu_tvit_mbconv_create.argtypes = [i32, i32, i32, vp, C.POINTER(C.c_int)]
        L.sam3cu_tvit_mbconv_forward.argtypes = [vp, vp, i32, i32, i32, vp]
        L.sam3cu_tvit_mbconv_destroy.argtypes = [vp]
        L.sam3cu_selftest_wait_timeout.argtypes = [C.c_ulonglong, C.POINTER(C.c_int)]
        L.sam3cu_tinyvit_create.restype = vp
        L.sam3cu_tinyvit_create.argtypes = [vp, vp, i32, i32, C.POINTER(C.c_int)]
        L.sam3cu_tinyvit_encode.argtypes = [vp, vp, i32, vp, i32]
        L.sam3cu_tinyvit_grid.argtypes = [vp]
        L.sam3cu_tinyvit_destroy.argtypes = [vp]
        _lib = L
    return _lib


def backend_ops() -> int:
    """Address of the struct sam3_backend_ops of the CUDA backend."""
    f = lib().sam3_cuda_backend_ops
    f.restype = C.c_void_p
    return f()


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().sam3cu_strerror(rc).decode()
        raise Sam3cuError(f"{what}: {msg} ({rc})")


def init(device: int = 0) -> None:
    check(lib().sam3cu_init(device), "sam3cu_init")


def device_error() -> int:
    return lib().sam3cu_last_device_error()


def launch_count(reset: bool = False) -> int:
    return lib().sam3cu_launch_count(1 if reset else 0)


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _f32(t, what):
    """bias / residual / gamma / beta must be contiguous float32 device tensors."""
    import torch
    if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or not t.is_cuda):
        raise TypeError(f"{what} must be a contiguous float32 CUDA tensor")
    return _ptr(t)


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


_TORCH_CODE = None


def dtype_code(t) -> int:
    import torch
    return {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}[t.dtype]


# ------------------------------------------------------------------ ops
def linear(x, w, bias=None, residual=None, act=ACT_NONE, out_dtype=None, out=None):
    """y = act(x . w^T + bias) + residual (cuda tensors; x, w 16-bit)."""
    import torch
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or x.dtype, device=x.device)
    check(lib().sam3cu_linear(_ptr(x), dtype_code(x), _ptr(w), _f32(bias, 'bias'), _f32(residual, 'residual'),
                              _ptr(out), dtype_code(out), M, K, N, act, _stream()), "sam3cu_linear")
    return out


def q8_repack(blocks, N: int, K: int):
    """Reference Q8_0 blocks (uint8 cuda tensor, 36 B each) -> (q, scales)."""
    import torch
    q = torch.empty((N, K), dtype=torch.int8, device=blocks.device)
    sc = torch.empty((K // 32, N), dtype=torch.float32, device=blocks.device)
    check(lib().sam3cu_q8_repack(_ptr(blocks), N, K, _ptr(q), _ptr(sc), _stream()), "q8_repack")
    return q, sc


def q8_quantize(src):
    import torch
    n = src.numel()
    blocks = torch.empty(((n + 31) // 32) * 36, dtype=torch.uint8, device=src.device)
    check(lib().sam3cu_q8_quantize(_ptr(src), _ptr(blocks), n, _stream()), "q8_quantize")
    return blocks


def linear_q8(x, q, scales, bias=None, residual=None, act=ACT_NONE, out_dtype=None, out=None):
    import torch
    M, K = x.shape
    N = q.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or x.dtype, device=x.device)
    check(lib().sam3cu_linear_q8(_ptr(x), dtype_code(x), _ptr(q), _ptr(scales), _ptr(bias),
                                 _ptr(residual), _ptr(out), dtype_code(out), M, K, N, act,
                                 _stream()), "sam3cu_linear_q8")
    return out


def layernorm(x, gamma=None, beta=None, out_dtype=None, out=None):
    import torch
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    check(lib().sam3cu_layernorm(_ptr(x), dtype_code(x), _f32(gamma, 'gamma'), _f32(beta, 'beta'), _ptr(out),
                                 dtype_code(out), rows, cols, _stream()), "sam3cu_layernorm")
    return out


def sdpa_packed(qkv, n_groups: int, seq: int, heads: int, head_dim: int = 64, out=None):
    """Attention over a fused [rows, 3*E] Q|K|V buffer -> [rows, E]."""
    import torch
    rows, three_e = qkv.shape
    E = three_e // 3
    if out is None:
        out = torch.empty((rows, E), dtype=qkv.dtype, device=qkv.device)
    base = qkv.data_ptr()
    es = qkv.element_size()
    check(lib().sam3cu_sdpa(base, base + E * es, base + 2 * E * es, three_e, _ptr(out), E,
                            dtype_code(qkv), n_groups, seq, heads, head_dim, _stream()), "sam3cu_sdpa")
    return out


def conv2d_nhwc_noalloc(x, w, bias=None, stride=1, pad=0, out=None):
    """CONV2D (NHWC x OHWI, groups 1) through the entry point that allocates
    no device memory (its column buffer is a static device array)."""
    import torch
    if x.dim() != 4 or w.dim() != 4:
        raise ValueError("x must be NHWC [n,H,W,C] and w OHWI [OC,kh,kw,C]")
    n, H, W, C = x.shape
    OC, kh, kw, C2 = w.shape
    if C != C2:
        raise ValueError(f"channel mismatch: x has {C}, w has {C2}")
    if w.dtype != x.dtype:
        raise TypeError(f"w dtype {w.dtype} differs from x dtype {x.dtype}")
    if not (x.is_contiguous() and w.is_contiguous()):
        raise ValueError("x and w must be contiguous")
    OH, OW = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    if out is None:
        out = torch.empty((n, OH, OW, OC), dtype=x.dtype, device=x.device)
    elif tuple(out.shape) != (n, OH, OW, OC) or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {x.dtype} tensor of shape {(n, OH, OW, OC)}")
    check(lib().sam3cu_conv2d_nhwc_noalloc(_ptr(x), _ptr(w), _f32(bias, 'bias'), _ptr(out),
                                           dtype_code(x), n, H, W, C, OC, kh, kw, stride, pad,
                                           _stream()), "sam3cu_conv2d_nhwc_noalloc")
    return out


# ------------------------------------------------------------------ ViT
def _map_file(path) -> np.ndarray:
    """A read-only uint8 view of a file (np.memmap), or of a bytes-like."""
    if isinstance(path, (bytes, bytearray, memoryview, np.ndarray)):
        return np.frombuffer(path, np.uint8) if not isinstance(path, np.ndarray) else path.view(np.uint8)
    return np.memmap(path, np.uint8, mode="r")


def sam3_check(path) -> tuple:
    """sam3_weight_open's validation of a .sam3 image: (n_tensors, version)."""
    image = _map_file(path)
    n, v = C.c_uint32(0), C.c_uint32(0)
    check(lib().sam3cu_sam3_check(image.ctypes.data, image.nbytes, C.byref(n), C.byref(v)),
          "sam3cu_sam3_check")
    return n.value, v.value


def sam3_find(path, name: str) -> Optional[dict]:
    """sam3_weight_find on a .sam3 image: dtype, dims, byte offset from the
    start of the file and byte size; None if the tensor is absent."""
    image = _map_file(path)
    dt, nd, off, nb = C.c_int(0), C.c_int(0), C.c_uint64(0), C.c_uint64(0)
    dims = (C.c_int * 4)()
    rc = lib().sam3cu_sam3_find(image.ctypes.data, image.nbytes, name.encode(), C.byref(dt), C.byref(nd),
                                dims, C.byref(off), C.byref(nb))
    if rc == ENOENT:
        return None
    check(rc, "sam3cu_sam3_find")
    return dict(dtype=dt.value, dims=tuple(dims[i] for i in range(nd.value)), offset=off.value,
                nbytes=nb.value)


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("img_size", "patch_size", "embed_dim", "depth",
                                       "n_heads", "window_size", "mlp_dim")]


BLOCK_KEYS = ("ln1_w", "ln1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ln2_w", "ln2_b",
              "fc1_w", "fc1_b", "fc2_w", "fc2_b")


class _Blk(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in BLOCK_KEYS]


class _W(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("patch_w", "patch_b", "pos_raw", "ln_pre_w",
                                          "ln_pre_b")] + [("blocks", _Blk * 32)]


CFG_KEYS = ("img_size", "patch_size", "embed_dim", "depth", "n_heads", "window_size", "mlp_dim")


class VitEncoder:
    """sam3_vit_init + sam3_vit_load + sam3_vit_build on one B200.

    ``weights`` is a dict of host float32 numpy arrays in the reference
    layouts (see sam3cu_vit_weights); ``weight_dtype`` is BF16, F16 or Q8_0.
    """

    def __init__(self, cfg: dict, weights: dict, weight_dtype: int = BF16, max_batch: int = 1):
        self.cfg = dict(cfg)
        c = _Cfg(*(cfg[k] for k in CFG_KEYS))
        w = _W()
        keep = []

        def put(obj, name, arr):
            a = np.ascontiguousarray(arr, np.float32)
            keep.append(a)
            setattr(obj, name, a.ctypes.data)

        for n in ("patch_w", "patch_b", "pos_raw", "ln_pre_w", "ln_pre_b"):
            put(w, n, weights[n])
        for i, blk in enumerate(weights["blocks"]):
            for n in BLOCK_KEYS:
                put(w.blocks[i], n, blk[n])
        st = C.c_int(0)
        h = lib().sam3cu_vit_create(C.byref(c), C.byref(w), weight_dtype, max_batch, C.byref(st))
        del keep
        if not h:
            check(st.value or -1, "sam3cu_vit_create")
        self.h = h
        self.max_batch = max_batch
        gs = cfg["img_size"] // cfg["patch_size"]
        self.np = gs * gs

    @classmethod
    def from_sam3(cls, path, cfg: Optional[dict] = None, weight_dtype: int = BF16,
                  max_batch: int = 1) -> "VitEncoder":
        """sam3_weight_open + sam3_vit_load from a .sam3 file: the file is
        memory-mapped and its tensors go to the device as stored (Q8_0
        blocks repacked there, never requantised).  cfg None: the encoder
        shape is read from the file."""
        image = _map_file(path)
        st = C.c_int(0)
        c = C.byref(_Cfg(*(cfg[k] for k in CFG_KEYS))) if cfg is not None else None
        h = lib().sam3cu_vit_create_from_sam3(image.ctypes.data, image.nbytes, c, weight_dtype,
                                              max_batch, C.byref(st))
        del image
        if not h:
            check(st.value or -1, "sam3cu_vit_create_from_sam3")
        self = cls.__new__(cls)
        self.h = h
        got = _Cfg()
        check(lib().sam3cu_vit_get_config(h, C.byref(got)), "sam3cu_vit_get_config")
        self.cfg = {k: getattr(got, k) for k in CFG_KEYS}
        self.max_batch = max_batch
        gs = self.cfg["img_size"] // self.cfg["patch_size"]
        self.np = gs * gs
        return self

    def close(self):
        if self.h:
            lib().sam3cu_vit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().sam3cu_vit_stream(self.h)

    def launches_per_encode(self, n: int) -> int:
        return lib().sam3cu_vit_launches_per_encode(self.h, n)

    def encode_host(self, images: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
        """Host in, host out: [n,3,img,img] f32 -> [n, np, e] f32."""
        images = np.ascontiguousarray(images, np.float32)
        n = images.shape[0]
        if out is None:
            out = np.empty((n, self.np, self.cfg["embed_dim"]), np.float32)
        check(lib().sam3cu_vit_encode(self.h, images.ctypes.data, n, out.ctypes.data, 0),
              "sam3cu_vit_encode")
        return out

    def encode_ptr(self, images_ptr: int, n: int, out_ptr: int, on_device: bool) -> None:
        check(lib().sam3cu_vit_encode(self.h, images_ptr, n, out_ptr, 1 if on_device else 0),
              "sam3cu_vit_encode")

    def profile(self, images, out) -> dict:
        """One direct-launch encode with an event after every launch: device
        ms and launch count per kernel kind (device tensors in/out)."""
        ms = (C.c_double * 4)()
        cnt = (C.c_int * 4)()
        check(lib().sam3cu_vit_profile(self.h, images.data_ptr(), images.shape[0], out.data_ptr(),
                                       ms, cnt), "sam3cu_vit_profile")
        return {k: (ms[i], cnt[i]) for i, k in enumerate(PROFILE_KINDS)}

    def profile_detail(self, images, out) -> dict:
        """As profile(), per PROFILE_DETAIL_KINDS (each linear, the Q8_0
        dequantisation, window / global attention, LayerNorm, other)."""
        ms = (C.c_double * len(PROFILE_DETAIL_KINDS))()
        cnt = (C.c_int * len(PROFILE_DETAIL_KINDS))()
        check(lib().sam3cu_vit_profile_detail(self.h, images.data_ptr(), images.shape[0], out.data_ptr(),
                                              ms, cnt), "sam3cu_vit_profile_detail")
        return {k: (ms[i], cnt[i]) for i, k in enumerate(PROFILE_DETAIL_KINDS)}

    def encode_async(self, images, out) -> None:
        """Device tensors; enqueue on the encoder's stream, no wait."""
        check(lib().sam3cu_vit_encode_async(self.h, images.data_ptr(), images.shape[0],
                                            out.data_ptr()), "sam3cu_vit_encode_async")


# ---------------------------------------------------------------- TinyViT
def tvit_expand_bias(compact, ws: int, ld: int = 0):
    """Host expansion of a compact [heads, ws*ws] TinyViT bias table into a
    dense float32 numpy array [heads, ws*ws, ld] (ld rounded up to a
    multiple of 4 by default, as the attention kernel needs)."""
    import numpy as np
    compact = np.ascontiguousarray(compact, np.float32)
    heads, n_off = compact.shape
    n = ws * ws
    ld = ld or (n + 3) // 4 * 4
    out = np.empty((heads, n, ld), np.float32)
    check(lib().sam3cu_tvit_expand_bias(compact.ctypes.data, heads, n_off, ws, out.ctypes.data, ld),
          "sam3cu_tvit_expand_bias")
    return out


def tvit_window_attention(qkv, n_windows: int, n_tokens: int, heads: int, head_dim: int,
                          bias=None, out=None):
    """TinyViT window attention on a per-head interleaved [T, 3*C] qkv
    device tensor; bias: float32 device tensor [heads, n_tokens, ld]."""
    import torch
    rows, ld_qkv = qkv.shape
    C_ = heads * head_dim
    if out is None:
        out = torch.empty((rows, C_), dtype=qkv.dtype, device=qkv.device)
    bias_ld = 0
    if bias is not None:
        _f32(bias, "bias")
        bias_ld = bias.shape[-1]
    check(lib().sam3cu_tvit_window_attention(qkv.data_ptr(), ld_qkv, out.data_ptr(), out.shape[1],
                                             dtype_code(qkv), n_windows, n_tokens, heads, head_dim,
                                             _ptr(bias), bias_ld, _stream()),
          "sam3cu_tvit_window_attention")
    return out


class _TvitBlockW(C.Structure):
    """struct sam3cu_tvit_block_weights (include/sam3cu.h)."""
    _fields_ = ([(n, C.c_void_p) for n in ("attn_norm_w", "attn_norm_b", "qkv_w", "qkv_b", "proj_w",
                                           "proj_b", "attn_bias")]
                + [("attn_bias_offsets", C.c_int)]
                + [(n, C.c_void_p) for n in ("lc_w", "lc_b", "lc_bn_w", "lc_bn_b", "lc_bn_mean",
                                             "lc_bn_var", "mlp_norm_w", "mlp_norm_b", "fc1_w",
                                             "fc1_b", "fc2_w", "fc2_b")])


class _TvitMbW(C.Structure):
    """struct sam3cu_tvit_mbconv_weights (include/sam3cu.h)."""
    _fields_ = [(f"{c}{i}_{k}" if c == "bn" else f"conv{i}_{k}", C.c_void_p)
                for i in (1, 2, 3) for c, ks in (("conv", ("w", "b")), ("bn", ("w", "b", "mean", "var")))
                for k in ks]


def _fill(struct, w: dict, keep: list):
    import numpy as np
    for name, ctype in struct._fields_:
        if ctype is not C.c_void_p:
            continue
        a = w.get(name)
        if a is None:
            continue
        a = np.ascontiguousarray(a, np.float32)
        keep.append(a)
        setattr(struct, name, a.ctypes.data)


class TvitBlock:
    """One TinyViTBlock on device (sam3cu_tvit_block_*).  w: host float32
    arrays keyed as struct sam3cu_tvit_block_weights ('attn_bias' is the
    compact [heads, ws*ws] table)."""

    def __init__(self, dim, heads, ws, mlp_dim, w: dict, dtype=BF16):
        s = _TvitBlockW()
        keep = []
        _fill(s, w, keep)
        if w.get("attn_bias") is not None:
            s.attn_bias_offsets = int(w["attn_bias"].shape[-1])
        st = C.c_int(0)
        self._h = lib().sam3cu_tvit_block_create(dim, heads, ws, mlp_dim, dtype, C.byref(s), C.byref(st))
        del keep
        if not self._h:
            check(st.value or -1, "sam3cu_tvit_block_create")

    def forward(self, x):
        """x: float32 CUDA tensor [n_images, H, W, dim], updated in place."""
        n, H, W, _ = x.shape
        check(lib().sam3cu_tvit_block_forward(self._h, x.data_ptr(), n, H, W, _stream()),
              "sam3cu_tvit_block_forward")
        return x

    def close(self):
        if self._h:
            lib().sam3cu_tvit_block_destroy(self._h)
            self._h = None

    __del__ = close


class TvitMBConv:
    """One MBConv block on device (sam3cu_tvit_mbconv_*)."""

    def __init__(self, dim, mid_dim, w: dict, dtype=BF16):
        s = _TvitMbW()
        keep = []
        _fill(s, w, keep)
        st = C.c_int(0)
        self._h = lib().sam3cu_tvit_mbconv_create(dim, mid_dim, dtype, C.byref(s), C.byref(st))
        del keep
        if not self._h:
            check(st.value or -1, "sam3cu_tvit_mbconv_create")

    def forward(self, x):
        n, H, W, _ = x.shape
        check(lib().sam3cu_tvit_mbconv_forward(self._h, x.data_ptr(), n, H, W, _stream()),
              "sam3cu_tvit_mbconv_forward")
        return x

    def close(self):
        if self._h:
            lib().sam3cu_tvit_mbconv_destroy(self._h)
            self._h = None

    __del__ = close


def selftest_wait_timeout(limit_ns: int = 20_000_000) -> bool:
    """Run the bounded-wait failure path once; True when the wait gave up,
    recorded its error and returned (see sam3cu_selftest_wait_timeout)."""
    out = C.c_int(0)
    check(lib().sam3cu_selftest_wait_timeout(limit_ns, C.byref(out)), "sam3cu_selftest_wait_timeout")
    return out.value == 1


class TvitConvW(C.Structure):
    """struct sam3cu_tvit_conv_weights."""
    _fields_ = [(n, C.c_void_p) for n in ("w", "b", "bn_w", "bn_b", "bn_mean", "bn_var")]


class TinyvitCfg(C.Structure):
    """struct sam3cu_tinyvit_config."""
    _fields_ = [("img_size", C.c_int), ("n_layers", C.c_int), ("embed_dims", C.c_int * 4),
                ("depths", C.c_int * 4), ("num_heads", C.c_int * 4), ("window_sizes", C.c_int * 4),
                ("embed_dim", C.c_int), ("mlp_ratio", C.c_int)]


class TinyvitLayerW(C.Structure):
    """struct sam3cu_tinyvit_layer_weights."""
    _fields_ = [("conv_blocks", C.c_void_p), ("blocks", C.c_void_p), ("pm_conv1", TvitConvW),
                ("pm_conv2", TvitConvW), ("pm_conv3", TvitConvW)]


class TinyvitW(C.Structure):
    """struct sam3cu_tinyvit_weights."""
    _fields_ = [("patch_embed_0", TvitConvW), ("patch_embed_1", TvitConvW), ("layers", TinyvitLayerW * 4),
                ("proj_conv1", TvitConvW), ("proj_bn", TvitConvW), ("proj_conv2", TvitConvW)]


def tinyvit_structs(cfg: dict, w: dict):
    """ctypes config and weight tree for a TinyViT weight dict (see
    synth.tinyvit_weights); returns (cfg_struct, weights_struct, keepalive)."""
    keep = []
    cs = TinyvitCfg()
    cs.img_size, cs.n_layers = cfg["img_size"], cfg["n_layers"]
    for k in ("embed_dims", "depths", "num_heads", "window_sizes"):
        getattr(cs, k)[:] = list(cfg[k]) + [0] * (4 - len(cfg[k]))
    cs.embed_dim, cs.mlp_ratio = cfg["embed_dim"], cfg["mlp_ratio"]
    ws = TinyvitW()
    for name in ("patch_embed_0", "patch_embed_1", "proj_conv1", "proj_bn", "proj_conv2"):
        _fill(getattr(ws, name), w[name], keep)
    for l, lw in enumerate(w["layers"]):
        L = ws.layers[l]
        if lw.get("conv_blocks"):
            arr = (_TvitMbW * len(lw["conv_blocks"]))()
            for i, d in enumerate(lw["conv_blocks"]):
                _fill(arr[i], d, keep)
            keep.append(arr)
            L.conv_blocks = C.addressof(arr)
        if lw.get("blocks"):
            arr = (_TvitBlockW * len(lw["blocks"]))()
            for i, d in enumerate(lw["blocks"]):
                _fill(arr[i], d, keep)
                arr[i].attn_bias_offsets = int(d["attn_bias"].shape[-1])
            keep.append(arr)
            L.blocks = C.addressof(arr)
        for name in ("pm_conv1", "pm_conv2", "pm_conv3"):
            if name in lw:
                _fill(getattr(L, name), lw[name], keep)
    return cs, ws, keep


class TinyViT:
    """The TinyViT backbone on device (sam3cu_tinyvit_*)."""

    def __init__(self, cfg: dict, w: dict, dtype=F16, max_batch=1):
        self.cfg = cfg
        cs, ws, keep = tinyvit_structs(cfg, w)
        st = C.c_int(0)
        self.h = lib().sam3cu_tinyvit_create(C.byref(cs), C.byref(ws), dtype, max_batch, C.byref(st))
        del keep
        if not self.h:
            check(st.value or -1, "sam3cu_tinyvit_create")
        self.grid = lib().sam3cu_tinyvit_grid(self.h)

    def encode_host(self, images):
        import numpy as np
        images = np.ascontiguousarray(images, np.float32)
        n = images.shape[0]
        out = np.empty((n, self.grid * self.grid, self.cfg["embed_dim"]), np.float32)
        check(lib().sam3cu_tinyvit_encode(self.h, images.ctypes.data, n, out.ctypes.data, 0),
              "sam3cu_tinyvit_encode")
        return out

    def encode_ptr(self, images_ptr: int, n: int, out_ptr: int, on_device: bool) -> None:
        check(lib().sam3cu_tinyvit_encode(self.h, images_ptr, n, out_ptr, 1 if on_device else 0),
              "sam3cu_tinyvit_encode")

    def close(self):
        if self.h:
            lib().sam3cu_tinyvit_destroy(self.h)
            self.h = None

    __del__ = close


# ---------------------------------------------------------------- FPN neck
class _NeckW(C.Structure):
    _fields_ = [("conv_w", (C.c_void_p * 4) * 4), ("conv_b", (C.c_void_p * 4) * 4)]


class FpnNeck:
    """sam3_neck_init + sam3_neck_build (necks.c) on one B200.  ``weights``:
    {"w": [[OHWI f32 per layer] per stage], "b": [[bias f32] per stage]} in
    the reference's build order; dtype BF16 or F16 (compute type)."""

    def __init__(self, d_model: int, dim: int, grid: int, scales, weights: dict, dtype: int = BF16,
                 max_batch: int = 1):
        self.scales = list(scales)
        sc = np.ascontiguousarray(self.scales, np.float32)
        nw = _NeckW()
        keep = [sc]
        for i, (ws, bs) in enumerate(zip(weights["w"], weights["b"])):
            for j, (wa, ba) in enumerate(zip(ws, bs)):
                wa = np.ascontiguousarray(wa, np.float32)
                ba = np.ascontiguousarray(ba, np.float32)
                keep += [wa, ba]
                nw.conv_w[i][j] = wa.ctypes.data
                nw.conv_b[i][j] = ba.ctypes.data
        st = C.c_int(0)
        h = lib().sam3cu_neck_create(d_model, dim, grid, len(self.scales), sc.ctypes.data, C.byref(nw), dtype,
                                     max_batch, C.byref(st))
        del keep
        if not h:
            check(st.value or -1, "sam3cu_neck_create")
        self.h = h
        self.d_model, self.dim, self.grid = d_model, dim, grid
        self.sizes = [lib().sam3cu_neck_out_size(h, i) for i in range(len(self.scales))]

    @property
    def stream(self) -> int:
        return lib().sam3cu_neck_stream(self.h)

    def outputs(self, n: int, device):
        import torch
        return [torch.empty((n, s, s, self.d_model), dtype=torch.float32, device=device) for s in self.sizes]

    def forward(self, feat, outs=None, sync: bool = True):
        """feat: cuda f32 [n, grid*grid, dim] -> list of [n, H_i, H_i, d_model] f32."""
        n = feat.shape[0]
        if outs is None:
            outs = self.outputs(n, feat.device)
        ptrs = (C.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
        fn = lib().sam3cu_neck_forward if sync else lib().sam3cu_neck_forward_async
        check(fn(self.h, feat.data_ptr(), n, ptrs), "sam3cu_neck_forward")
        return outs

    def close(self):
        if self.h:
            lib().sam3cu_neck_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
